"""KDA (per-dimension gate) on the IR: the canonical program's structure and the
per-dimension resident-scan lowering (LowerPerDimScan) on CPU; the programs on CUDA
against the oracle's kda_forward (pinned to the reference's kda_reference in
tests/test_oracle.py) at the reference's gate (rel-L2 2e-2)."""
import pytest
import torch

from oracle import gdn_oracle as orc
from pto_fuser import FusedNode, OpaqueNode
from pto_fuser.forwards import build_kda_program, make_kda_inputs, prepare_kda_bindings
from pto_fuser.transforms import LowerPerDimScan, LowerResidentScan

B, H, NC, C, D = 1, 2, 4, 64, 64


def test_kda_program_and_perdim_scan_rewrite():
    prog = build_kda_program(B, H, NC, C, D, D ** -0.5)
    assert sum(isinstance(n, OpaqueNode) for n in prog.nodes) == 1
    assert LowerResidentScan(B, H, NC, C, D).match(prog) == 0   # GDN's scalar scan: no
    t = LowerPerDimScan(B, H, NC, C, D)
    assert t.match(prog) == 1
    res = t.apply(prog)
    assert res.changed and t.match(res.program) == 0
    scans = [n for n in res.program.nodes if isinstance(n, FusedNode)]
    assert len(scans) == 1 and scans[0].kernel == "chunk_h_scan"
    assert scans[0].params["perdim_decay"] is True
    assert not any(getattr(n, "output", "").startswith("WS0") for n in res.program.nodes)


@pytest.mark.gpu
@pytest.mark.parametrize("lower", [False, True])
def test_kda_programs_on_gpu(lower):
    from pto_fuser import StagedExecutor
    inp = make_kda_inputs(B, H, NC, C, D, device="cuda")
    binds = prepare_kda_bindings(**inp)
    prog = build_kda_program(B, H, NC, C, D, D ** -0.5)
    if lower:
        prog = LowerPerDimScan(B, H, NC, C, D).apply(prog).program
    o = StagedExecutor().run(prog, binds)["o"]
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy()
    ref = orc.kda_forward(f(inp["q"]), f(inp["k"]), f(inp["v"]), f(inp["beta"]),
                          f(inp["g_in"]), D ** -0.5)
    assert orc.rel_l2(f(o), ref) < 2e-2
