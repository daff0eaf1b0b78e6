"""KDA (per-dimension gate) on the IR: the canonical program's structure and the
per-dimension resident-scan lowering (LowerPerDimScan) on CPU; the programs on CUDA
against the oracle's kda_forward (pinned to the reference's kda_reference in
tests/test_oracle.py) at the reference's gate (rel-L2 2e-2)."""
import pytest
import torch

from oracle import gdn_oracle as orc
from pto_fuser import FusedNode, OpaqueNode
from pto_fuser.forwards import build_kda_program, make_kda_inputs, prepare_kda_bindings
from pto_fuser.template import FuseContractionEpilogue
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


def test_kda_chunk_o_prologue_template():
    """The per-dim chunk_o score becomes one qk_prologue node (k-side mul absorbed,
    q-side kept for the inter-chunk term); kkt stays a plain einsum, as in the
    reference (transforms/kda.py:1-8)."""
    prog = build_kda_program(B, H, NC, C, D, D ** -0.5)
    t = FuseContractionEpilogue(B, H, NC, C, D)
    assert t.match(prog) == 1
    res = t.apply(prog)
    fused = [n for n in res.program.nodes if isinstance(n, FusedNode)]
    assert [n.kernel for n in fused] == ["qk_prologue_v2"]    # C * D = 4096: the v2 key
    assert fused[0].inputs == ["qF", "kF", "coef_ag", "coef_bg"]
    outs = {o for n in res.program.nodes for o in ([n.output] if hasattr(n, "output") else [])}
    assert "k_eff" not in outs and "q_eff" in outs and "Aqk" not in outs
    assert "Araw" in outs                                      # kkt left staged
    assert t.match(res.program) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("lower", ["none", "prologue", "flash"])
def test_kda_programs_on_gpu(lower):
    from pto_fuser import StagedExecutor
    from pto_fuser.template import FusePerDimChunkOFlash
    inp = make_kda_inputs(B, H, NC, C, D, device="cuda")
    binds = prepare_kda_bindings(**inp)
    prog = build_kda_program(B, H, NC, C, D, D ** -0.5)
    if lower != "none":
        prog = LowerPerDimScan(B, H, NC, C, D).apply(prog).program
        t = FuseContractionEpilogue if lower == "prologue" else FusePerDimChunkOFlash
        prog = t(B, H, NC, C, D).apply(prog).program
        want = "qk_prologue" if lower == "prologue" else "qkvp_flash_native"
        assert any(isinstance(n, FusedNode) and n.kernel.startswith(want) for n in prog.nodes)
    o = StagedExecutor().run(prog, binds)["o"]
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy()
    ref = orc.kda_forward(f(inp["q"]), f(inp["k"]), f(inp["v"]), f(inp["beta"]),
                          f(inp["g_in"]), D ** -0.5)
    assert orc.rel_l2(f(o), ref) < 2e-2


@pytest.mark.gpu
def test_kda_compile_verified_on_gpu():
    """compile_program on CUDA: the verifier times and checks each proposed transform
    (per-dim scan, qk_prologue template) and the compiled program still matches the
    oracle, whichever transforms it kept."""
    from pto_fuser import CostModel, Features, Policy, StagedExecutor, compile_program
    inp = make_kda_inputs(B, H, NC, C, D, device="cuda")
    binds = prepare_kda_bindings(**inp)
    prog = build_kda_program(B, H, NC, C, D, D ** -0.5)
    # every supported transform proposed (uncalibrated), so the verifier sees them all
    res = compile_program(prog, Features(B, H, NC, C, D), policy=Policy(CostModel(table={})),
                          bindings=binds, iters=5, warmup=2)
    assert res.report.verified
    assert {r.name for r in res.report.records} >= {"lower-perdim-scan",
                                                      "fuse-contraction-epilogue"}
    o = StagedExecutor().run(res.program, binds)["o"]
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy()
    ref = orc.kda_forward(f(inp["q"]), f(inp["k"]), f(inp["v"]), f(inp["beta"]),
                          f(inp["g_in"]), D ** -0.5)
    assert orc.rel_l2(f(o), ref) < 2e-2


@pytest.mark.gpu
@pytest.mark.parametrize("C_,D_,DV", [(64, 64, 64), (128, 128, 128), (32, 64, 96)])
def test_qkvp_flash_kernel(C_, D_, DV):
    """ptof_qkvp_flash_exec against a torch fp32 product on the same fp16 operands."""
    from pto_fuser.fused import default_fused_registry
    M = 6
    g = torch.Generator(device="cuda").manual_seed(C_ + D_)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g).half()
    q, k, v = r(M, C_, D_), r(M, C_, D_), r(M, C_, DV)
    ag = torch.exp(-torch.rand(M, C_, D_, device="cuda", generator=g)).half()
    bg = (1.0 / ag.float()).half()
    reg = default_fused_registry()
    o = reg.run("qkvp_flash_native_v2", [q, k, v, ag, bg],
                {"nc": M, "H": 1, "C": C_, "D": D_, "DV": DV})[0]
    s = (q.float() * ag.float()) @ (k.float() * bg.float()).transpose(1, 2)
    ref = torch.tril(s) @ v.float()
    torch.cuda.synchronize()
    assert orc.rel_l2(o.cpu().numpy(), ref.cpu().numpy()) < 1e-4
