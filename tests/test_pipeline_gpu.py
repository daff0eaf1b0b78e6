"""GPU tests of the API stack: the staged executor on the canonical programs, the
fused-node keys against their fp32 references, CUDA-graph replay, and the verified
compile driver (mirroring the reference's *_npu.py device tests)."""
import pytest
import torch

from pto_fuser import (CostModel, Features, Policy, FusedNode, GraphReplayExecutor, StagedExecutor,
                       compile_program, default_registry, frob_rel, gate_determinism,
                       shared_fused_registry)
from pto_fuser.forwards import (build_deltanet_program, build_gdn_program, build_kkt_fused_program,
                                build_scan_fused_program, build_scan_staged_program,
                                deltanet_reference, gdn_reference, kkt_reference, make_gdn_inputs,
                                make_inputs, make_kkt_inputs, make_scan_inputs,
                                prepare_gdn_bindings, scan_reference)
from pto_fuser.transforms import FuseGDNForward

pytestmark = pytest.mark.gpu
TOL = 2e-2   # the reference's staged-vs-fused gate (compile.py:50)


def _gdn_case(B=1, H=2, nc=4, C=64, D=128):
    inp = make_gdn_inputs(B, H, nc, C, D, device="cuda")
    scale = D ** -0.5
    ref = gdn_reference(inp["q"], inp["k"], inp["v"], inp["beta"], inp["g_in"], scale)
    binds = prepare_gdn_bindings(inp["q"], inp["k"], inp["v"], inp["beta"], inp["g_in"])
    return build_gdn_program(B, H, nc, C, D, scale), binds, ref


def test_staged_gdn_matches_reference():
    prog, binds, ref = _gdn_case()
    out = StagedExecutor().run(prog, binds)["o"]
    assert frob_rel(out, ref) < TOL


def test_fused_forward_node_matches_reference():
    prog, binds, ref = _gdn_case()
    fused = FuseGDNForward(1, 2, 4, 64, 128).apply(prog).program
    out = StagedExecutor().run(fused, binds)["o"]
    assert frob_rel(out, ref) < TOL


def test_partial_lowering_runs_compat_kernels():
    """C = 32: the whole-forward kernel does not apply; the resident scan, the
    gated kkt and the chunk_o flash keys run instead."""
    prog, binds, ref = _gdn_case(C=32)
    # every supported transform proposed (uncalibrated policy): this exercises the keys
    res = compile_program(prog, Features(1, 2, 4, 32, 128), policy=Policy(CostModel(table={})),
                          verify=False)
    kinds = {n.kernel for n in res.program.nodes if isinstance(n, FusedNode)}
    assert {"chunk_h_scan", "qkv_flash_native_v2"} <= kinds
    out = StagedExecutor().run(res.program, binds)["o"]
    assert frob_rel(out, ref) < TOL


def test_graph_replay_matches_eager_and_is_deterministic():
    prog, binds, ref = _gdn_case()
    fused = FuseGDNForward(1, 2, 4, 64, 128).apply(prog).program
    eager = StagedExecutor().run(fused, binds)["o"]
    gr = GraphReplayExecutor().capture(fused, binds)
    assert torch.equal(gr.replay(binds)["o"], eager)
    assert gate_determinism(lambda: gr.replay(binds)).passed
    with pytest.raises(ValueError):
        gr.replay({k: v[..., :1] if k == "qF" else v for k, v in binds.items()})


def test_compile_verified_keeps_whole_forward():
    prog, binds, ref = _gdn_case(B=1, H=4, nc=8)
    res = compile_program(prog, Features(1, 4, 8, 64, 128), bindings=binds, iters=5, warmup=2)
    kept = [r.name for r in res.report.kept]
    assert res.report.verified and kept == ["fuse-gdn-forward"], str(res.report)
    out = StagedExecutor().run(res.program, binds)["o"]
    assert frob_rel(out, ref) < TOL


def test_chunk_h_scan_key():
    inp = make_scan_inputs(1, 2, 3)
    ref = scan_reference(inp, 1, 2, 3)
    got = StagedExecutor().run(build_scan_fused_program(1, 2, 3), inp)
    staged = StagedExecutor().run(build_scan_staged_program(1, 2, 3), inp)
    for n in ("h_out", "final"):
        assert frob_rel(got[n], ref[n]) < 1e-2, n
        assert frob_rel(staged[n], ref[n]) < 2e-2, n


def test_kkt_gated_key():
    inp = make_kkt_inputs(2, 4)
    ref = kkt_reference(inp, 2, 4)["L"]
    got = StagedExecutor().run(build_kkt_fused_program(2, 4), inp)["L"]
    assert frob_rel(got, ref) < 2e-3


def test_tri_inv_opaque():
    M, C = 8, 64
    A = torch.tril(torch.randn(M, C, C, device="cuda") * 0.1, -1).half()
    T = default_registry().run("tri_inv_rec_unroll", [A], {})
    eye = torch.eye(C, device="cuda").expand(M, C, C)
    ref = torch.linalg.solve_triangular(eye + A.float(), eye, upper=False, unitriangular=True)
    assert frob_rel(T, ref) < 1e-5


def test_qkv_flash_key():
    M, C, D = 6, 64, 128
    q, k, v = (torch.randn(M, C, D, device="cuda").half() for _ in range(3))
    g = torch.nn.functional.logsigmoid(torch.randn(M, C, device="cuda")).cumsum(-1)
    ones = torch.ones(M, C, device="cuda").half()
    o = shared_fused_registry().run("qkv_flash_native_v2", [q, k, v, g, ones], {})[0]
    s = (q.float() @ k.float().transpose(-1, -2)) * torch.exp(
        torch.clamp(g[:, :, None] - g[:, None, :], max=0.0))
    ref = torch.tril(s) @ v.float()
    assert frob_rel(o, ref) < 1e-5


def test_deltanet_program_matches_reference():
    B, H, nc, C, D = 1, 2, 3, 64, 64
    inp = make_inputs(B, H, nc, C, D)
    prog = build_deltanet_program(B, H, nc, C, D, D ** -0.5)
    out = StagedExecutor().run(prog, inp)
    ref = deltanet_reference(inp["q"], inp["k"], inp["v"], inp["beta"], B, H, nc, C, D, D ** -0.5)
    for n in ("A", "T", "W", "U", "v_new", "h_state", "o"):
        assert frob_rel(out[n], ref[n]) < TOL, n
