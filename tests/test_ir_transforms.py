"""Device-free structural tests of the IR, transforms, templates, cost model,
policy and the unverified compile driver (mirroring the reference's test_ir.py,
test_transform.py, test_template.py and test_compile.py)."""
import pytest
import torch

from pto_fuser import (CostModel, EinsumNode, Features, FusedNode, OpaqueNode, Policy, Program,
                       TensorOp, VecGlueNode, canonicalize, compile_program, epilogue_report)
from pto_fuser.forwards import build_deltanet_program, build_gdn_program
from pto_fuser.ir import node_outputs
from pto_fuser.template import FuseChunkOFlash, FuseContractionEpilogue
from pto_fuser.transforms import FuseGDNForward, LowerResidentScan

B, H, NC, C, D = 1, 4, 4, 64, 128


def _gdn():
    return build_gdn_program(B, H, NC, C, D, D ** -0.5)


def test_program_rejects_use_before_def():
    with pytest.raises(ValueError):
        Program(nodes=[VecGlueNode("add", ["a", "b"], "c")], inputs=["a"], outputs=["c"])


def test_program_rejects_missing_output():
    with pytest.raises(ValueError):
        Program(nodes=[VecGlueNode("add", ["a", "a"], "c")], inputs=["a"], outputs=["d"])


def test_fused_node_multi_output():
    n = FusedNode(kernel="chunk_h_scan", inputs=["w"], outputs=["h_out", "final"])
    assert node_outputs(n) == ["h_out", "final"] and n.output == "h_out"
    Program(nodes=[n], inputs=["w"], outputs=["h_out", "final"])


def test_gdn_program_shape():
    prog = _gdn()
    kinds = {}
    for n in prog.nodes:
        kinds[type(n).__name__] = kinds.get(type(n).__name__, 0) + 1
    assert kinds["OpaqueNode"] == 1 and prog.outputs == ["o"]
    assert kinds["EinsumNode"] == 6 + 2 * NC


def test_canonicalize_is_idempotent_and_nn():
    c1 = canonicalize(_gdn())
    c2 = canonicalize(c1)
    es = [n for n in c1.nodes if isinstance(n, EinsumNode)]
    assert all(n.read_mode == "NN" and not n.fuse_out for n in es)
    assert [str(n) for n in c1.nodes] == [str(n) for n in c2.nodes]


def test_fuse_gdn_forward_single_node():
    t = FuseGDNForward(B, H, NC, C, D)
    prog = _gdn()
    assert t.match(prog) == 1
    out = t.apply(prog).program
    assert len(out.nodes) == 1 and out.nodes[0].kernel == "gdn_chunk_fwd"
    assert out.nodes[0].params["scale"] == pytest.approx(D ** -0.5)
    assert t.match(out) == 0


def test_fuse_gdn_forward_not_on_deltanet():
    assert FuseGDNForward(B, H, NC, C, D).match(build_deltanet_program(B, H, NC, C, D, 0.1)) == 0


def test_resident_scan_rewrite():
    t = LowerResidentScan(B, H, NC, C, D)
    prog = canonicalize(_gdn())
    assert t.match(prog) == 1
    out = t.apply(prog).program
    kernels = [n.kernel for n in out.nodes if isinstance(n, FusedNode)]
    assert kernels == ["chunk_h_scan"]
    assert not any(n.output.startswith("WS0") for n in out.nodes)
    assert t.match(out) == 0


def test_templates_and_flash():
    prog = canonicalize(_gdn())
    rep = str(epilogue_report(prog))
    assert "template kkt-gated-native" in rep and "template chunk-o-gated-native" in rep
    flash = FuseChunkOFlash(B, H, NC, C, D)
    assert flash.match(prog) == 1
    prog2 = flash.apply(prog).program
    assert any(isinstance(n, FusedNode) and n.kernel == "qkv_flash_native_v2" for n in prog2.nodes)
    gen = FuseContractionEpilogue(B, H, NC, C, D, v2=True)
    prog3 = gen.apply(prog2).program
    ks = {n.kernel for n in prog3.nodes if isinstance(n, FusedNode)}
    assert ks == {"qkv_flash_native_v2", "kkt_gated_native_v2"}


UNCALIBRATED = CostModel(table={})   # every supported transform proposed (neutral seeds)


def test_cost_and_policy():
    f = Features(B, H, NC, C, D)
    cm = UNCALIBRATED
    assert cm.predict("fuse-gdn-forward", f).worth_trying
    assert not cm.predict("fuse-gdn-forward", Features(B, H, NC, 32, 128)).worth_trying
    assert not cm.predict("enable-direct-reads", f).worth_trying
    assert not cm.predict("unknown", f).worth_trying
    names = [p.name for p in Policy(cm).pipeline(canonicalize(_gdn()), f)]
    assert names[0] == "fuse-gdn-forward"
    assert names.index("lower-resident-scan") < names.index("fuse-contraction-epilogue")
    # the calibrated model (fitted from B200 measurements) still leads with the fused
    # forward and prunes what measured slower than the program without it (the chunk_o
    # keys at C = 128)
    calibrated = [p.name for p in Policy().pipeline(canonicalize(_gdn()), f)]
    assert calibrated[0] == "fuse-gdn-forward"
    big = Features(B, H, NC, 128, 128)
    if CostModel().table is not None:
        assert not CostModel().predict("fuse-chunk-o-flash", big).worth_trying
    assert f.M == B * H * NC and f.N == B * H and f.T == NC * C


def test_compile_unverified_whole_forward():
    res = compile_program(_gdn(), Features(B, H, NC, C, D), verify=False)
    assert [n.kernel for n in res.program.nodes] == ["gdn_chunk_fwd"]
    assert not res.report.verified and [r.name for r in res.report.kept] == ["fuse-gdn-forward"]
    assert "kept 1 of" in str(res.report)


def test_compile_unverified_partial_lowering():
    """With the whole-forward fusion not proposed (C=32), the partial fusions fire."""
    prog = build_gdn_program(B, H, NC, 32, D, D ** -0.5)
    res = compile_program(prog, Features(B, H, NC, 32, D), policy=Policy(UNCALIBRATED),
                          verify=False)
    ks = {n.kernel for n in res.program.nodes if isinstance(n, FusedNode)}
    assert ks == {"chunk_h_scan", "qkv_flash_native_v2", "kkt_gated_native_v2"}


def test_policy_and_compile_kda():
    """KDA: the per-dim scan and the epilogue generator (its qk_prologue template)
    apply, the scalar-decay scan and the whole-forward fusion do not (reference
    tests/test_compile.py:64-70); the per-dim flash runs before the generator and
    consumes the score, so the compiled kernel set is the reference's
    (tests/test_compile.py:91-97)."""
    from pto_fuser.forwards import build_kda_program
    prog = build_kda_program(1, 16, 8, 128, 128, 128 ** -0.5)
    f = Features(1, 16, 8, 128, 128)
    pol = Policy(UNCALIBRATED)
    names = [p.name for p in pol.pipeline(canonicalize(prog), f)]
    assert "lower-perdim-scan" in names and "fuse-contraction-epilogue" in names
    assert "lower-resident-scan" not in names and "fuse-gdn-forward" not in names
    res = compile_program(prog, f, policy=pol, verify=False)
    ks = {n.kernel for n in res.program.nodes if isinstance(n, FusedNode)}
    assert ks == {"chunk_h_scan", "qkvp_flash_native_v2"}
    # perdim scan + perdim flash (the generator then finds no score; the reference's two
    # read-mode levers are not proposed on B200)
    assert [r.name for r in res.report.kept] == ["lower-perdim-scan", "fuse-perdim-chunk-o-flash"]
    # without the flash, the generator's qk_prologue template takes the score
    from pto_fuser.template import FusePerDimChunkOFlash
    assert FusePerDimChunkOFlash(1, 16, 8, 128, 128).match(canonicalize(prog)) == 1


@pytest.mark.parametrize("per_dim", [False, True])
def test_policy_and_compile_chunked_linear(per_dim):
    """Chunked linear attention: batch-chunk-intra-score is proposed and lowers the
    per-chunk scores to one kernel (gated_qk_native_v2 for a scalar gate, qk_prologue
    for GLA's per-channel gate; C * d_k = 1024 -> the V1 prologue key)."""
    from pto_fuser.forwards.chunked import build_chunked_linear_program
    N, nc, C_, dk = 2, 4, 16, 64
    prog = build_chunked_linear_program(N, nc, C_, dk, dk)
    f = Features(1, N, nc, C_, dk, per_dim_gate=per_dim)
    names = [p.name for p in Policy().pipeline(canonicalize(prog), f)]
    assert "batch-chunk-intra-score" in names
    res = compile_program(prog, f, verify=False)
    ks = {n.kernel for n in res.program.nodes if isinstance(n, FusedNode)}
    assert ks == ({"qk_prologue"} if per_dim else {"gated_qk_native_v2"})
