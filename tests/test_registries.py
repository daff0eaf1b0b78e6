"""Device-free tests of the opaque and fused-kernel registries, capture mode and
the graph-replay guard (mirroring the reference's test_fusion.py / test_graph.py)."""
import pytest
import torch

from pto_fuser import (GraphReplayExecutor, OpaqueContract, OpaqueRegistry, capture_mode,
                       default_fused_registry, default_registry)
from pto_fuser import registry as reg
from pto_fuser.forwards import build_kkt_fused_program, build_scan_fused_program, build_scan_staged_program


def test_fused_registry_contracts():
    r = default_fused_registry()
    scan = r.contract("chunk_h_scan")
    assert scan.in_slots == ["w", "u", "k", "decay"] and scan.out_names == ["h_out", "final"]
    kkt = r.contract("kkt_gated")
    assert kkt.in_slots == ["k", "g_sum", "beta"] and kkt.out_names == ["L"]
    assert r.contract("gdn_chunk_fwd").out_names == ["o"]
    for key in ("kkt_gated_native", "kkt_gated_native_v2", "gated_qk_native", "gated_qk_native_v2",
                "qkv_flash_native", "qkv_flash_native_v2", "gated_qk"):
        assert key in r.keys()
    with pytest.raises(KeyError):
        r.kernel("nope", {})
    with pytest.raises(ValueError):
        r.register("chunk_h_scan", None)


def test_opaque_registry():
    r = default_registry()
    c = r.contract("tri_inv_rec_unroll")
    assert c.in_dtypes == [torch.float16] and c.out_dtype == torch.float32
    with pytest.raises(KeyError):
        r.run("nope", [], {})
    with pytest.raises(ValueError):
        r.register("tri_inv_rec_unroll", factory=lambda: None, lowering=lambda *a: None,
                   contract=OpaqueContract([], None))


def test_fused_programs():
    staged, fused = build_scan_staged_program(2, 4, 3), build_scan_fused_program(2, 4, 3)
    assert staged.inputs == fused.inputs and staged.outputs == fused.outputs
    assert len(staged.nodes) > len(fused.nodes) == 1
    assert build_kkt_fused_program(4, 8).outputs == ["L"]


def test_capture_mode_nesting_and_restore():
    assert reg._CAPTURE_MODE is False
    with capture_mode():
        with capture_mode():
            assert reg._CAPTURE_MODE
        assert reg._CAPTURE_MODE
    assert reg._CAPTURE_MODE is False
    with pytest.raises(RuntimeError):
        with capture_mode():
            raise RuntimeError("x")
    assert reg._CAPTURE_MODE is False


def test_replay_before_capture_raises():
    with pytest.raises(RuntimeError, match="capture"):
        GraphReplayExecutor().replay({})
