"""Parity of the fused kkt + triangular-inverse kernel (BASELINE config 1's stage,
ptof_kkt_inv_exec) with the CPU oracle's kkt_inv, which restates
examples/attention/_gdn_full.py:73-78 and is pinned by tests/test_oracle.py."""
import numpy as np
import pytest
import torch

from oracle import gdn_oracle as orc

pytestmark = pytest.mark.gpu

TOL = 1e-2   # bf16 / fp16 inputs, fp32 accumulation


def _run(B, H, T, D, dtype=torch.bfloat16, gate="raw", layout="bhtd", mu=2.0, seed=0,
         beta_dtype=None):
    from pto_fuser import make_gdn_inputs, native as nv
    inp = make_gdn_inputs(B, H, T, D, dtype=dtype, device="cuda", mu=mu, seed=seed, layout=layout)
    k, beta, g = inp["k"], inp["beta"], inp["g"]
    if beta_dtype is not None:
        beta = beta.to(beta_dtype)
    gk = g
    if gate == "cumsum":
        gl = g if layout == "bhtd" else g.transpose(1, 2)
        gl = gl.reshape(B, H, T // 64, 64).cumsum(-1).reshape(B, H, T)
        gk = (gl if layout == "bhtd" else gl.transpose(1, 2)).contiguous()
    out = torch.full((B, H, T // 64, 64, 64), float("nan"), device="cuda")
    ws = nv.lib().ptof_ws_setup()
    gates = {"raw": nv.GATE_RAW, "cumsum": nv.GATE_CUMSUM, "none": nv.GATE_NONE}
    rc = nv.lib().ptof_kkt_inv_exec(
        ws, k.data_ptr(), beta.data_ptr(), gk.data_ptr(), out.data_ptr(), B, H, T, D,
        nv.dtype_code(dtype), nv.dtype_code(beta.dtype), gates[gate],
        nv.LAYOUT_BHTD if layout == "bhtd" else nv.LAYOUT_BTHD, nv.stream_handle())
    nv.check(rc)
    nv.check(nv.lib().ptof_check_status(ws, nv.stream_handle()))
    nv.lib().ptof_ws_teardown(ws)
    f = lambda t: t.float().cpu().numpy()
    kk, bb, gg = f(k), f(beta), f(g)
    if layout == "bthd":
        kk, bb, gg = kk.transpose(0, 2, 1, 3), bb.transpose(0, 2, 1), gg.transpose(0, 2, 1)
    _, Tref = orc.kkt_inv(kk, bb, gg, gate="raw" if gate != "none" else "none")
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    err = orc.rel_l2(got, Tref)
    assert err < TOL, err
    return err


@pytest.mark.parametrize("D", [128, 64])
def test_kkt_inv_bf16(D):
    _run(2, 4, 512, D)


@pytest.mark.parametrize("gate,layout", [("cumsum", "bhtd"), ("none", "bhtd"), ("raw", "bthd")])
def test_kkt_inv_gate_layout(gate, layout):
    _run(1, 3, 384, 128, gate=gate, layout=layout)


def test_kkt_inv_fp16_strong_decay_fp32_beta():
    _run(1, 2, 256, 128, dtype=torch.float16, mu=0.0, beta_dtype=torch.float32)


def test_kkt_inv_many_chunks_per_cta():
    """More chunks than CTAs (persistent loop, ring and TMEM buffer reuse)."""
    _run(4, 32, 2048, 128)   # 4096 chunks
