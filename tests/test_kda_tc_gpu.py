"""The fused tensor-core KDA forward (ptof_kda_fwd_exec) against the oracle's
kda_forward, itself pinned to the reference's kda_reference by a golden vector
(examples/attention/_kda_full.py:38-77; tests/test_oracle.py), at the bf16 tolerance
of the parity tests: outputs and final states, with and without an initial state,
with the reference's KDA gate distribution and with gates ten times stronger, and the
segment-chaining property of the final state."""
import numpy as np
import pytest
import torch

from oracle import gdn_oracle as orc

pytestmark = pytest.mark.gpu
TOL = 1e-2   # bf16 operands, fp32 accumulation


def _inputs(B, H, T, D=64, gscale=0.05, s0_std=None, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, H, T, D, device="cuda", generator=g), dim=-1).bfloat16()
    k = nrm(torch.randn(B, H, T, D, device="cuda", generator=g), dim=-1).bfloat16()
    v = torch.randn(B, H, T, D, device="cuda", generator=g).bfloat16()
    beta = torch.sigmoid(torch.randn(B, H, T, device="cuda", generator=g)).bfloat16()
    gg = -torch.rand(B, H, T, D, device="cuda", generator=g) * gscale
    S0 = None if s0_std is None else torch.randn(B, H, D, D, device="cuda", generator=g) * s0_std
    return q, k, v, beta, gg.contiguous(), S0


def _oracle(q, k, v, beta, g, S0, D=64):
    B, H, T, _ = q.shape
    f = lambda t: t.float().cpu().numpy()
    r = lambda t: f(t).reshape(B, H, T // 64, 64, *t.shape[3:])
    o, S = orc.kda_forward(r(q), r(k), r(v), r(beta), r(g), D ** -0.5,
                           S0=None if S0 is None else f(S0), return_state=True)
    return o.reshape(B, H, T, D), S


@pytest.mark.parametrize("B,H,T,gscale,s0", [(1, 2, 256, 0.05, None), (2, 3, 512, 0.05, 0.02),
                                             (1, 4, 1024, 0.5, None), (2, 2, 64, 0.05, 0.1)])
def test_kda_tc_matches_oracle(B, H, T, gscale, s0):
    from pto_fuser import KDAChunkForward
    q, k, v, beta, g, S0 = _inputs(B, H, T, gscale=gscale, s0_std=s0, seed=T + H)
    run = KDAChunkForward(B, H, T)
    o, S = run(q, k, v, beta, g, S0)
    run.check_status()
    ref_o, ref_S = _oracle(q, k, v, beta, g, S0)
    eo = orc.rel_l2(o.float().cpu().numpy(), ref_o)
    eS = orc.rel_l2(S.cpu().numpy(), ref_S)
    assert eo < TOL and eS < TOL, (eo, eS)
    run.close()


def test_kda_tc_chained_halves_and_determinism():
    from pto_fuser import KDAChunkForward
    B, H, T = 2, 4, 2048
    q, k, v, beta, g, _ = _inputs(B, H, T, seed=7)
    full = KDAChunkForward(B, H, T)
    o, S = full(q, k, v, beta, g)
    o2, S2 = full(q, k, v, beta, g)
    full.check_status()
    assert torch.equal(o, o2) and torch.equal(S, S2)
    h = T // 2
    half = KDAChunkForward(B, H, h)
    sl = lambda t, a, b: t[:, :, a:b].contiguous()
    oa, Sa = half(sl(q, 0, h), sl(k, 0, h), sl(v, 0, h), sl(beta, 0, h), sl(g, 0, h))
    ob, Sb = half(sl(q, h, T), sl(k, h, T), sl(v, h, T), sl(beta, h, T), sl(g, h, T), Sa)
    half.check_status()
    rel = lambda a, b: ((a.float() - b.float()).norm() / b.float().norm()).item()
    assert max(rel(oa, o[:, :, :h]), rel(ob, o[:, :, h:]), rel(Sb, S)) < 1e-5
    full.close()
    half.close()


def test_kda_tc_rejects_unsupported_shapes():
    import ctypes
    from pto_fuser import native as nv
    p = nv.GdnParams(1, 1, 128, 64, 128, 128, nv.BF16, nv.BF16, nv.BF16, nv.GATE_RAW,
                     nv.LAYOUT_BHTD, 0.1)
    assert not nv.lib().ptof_kda_fwd_setup(ctypes.byref(p))
    assert "Dk = Dv = 64" in nv.last_error()
