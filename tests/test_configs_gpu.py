"""Full-size checks of the BASELINE configurations (1-4) on the GPU.

The CPU oracle cannot run these sizes in seconds, so each test combines
* a size-independent property of the whole run:
  - GDN forward: one pass over the full sequence equals two chained passes, the
    second seeded with the first one's final state;
  - kkt + inverse: T (I + A) = I for every chunk, with A recomputed in fp32;
* an oracle check of whole (b, h) pairs at the full sequence length: every output
  token and the final state of the first and the last pair (the oracle walks one
  pair of 131,072 tokens in well under a minute), so rounding that accumulates
  over hundreds or thousands of chunks is pinned at the lengths the bench runs;
* and an oracle check of a prefix of the first heads (the forward is causal, so a
  prefix of the output depends only on that prefix of the inputs).
Inputs are drawn on the device with BASELINE's distributions (config 4 alone has
6 GB of activations).
"""
import numpy as np
import pytest
import torch

from oracle import gdn_oracle as orc

pytestmark = pytest.mark.gpu

TOL = 1e-2   # bf16 operands, fp32 accumulation


def _inputs(B, H, T, D, mu=2.0, s0_std=None, gated=True, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nrm = torch.nn.functional.normalize
    bf = torch.bfloat16
    q = nrm(torch.randn(B, H, T, D, device="cuda", generator=g), dim=-1).to(bf)
    k = nrm(torch.randn(B, H, T, D, device="cuda", generator=g), dim=-1).to(bf)
    v = torch.randn(B, H, T, D, device="cuda", generator=g).to(bf)
    beta = torch.sigmoid(torch.randn(B, H, T, device="cuda", generator=g)).to(bf)
    gg = torch.nn.functional.logsigmoid(torch.randn(B, H, T, device="cuda", generator=g) + mu)
    if not gated:
        gg = torch.zeros_like(gg)
    S0 = None
    if s0_std is not None:
        S0 = torch.randn(B, H, D, D, device="cuda", generator=g) * s0_std
    return q, k, v, beta, gg.contiguous(), S0


def _rel(a, b):
    a, b = a.float(), b.float()
    return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-30)).item()


def _full_length_pairs(q, k, v, beta, g, S0, o, S, D, gate, pairs):
    """Oracle (float64) on whole (b, h) pairs at the full length: rel-L2 of o and of
    the final state, per pair. Returns the worst of each."""
    B, H = q.shape[:2]
    worst_o = worst_S = 0.0
    for p in pairs:
        b, h = divmod(p, H)
        f = lambda t: t[b:b + 1, h:h + 1].float().cpu().numpy()
        s0 = None if S0 is None else f(S0)
        gs = None if gate == "none" else f(g)
        ref_o, ref_S = orc.gdn_forward(f(q), f(k), f(v), f(beta), gs, D ** -0.5, S0=s0,
                                       gate=gate)
        eo = orc.rel_l2(o[b:b + 1, h:h + 1].float().cpu().numpy(), ref_o)
        eS = orc.rel_l2(S[b:b + 1, h:h + 1].cpu().numpy(), ref_S)
        print(f"full-length pair {p} (T={q.shape[2]}): rel-L2 o {eo:.3e}  S_final {eS:.3e}")
        worst_o, worst_S = max(worst_o, eo), max(worst_S, eS)
    return worst_o, worst_S


def _forward_checks(B, H, T, D, mu=2.0, s0_std=None, gate="raw", heads=2, prefix=1024):
    from pto_fuser import GDNChunkForward
    q, k, v, beta, g, S0 = _inputs(B, H, T, D, mu=mu, s0_std=s0_std, gated=gate != "none")
    full = GDNChunkForward(B, H, T, D, D, gate=gate)
    o, S = full(q, k, v, beta, g, S0)
    full.check_status()
    assert torch.isfinite(o.float()).all() and torch.isfinite(S).all()
    # the oracle on whole pairs, every token and the final state
    e_o, e_S = _full_length_pairs(q, k, v, beta, g, S0, o, S, D, gate, (0, B * H - 1))
    assert e_o < TOL and e_S < TOL, (e_o, e_S)
    # two chained halves
    h = T // 2
    half = GDNChunkForward(B, H, h, D, D, gate=gate)
    sl = lambda t, a, b: t[:, :, a:b].contiguous()
    o1, S1 = half(sl(q, 0, h), sl(k, 0, h), sl(v, 0, h), sl(beta, 0, h), sl(g, 0, h), S0)
    o2, S2 = half(sl(q, h, T), sl(k, h, T), sl(v, h, T), sl(beta, h, T), sl(g, h, T), S1)
    half.check_status()
    e_chain = max(_rel(o1, o[:, :, :h]), _rel(o2, o[:, :, h:]), _rel(S2, S))
    assert e_chain < 1e-5, e_chain
    # oracle on the first heads and a prefix of the sequence
    f = lambda t: t[:1, :heads].float().cpu().numpy()
    qs, ks, vs = (f(t)[:, :, :prefix] for t in (q, k, v))
    bs, gs = f(beta)[:, :, :prefix], f(g)[:, :, :prefix]
    s0 = None if S0 is None else f(S0)
    ref_o, _ = orc.gdn_forward(qs, ks, vs, bs, gs, D ** -0.5, S0=s0, gate=gate)
    e_or = orc.rel_l2(o[:1, :heads, :prefix].float().cpu().numpy(), ref_o)
    assert e_or < TOL, e_or
    full.close()
    half.close()


def test_config2_full_size():
    """GDN forward, bf16, B4 H32 T16384 D128 (the bench workload)."""
    _forward_checks(4, 32, 16384, 128)


def test_config3_deltanet_full_size():
    """Ungated DeltaNet, bf16, B16 H16 T4096 D64."""
    _forward_checks(16, 16, 4096, 64, gate="none", heads=2, prefix=4096)


def test_config4_long_context_full_size():
    """Long context, bf16, B1 H64 T131072 D128, S0 ~ N(0, 0.02^2), g = logsigmoid(N(3,1))."""
    _forward_checks(1, 64, 131072, 128, mu=3.0, s0_std=0.02, heads=2, prefix=2048)


def test_config1_kkt_inv_full_size():
    """kkt + inverse alone, B8 H32 T8192 D128, fp32 T: T (I + A) = I on every chunk,
    and the oracle on the first chunks."""
    from pto_fuser import native as nv
    B, H, T, D, C = 8, 32, 8192, 128, 64
    q, k, v, beta, g, _ = _inputs(B, H, T, D)
    del q, v
    nc = T // C
    out = torch.empty(B, H, nc, C, C, device="cuda")
    ws = nv.lib().ptof_ws_setup()
    nv.check(nv.lib().ptof_kkt_inv_exec(ws, k.data_ptr(), beta.data_ptr(), g.data_ptr(),
                                        out.data_ptr(), B, H, T, D, nv.BF16, nv.BF16,
                                        nv.GATE_RAW, nv.LAYOUT_BHTD, nv.stream_handle()))
    nv.check(nv.lib().ptof_check_status(ws, nv.stream_handle()))
    nv.lib().ptof_ws_teardown(ws)
    assert torch.isfinite(out).all()
    # A in fp32 from the same bf16 inputs, chunk by chunk (the stage's definition)
    kc = k.float().view(B, H, nc, C, D)
    gc = g.view(B, H, nc, C).cumsum(-1)
    bc = beta.float().view(B, H, nc, C)
    eye = torch.eye(C, device="cuda")
    worst = 0.0
    for b in range(B):   # one batch row at a time bounds the temporary memory
        kk = kc[b] @ kc[b].transpose(-1, -2)
        dg = gc[b].unsqueeze(-1) - gc[b].unsqueeze(-2)
        coef = torch.where(dg <= 0, torch.exp(torch.clamp(dg, max=0.0)), torch.zeros_like(dg))
        A = torch.tril(kk * coef * bc[b].unsqueeze(-1), -1)
        resid = out[b] @ (eye + A) - eye
        worst = max(worst, (torch.linalg.matrix_norm(resid) / C ** 0.5).max().item())
    assert worst < TOL, worst
    # oracle on the first 16 chunks of head (0, 0)
    f = lambda t: t[:1, :1, :16 * C].float().cpu().numpy()
    _, Tref = orc.kkt_inv(f(k), f(beta), f(g))
    e = orc.rel_l2(out[:1, :1, :16].cpu().numpy(), Tref)
    assert e < TOL, e
