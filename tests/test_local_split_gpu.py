"""The chunk-segment scan inside one GPU with a long head segment (GDNLocalSplit):
heads run from the true initial state, tail segments as A and B runs on strided views
of the caller's tensors, then seg_scan and the strided fix-up. Compared with the
serial fused forward (same kernels, one chain per pair) and with the oracle."""
import pytest
import torch

from oracle import gdn_oracle as orc

pytestmark = pytest.mark.gpu


def _inputs(P, T, D=128, s0=None, seed=0):
    from pto_fuser import make_gdn_inputs
    inp = make_gdn_inputs(1, P, T, D, dtype=torch.bfloat16, device="cuda", seed=seed,
                          s0_std=s0, mu=2.0)
    return {k: t[0] for k, t in inp.items()}


@pytest.mark.parametrize("P,T,L0,s,Ls,s0", [(4, 1024, 512, 2, 256, None),
                                            (3, 2048, 768, 5, 256, 0.02),
                                            (2, 4096, 1536, 1, 2560, None)])
def test_local_split_matches_serial_forward_and_oracle(P, T, L0, s, Ls, s0):
    from pto_fuser import GDNChunkForward
    from pto_fuser.segment import GDNLocalSplit
    inp = _inputs(P, T, s0=s0, seed=P + T)
    S0 = inp.get("S0")
    a = (inp["q"], inp["k"], inp["v"], inp["beta"], inp["g"])
    run = GDNLocalSplit(P, T, 128, L0, s, Ls)
    o, S = run(*a, S0)
    run.check_status()
    ser = GDNChunkForward(1, P, T, 128, 128)
    ref_o, ref_S = ser(*(t[None] for t in a), None if S0 is None else S0[None])
    ser.check_status()
    rel = lambda x, y: ((x.float() - y.float()).norm() / y.float().norm()).item()
    assert rel(o, ref_o[0]) < 5e-3 and rel(S, ref_S[0]) < 5e-3, (rel(o, ref_o[0]), rel(S, ref_S[0]))
    f = lambda t: t[None, :1].float().cpu().numpy()
    oo, So = orc.gdn_forward(f(inp["q"]), f(inp["k"]), f(inp["v"]), f(inp["beta"]), f(inp["g"]),
                             128 ** -0.5, S0=None if S0 is None else f(S0))
    assert orc.rel_l2(o[:1].float().cpu().numpy(), oo[0]) < 1e-2
    assert orc.rel_l2(S[:1].cpu().numpy(), So[0]) < 1e-2
    run.close()
    ser.close()


@pytest.mark.parametrize("P", [32, 16])
def test_bench_rank_plans_match_serial_forward_and_oracle(P):
    """The plans a strong-scaled config-2 rank runs (32 or 16 pairs of 16,384 tokens on
    148 SMs, from plan_local_split) against the serial forward and, on pair 0, the
    oracle at full length."""
    from pto_fuser import GDNChunkForward
    from pto_fuser.segment import GDNLocalSplit, plan_local_split
    T = 16384
    L0, s, Ls = plan_local_split(P, T, 148)
    inp = _inputs(P, T, seed=P)
    a = (inp["q"], inp["k"], inp["v"], inp["beta"], inp["g"])
    run = GDNLocalSplit(P, T, 128, L0, s, Ls)
    o, S = run(*a)
    run.check_status()
    ser = GDNChunkForward(1, P, T, 128, 128)
    ref_o, ref_S = ser(*(t[None] for t in a))
    ser.check_status()
    rel = lambda x, y: ((x.float() - y.float()).norm() / y.float().norm()).item()
    assert rel(o, ref_o[0]) < 5e-3 and rel(S, ref_S[0]) < 5e-3, (rel(o, ref_o[0]), rel(S, ref_S[0]))
    f = lambda t: t[None, :1].float().cpu().numpy()
    oo, So = orc.gdn_forward(f(inp["q"]), f(inp["k"]), f(inp["v"]), f(inp["beta"]), f(inp["g"]),
                             128 ** -0.5)
    assert orc.rel_l2(o[:1].float().cpu().numpy(), oo[0]) < 1e-2
    assert orc.rel_l2(S[:1].cpu().numpy(), So[0]) < 1e-2
    run.close()
    ser.close()
