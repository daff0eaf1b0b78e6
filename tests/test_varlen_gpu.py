"""Variable-length sequences with grouped query/key heads (ptof_gdn_fwd_varlen_*):
parity with the CPU oracle's gdn_forward_varlen on ragged lengths (partial last
chunks, a sequence shorter than one chunk, an empty one), GQA, initial states, and
the given-cumsum gate; plus equality with the fixed-length entry when every
sequence has the same length and Hg = H."""
import numpy as np
import pytest
import torch

from oracle import gdn_oracle as orc

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _inputs(lens, H, Hg, D, dtype=torch.bfloat16, mu=2.0, s0=None, seed=0):
    g = torch.Generator().manual_seed(seed)
    T = int(sum(lens))
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(T, Hg, D, generator=g), dim=-1)
    k = nrm(torch.randn(T, Hg, D, generator=g), dim=-1)
    v = torch.randn(T, H, D, generator=g)
    beta = torch.sigmoid(torch.randn(T, H, generator=g))
    gg = torch.nn.functional.logsigmoid(torch.randn(T, H, generator=g) + mu)
    S0 = torch.randn(len(lens), H, D, D, generator=g) * s0 if s0 else None
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    dev = lambda t, dt=dtype: t.to(device="cuda", dtype=dt).contiguous()
    return dict(q=dev(q), k=dev(k), v=dev(v), beta=dev(beta), g=dev(gg, torch.float32),
                S0=None if S0 is None else dev(S0, torch.float32), cu=dev(cu, torch.int32))


def _check(lens, H, Hg, D, gate="raw", s0=None, mu=2.0):
    from pto_fuser import GDNChunkForwardVarlen
    inp = _inputs(lens, H, Hg, D, mu=mu, s0=s0)
    T = int(sum(lens))
    g = inp["g"]
    if gate == "cumsum":   # chunk-local cumsum within each sequence's own chunks
        gc = g.clone()
        cu = inp["cu"].tolist()
        for a, b in zip(cu[:-1], cu[1:]):
            for c0 in range(a, b, 64):
                gc[c0:min(c0 + 64, b)] = g[c0:min(c0 + 64, b)].cumsum(0)
        g = gc.contiguous()
    r = GDNChunkForwardVarlen(len(lens), H, Hg, T, max(max(lens), 1), D, D, gate=gate)
    o, S = r(inp["q"], inp["k"], inp["v"], inp["beta"], g, inp["cu"], inp["S0"])
    torch.cuda.synchronize()
    r.check_status()
    f = lambda t: None if t is None else t.float().cpu().numpy()
    ref_o, ref_S = orc.gdn_forward_varlen(f(inp["q"]), f(inp["k"]), f(inp["v"]), f(inp["beta"]),
                                          f(g), inp["cu"].tolist(), D ** -0.5, S0=f(inp["S0"]),
                                          gate=gate)
    eo = orc.rel_l2(f(o), ref_o)
    eS = orc.rel_l2(f(S), ref_S)
    assert eo < TOL and eS < TOL, (eo, eS)
    r.close()


@pytest.mark.parametrize("D", [128, 64])
def test_varlen_ragged(D):
    _check([200, 64, 37, 130, 1], H=4, Hg=4, D=D)


def test_varlen_gqa_initial_state():
    _check([150, 256, 70], H=8, Hg=2, D=128, s0=0.02, mu=3.0)


def test_varlen_empty_sequence_and_cumsum_gate():
    _check([96, 0, 64, 129], H=2, Hg=1, D=128, gate="cumsum")


def test_varlen_equal_lengths_match_fixed_length_entry():
    from pto_fuser import GDNChunkForward, GDNChunkForwardVarlen
    N, H, T, D = 2, 4, 256, 128
    inp = _inputs([T] * N, H, H, D)
    to_bhtd = lambda t: t.view(N, T, *t.shape[1:]).transpose(1, 2).contiguous()
    fixed = GDNChunkForward(N, H, T, D, D)
    o_f, S_f = fixed(to_bhtd(inp["q"]), to_bhtd(inp["k"]), to_bhtd(inp["v"]),
                     to_bhtd(inp["beta"]), to_bhtd(inp["g"]))
    var = GDNChunkForwardVarlen(N, H, H, N * T, T, D, D)
    o_v, S_v = var(inp["q"], inp["k"], inp["v"], inp["beta"], inp["g"], inp["cu"])
    torch.cuda.synchronize()
    assert torch.equal(to_bhtd(o_v), o_f)
    assert torch.equal(S_v, S_f)
