"""The CPU oracle pinned against golden vectors made by the reference's own code
(tests/golden/make_golden.py), plus its internal consistency properties."""
import os

import numpy as np
import pytest

from oracle import gdn_oracle as orc

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return dict(np.load(os.path.join(GOLD, name)))


def _bhtd(x):  # [B,H,nc,C,D] -> [B,H,T,D]
    B, H, nc, C = x.shape[:4]
    return x.reshape(B, H, nc * C, *x.shape[4:])


@pytest.mark.parametrize("name", ["gdn_d64.npz", "gdn_d128.npz"])
def test_gdn_forward_matches_reference(name):
    z = _load(name)
    o, _ = orc.gdn_forward(_bhtd(z["q"]), _bhtd(z["k"]), _bhtd(z["v"]), _bhtd(z["beta"]),
                           _bhtd(z["g_in"]), float(z["scale"]))
    assert orc.rel_l2(o, _bhtd(z["o"])) < 1e-5


def test_deltanet_matches_reference():
    z = _load("deltanet_d64.npz")
    out = orc.deltanet_forward(_bhtd(z["q"]), _bhtd(z["k"]), _bhtd(z["v"]), _bhtd(z["beta"]),
                               float(z["scale"]))
    for n in ("A", "T", "W", "U", "v_new", "h_state", "o"):
        assert orc.rel_l2(out[n], z[n]) < 1e-5, n


def test_deltanet_is_ungated_gdn():
    z = _load("deltanet_d64.npz")
    q, k, v, b = (_bhtd(z[n]) for n in ("q", "k", "v", "beta"))
    o, _ = orc.gdn_forward(q, k, v, b, None, float(z["scale"]), gate="none")
    assert orc.rel_l2(o, _bhtd(z["o"])) < 1e-5


def test_kkt_gated_matches_reference():
    z = _load("kkt_c128.npz")              # mega layout: k [1,T,H,D], g/beta [1,T,H]
    k, g, b = z["k"][0], z["g_sum"][0], z["beta"][0]
    T, H, D = k.shape
    C = 128
    kc = k.reshape(T // C, C, H, D).transpose(0, 2, 1, 3)           # [nc,H,C,D]
    gc = g.reshape(T // C, C, H).transpose(0, 2, 1)
    bc = b.reshape(T // C, C, H).transpose(0, 2, 1)
    L = orc.kkt_gated(kc, kc, gc, bc, causal=False)                   # [nc,H,C,C]
    ref = z["L"].reshape(T // C, C, H, C).transpose(0, 2, 1, 3)
    assert orc.rel_l2(L, ref) < 2e-3                                  # ref L is fp16


def test_chunk_h_scan_matches_reference():
    z = _load("scan_c128.npz")
    h, fin = orc.chunk_h_scan(z["w"], z["u"], z["k"], z["decay"])
    assert orc.rel_l2(h, z["h_out"]) < 1e-5
    assert orc.rel_l2(fin, z["final"]) < 1e-5


def test_tri_inv_is_inverse():
    rng = np.random.default_rng(0)
    A = np.tril(rng.standard_normal((5, 64, 64)) * 0.1, -1)
    T = orc.tri_inv(A)
    eye = np.eye(64)
    assert np.abs((eye + A) @ T - eye).max() < 1e-10


def test_final_state_chains_segments():
    """Running two halves with S0 = the first half's final state reproduces the
    whole sequence: pins the final-state / S0 restatement the reference lacks."""
    rng = np.random.default_rng(1)
    B, H, T, D = 1, 2, 256, 32
    q = rng.standard_normal((B, H, T, D)); q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = rng.standard_normal((B, H, T, D)); k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, H, T, D))
    b = 1 / (1 + np.exp(-rng.standard_normal((B, H, T))))
    g = -np.log1p(np.exp(-(rng.standard_normal((B, H, T)) + 2)))
    o, S = orc.gdn_forward(q, k, v, b, g, 0.1)
    h = T // 2
    o1, S1 = orc.gdn_forward(q[:, :, :h], k[:, :, :h], v[:, :, :h], b[:, :, :h], g[:, :, :h], 0.1)
    o2, S2 = orc.gdn_forward(q[:, :, h:], k[:, :, h:], v[:, :, h:], b[:, :, h:], g[:, :, h:], 0.1,
                             S0=S1)
    assert orc.rel_l2(np.concatenate([o1, o2], axis=2), o) < 1e-12
    assert orc.rel_l2(S2, S) < 1e-12


def test_qkv_flash_matches_gdn_intra_term():
    """With W = U = 0 contributions removed (S = 0, one chunk), o = scale*intra."""
    rng = np.random.default_rng(2)
    q = rng.standard_normal((1, 1, 64, 16)); k = rng.standard_normal((1, 1, 64, 16))
    v = rng.standard_normal((1, 1, 64, 16)); g = -np.abs(rng.standard_normal((1, 1, 64))) * 0.1
    gs = orc.chunk_cumsum(g)
    intra = orc.qkv_flash(q.reshape(1, 1, 1, 64, 16), k.reshape(1, 1, 1, 64, 16),
                          v.reshape(1, 1, 1, 64, 16), gs)
    ref = np.einsum("ij,je->ie", np.tril((q[0, 0] @ k[0, 0].T)
                                          * np.exp(np.minimum(gs[0, 0, 0][:, None] - gs[0, 0, 0][None, :], 0))),
                    v[0, 0])
    assert orc.rel_l2(intra[0, 0, 0], ref) < 1e-12


def test_varlen_oracle_reduces_to_fixed_length():
    """gdn_forward_varlen on equal-length sequences with Hg = H equals gdn_forward, and
    padding a sequence to whole chunks leaves its outputs unchanged."""
    rng = np.random.default_rng(5)
    N, H, T, D = 2, 2, 128, 16
    q = rng.standard_normal((N, H, T, D)); k = rng.standard_normal((N, H, T, D))
    v = rng.standard_normal((N, H, T, D))
    beta = 1 / (1 + np.exp(-rng.standard_normal((N, H, T))))
    g = -np.log1p(np.exp(-(rng.standard_normal((N, H, T)) + 2)))
    o, S = orc.gdn_forward(q, k, v, beta, g, 0.25)
    pk = lambda x: x.transpose(0, 2, 1, *range(3, x.ndim)).reshape(N * T, H, *x.shape[3:])
    ov, Sv = orc.gdn_forward_varlen(pk(q), pk(k), pk(v), pk(beta), pk(g), [0, T, 2 * T], 0.25)
    assert np.allclose(ov, pk(o)) and np.allclose(Sv, S)
    # a 100-token prefix of the first sequence: padded inside the oracle
    ov2, _ = orc.gdn_forward_varlen(pk(q)[:100], pk(k)[:100], pk(v)[:100], pk(beta)[:100],
                                    pk(g)[:100], [0, 100], 0.25)
    o_pref, _ = orc.gdn_forward(q[:1, :, :128], k[:1, :, :128], v[:1, :, :128],
                                np.where(np.arange(128) < 100, beta[:1], 0.0),
                                np.where(np.arange(128) < 100, g[:1], 0.0), 0.25)
    assert np.allclose(ov2, o_pref[0].transpose(1, 0, 2)[:100])


def test_kda_oracle_matches_reference_golden():
    """kda_forward against the reference's own kda_reference (_kda_full.py:38-77)."""
    z = np.load(os.path.join(GOLD, "kda_d32.npz"))
    o = orc.kda_forward(z["q"], z["k"], z["v"], z["beta"], z["g_in"], 32 ** -0.5)
    assert orc.rel_l2(o, z["o"]) < 1e-5


def test_linear_attention_oracle_matches_reference_golden():
    """linear_attention_recurrent against the reference's chunked_linear_reference."""
    z = np.load(os.path.join(GOLD, "linear_gla.npz"))
    N, nc, C = z["q"].shape[:3]
    f = lambda x: x.reshape(N, nc * C, -1)
    o = orc.linear_attention_recurrent(f(z["q"]), f(z["k"]), f(z["v"]), f(z["gates"]))
    assert orc.rel_l2(o, f(z["o"])) < 1e-5
