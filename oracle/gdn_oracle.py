"""CPU oracle for the chunked Gated DeltaNet forward — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline / reference arm) may
import it. The product path (``pto_fuser``) never calls into it.

It restates, in numpy, the reference's own fp32 torch algorithms (the reference
package is vloncar/pto-fuser; paths below are relative to that project):

  * ``gdn_forward``        examples/attention/_gdn_full.py:57-97 (``gdn_reference``),
                           plus the final state (the ``final`` convention of
                           src/pto_fuser/forwards/fused_stages.py:61) and an optional
                           initial state S0 (the reference hard-codes S=0 at :67);
  * ``deltanet_forward``   src/pto_fuser/forwards/deltanet.py:114-143;
  * ``kkt_gated``          src/pto_fuser/forwards/fused_stages.py:140-156;
  * ``chunk_h_scan``       src/pto_fuser/forwards/fused_stages.py:46-62;
  * ``tri_inv``            src/pto_fuser/registry.py:107-127 semantics, (I+A)^-1 for a
                           strictly-lower A (solve_triangular in _gdn_full.py:76-78);
  * ``qkv_flash``          src/pto_fuser/fused.py:368-387 semantics (chunk_o intra term);
  * ``segment_scan``       affine maps of token segments applied in order (no
                           counterpart in the reference; checked against gdn_forward
                           run serially).

Parity is pinned: tests/test_oracle.py checks every function here against golden
vectors produced by running the reference's own torch code
(tests/golden/make_golden.py, committed with the vectors).

Arithmetic is float64 by default (``dtype=np.float32`` reproduces fp32 rounding).
Chunk-parallel stages are vectorised over all chunks; the state scan loops over
chunks, vectorised over the (batch, head) pairs.
"""
from __future__ import annotations

import numpy as np

C_DEFAULT = 64


def _f(x, dtype):
    return np.asarray(x, dtype=dtype)


def chunk_cumsum(g, C=C_DEFAULT, dtype=np.float64):
    """Chunk-local inclusive prefix sum of the per-token log decay
    (_gdn_full.py:63 ``g_in.cumsum(dim=3)`` on the [B,H,nc,C] view)."""
    g = _f(g, dtype)
    B, H, T = g.shape
    return g.reshape(B, H, T // C, C).cumsum(axis=-1)


def tri_inv(A, dtype=np.float64):
    """(I + A)^-1 for strictly-lower A [..., C, C] by row-wise forward substitution
    (unit lower-triangular solve, _gdn_full.py:76-78; registry.py:107-127)."""
    A = _f(A, dtype)
    C = A.shape[-1]
    Tm = np.zeros_like(A)
    eye = np.eye(C, dtype=dtype)
    Tm[..., 0, :] = eye[0]
    for i in range(1, C):
        # row i of T: e_i - sum_{k<i} A[i,k] T[k,:]
        Tm[..., i, :] = eye[i] - np.einsum("...k,...kc->...c", A[..., i, :i], Tm[..., :i, :])
    return Tm


def _kkt_A(k, beta, gs, dtype):
    """A = tril((k k^T) * safe_exp(g_i - g_j) * beta_i, -1) per chunk (_gdn_full.py:73-75)."""
    C = k.shape[-2]
    kk = np.einsum("...id,...jd->...ij", k, k)
    x = gs[..., :, None] - gs[..., None, :]
    coef = np.where(x <= 0, np.exp(np.minimum(x, 0)), 0.0).astype(dtype)
    A = kk * coef * beta[..., :, None]
    return np.tril(A, -1)


def kkt_inv(k, beta, g, C=C_DEFAULT, gate="raw", dtype=np.float64):
    """The kkt + tri-inv stage alone: per chunk
    A = tril(beta KK^T exp(g_i - g_j), -1) and T = (I + A)^-1.

    k [B,H,T,D], beta [B,H,T], g [B,H,T] -> (A, T) each [B,H,nc,C,C]."""
    k = _f(k, dtype)
    B, H, T, D = k.shape
    nc = T // C
    kc = k.reshape(B, H, nc, C, D)
    bc = _f(beta, dtype).reshape(B, H, nc, C)
    gs = _gate(g, B, H, T, C, gate, dtype)
    A = _kkt_A(kc, bc, gs, dtype)
    return A, tri_inv(A, dtype)


def _gate(g, B, H, T, C, gate, dtype):
    if gate == "none" or g is None:
        return np.zeros((B, H, T // C, C), dtype=dtype)
    if gate == "cumsum":
        return _f(g, dtype).reshape(B, H, T // C, C)
    return chunk_cumsum(g, C, dtype)


def gdn_forward(q, k, v, beta, g, scale, S0=None, C=C_DEFAULT, gate="raw",
                dtype=np.float64):
    """Full GDN chunk forward, restating gdn_reference (_gdn_full.py:57-97).

    q,k [B,H,T,Dk], v [B,H,T,Dv], beta [B,H,T], g [B,H,T] (per-token log decay for
    gate="raw", the chunk-local cumsum for gate="cumsum", ignored for gate="none"),
    S0 [B,H,Dk,Dv] or None. Returns (o [B,H,T,Dv], S_final [B,H,Dk,Dv])."""
    q, k, v = _f(q, dtype), _f(k, dtype), _f(v, dtype)
    B, H, T, Dk = q.shape
    Dv = v.shape[-1]
    nc = T // C
    qc = q.reshape(B, H, nc, C, Dk)
    kc = k.reshape(B, H, nc, C, Dk)
    vc = v.reshape(B, H, nc, C, Dv)
    bc = _f(beta, dtype).reshape(B, H, nc, C)
    gs = _gate(g, B, H, T, C, gate, dtype)

    # chunk-independent stages, all chunks at once (_gdn_full.py:72-82)
    A = _kkt_A(kc, bc, gs, dtype)
    Tm = tri_inv(A, dtype)
    eg = np.exp(gs)
    W = np.einsum("...ij,...jd->...id", Tm, kc * (bc * eg)[..., None])
    U = np.einsum("...ij,...jd->...id", Tm, vc * bc[..., None])

    # intra-chunk gated causal scores (_gdn_full.py:88-92)
    x = gs[..., :, None] - gs[..., None, :]
    causal = np.tril(np.ones((C, C), dtype=dtype))
    Aqk = np.einsum("...id,...jd->...ij", qc, kc) * np.exp(np.minimum(x, 0)) * causal

    # the state scan over chunks (_gdn_full.py:83-87), then chunk_o (:88-94)
    S = np.zeros((B, H, Dk, Dv), dtype=dtype) if S0 is None else _f(S0, dtype).copy()
    o = np.empty((B, H, nc, C, Dv), dtype=dtype)
    for c in range(nc):
        gcc = gs[:, :, c]                               # [B,H,C]
        gl = gcc[..., -1]                               # [B,H]
        inter = np.einsum("bhid,bhde->bhie", qc[:, :, c], S) * np.exp(gcc)[..., None]
        vn = U[:, :, c] - np.einsum("bhid,bhde->bhie", W[:, :, c], S)
        o[:, :, c] = inter + np.einsum("bhij,bhje->bhie", Aqk[:, :, c], vn)
        S = (np.exp(gl)[..., None, None] * S
             + np.einsum("bhid,bhie->bhde", kc[:, :, c],
                         vn * np.exp(gl[..., None] - gcc)[..., None]))
    return (o * scale).reshape(B, H, T, Dv), S


def deltanet_forward(q, k, v, beta, scale, C=C_DEFAULT, dtype=np.float64):
    """Ungated DeltaNet forward, restating deltanet_reference
    (src/pto_fuser/forwards/deltanet.py:114-143). Returns a dict with A, T, W, U,
    v_new, h_state ([B,H,nc,...]) and o [B,H,nc,C,D], as the reference does."""
    q, k, v = _f(q, dtype), _f(k, dtype), _f(v, dtype)
    B, H, T, D = q.shape
    Dv = v.shape[-1]
    nc = T // C
    qc, kc = q.reshape(B, H, nc, C, D), k.reshape(B, H, nc, C, D)
    vc = v.reshape(B, H, nc, C, Dv)
    bc = _f(beta, dtype).reshape(B, H, nc, C)
    kb, vb = kc * bc[..., None], vc * bc[..., None]
    A = np.tril(np.einsum("...id,...jd->...ij", kb, kc), -1)
    Tm = tri_inv(A, dtype)
    W = np.einsum("...ij,...jd->...id", Tm, kb)
    U = np.einsum("...ij,...jd->...id", Tm, vb)
    h = np.zeros((B, H, nc, D, Dv), dtype=dtype)
    vn = np.zeros((B, H, nc, C, Dv), dtype=dtype)
    S = np.zeros((B, H, D, Dv), dtype=dtype)
    for c in range(nc):
        h[:, :, c] = S
        vn[:, :, c] = U[:, :, c] - np.einsum("bhid,bhde->bhie", W[:, :, c], S)
        S = S + np.einsum("bhid,bhie->bhde", kc[:, :, c], vn[:, :, c])
    o_inter = np.einsum("...id,...de->...ie", qc, h)
    Aqk = np.tril(np.einsum("...id,...jd->...ij", qc, kc))
    o = (o_inter + np.einsum("...ij,...je->...ie", Aqk, vn)) * scale
    return dict(A=A, T=Tm, W=W, U=U, v_new=vn, h_state=h, o=o, S_final=S)


def chunk_h_scan(w, u, k, decay, dtype=np.float64):
    """Simplified resident-state recurrence, restating scan_reference
    (src/pto_fuser/forwards/fused_stages.py:46-62): token-major operands
    w,u,k [B,nc,C,H,D], decay [B,H,nc] -> h_out [B,nc,H,D,D], final [B,H,D,D]."""
    w, u, k, decay = _f(w, dtype), _f(u, dtype), _f(k, dtype), _f(decay, dtype)
    B, nc, C, H, D = w.shape
    Dv = u.shape[-1]
    h_out = np.zeros((B, nc, H, D, Dv), dtype=dtype)
    S = np.zeros((B, H, D, Dv), dtype=dtype)
    for c in range(nc):
        h_out[:, c] = S
        ws = np.einsum("bihd,bhde->bihe", w[:, c], S)
        vcur = u[:, c] - ws
        S = decay[:, :, c][..., None, None] * S + np.einsum("bihd,bihe->bhde", k[:, c], vcur)
    return h_out, S


def kkt_gated(a, b, g_sum, beta, causal=False, dtype=np.float64):
    """Gated masked a@b^T per chunk, restating kkt_reference
    (src/pto_fuser/forwards/fused_stages.py:140-156) for any chunk batch layout:
    a, b [..., C, D], g_sum, beta [..., C];
    L = a b^T * exp(min(g_i + log(beta_i) - g_j, 0)) * mask (strict-lower, or causal
    incl. the diagonal when ``causal``)."""
    a, b = _f(a, dtype), _f(b, dtype)
    gs, bs = _f(g_sum, dtype), _f(beta, dtype)
    C = a.shape[-2]
    qk = np.einsum("...id,...jd->...ij", a, b)
    with np.errstate(divide="ignore"):
        gv = gs + np.log(bs)
    coeff = np.exp(np.minimum(gv[..., :, None] - gs[..., None, :], 0.0))
    mask = np.tril(np.ones((C, C), dtype=dtype), 0 if causal else -1)
    return qk * coeff * mask


def qkv_flash(q, k, v, g_sum, dtype=np.float64):
    """chunk_o intra term o = tril(q k^T * exp(min(g_i - g_j, 0))) v per chunk
    (the qkv_flash contract, src/pto_fuser/fused.py:368-387): q,k [...,C,D],
    v [...,C,DV], g_sum [...,C] -> [...,C,DV]."""
    q, k, v, gs = _f(q, dtype), _f(k, dtype), _f(v, dtype), _f(g_sum, dtype)
    C = q.shape[-2]
    s = np.einsum("...id,...jd->...ij", q, k)
    s = s * np.exp(np.minimum(gs[..., :, None] - gs[..., None, :], 0.0))
    s = s * np.tril(np.ones((C, C), dtype=dtype))
    return np.einsum("...ij,...je->...ie", s, v)


def rel_l2(got, ref) -> float:
    """Relative Frobenius error ||got - ref|| / ||ref|| (gate.frob_rel,
    src/pto_fuser/gate.py:25-27)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def gdn_forward_varlen(q, k, v, beta, g, cu_seqlens, scale, S0=None, C=C_DEFAULT, gate="raw",
                       dtype=np.float64):
    """Variable-length, grouped-query GDN forward: sequences packed token-major.

    q, k [T_total, Hg, Dk]; v [T_total, H, Dv]; beta, g [T_total, H]; sequence n spans
    tokens [cu_seqlens[n], cu_seqlens[n+1]); value head h reads query/key head
    h // (H // Hg); S0 [N, H, Dk, Dv] or None. Each sequence is gdn_forward on its own
    tokens (chunks start at its first token), padded at the end to whole chunks with
    beta = 0 and a flat gate (raw decay 0, or the last cumsum value repeated), which
    leaves the recurrence over the real tokens unchanged.
    Returns (o [T_total, H, Dv], S_final [N, H, Dk, Dv])."""
    q, k, v = _f(q, dtype), _f(k, dtype), _f(v, dtype)
    beta, g = _f(beta, dtype), _f(g, dtype) if g is not None else None
    cu = [int(x) for x in cu_seqlens]
    N = len(cu) - 1
    T_total, Hg, Dk = q.shape
    H, Dv = v.shape[1], v.shape[2]
    grp = H // Hg
    o = np.zeros((T_total, H, Dv), dtype=dtype)
    S_out = np.zeros((N, H, Dk, Dv), dtype=dtype)
    for n in range(N):
        a, b = cu[n], cu[n + 1]
        L = b - a
        if L == 0:
            if S0 is not None:
                S_out[n] = _f(S0, dtype)[n]
            continue
        Lp = -(-L // C) * C
        pad = lambda x: np.concatenate([x, np.zeros((Lp - L,) + x.shape[1:], dtype)], 0)
        qh = pad(q[a:b])[:, np.arange(H) // grp].transpose(1, 0, 2)[None]
        kh = pad(k[a:b])[:, np.arange(H) // grp].transpose(1, 0, 2)[None]
        vh = pad(v[a:b]).transpose(1, 0, 2)[None]
        bh = pad(beta[a:b]).T[None]
        if g is None or gate == "none":
            gh = np.zeros_like(bh)
        elif gate == "cumsum":
            gp = np.concatenate([g[a:b], np.repeat(g[b - 1:b], Lp - L, 0)], 0)
            gh = gp.T[None]
        else:
            gh = pad(g[a:b]).T[None]
        s0 = None if S0 is None else _f(S0, dtype)[n:n + 1]
        on, Sn = gdn_forward(qh, kh, vh, bh, gh, scale, S0=s0, C=C, gate=gate, dtype=dtype)
        o[a:b] = on[0].transpose(1, 0, 2)[:L]
        S_out[n] = Sn[0]
    return o, S_out


def linear_attention_recurrent(q, k, v, gates, dtype=np.float64):
    """Token-recurrent gated linear attention, the definition the chunked linear family
    (vanilla LA, RetNet, Mamba-2, GLA) computes: S_t = diag(g_t) S_{t-1} + k_t^T v_t,
    o_t = q_t S_t (examples/attention/_chunked.py:14-17, chunked_linear_reference
    :194-208). q, k, gates [N, T, d_k] (gates in (0, 1]), v [N, T, d_v] -> o [N, T, d_v]."""
    q, k, v, g = (_f(x, dtype) for x in (q, k, v, gates))
    N, T, d_k = q.shape
    o = np.zeros((N, T, v.shape[-1]), dtype=dtype)
    for n in range(N):
        S = np.zeros((d_k, v.shape[-1]), dtype=dtype)
        for t in range(T):
            S = g[n, t][:, None] * S + np.outer(k[n, t], v[n, t])
            o[n, t] = q[n, t] @ S
    return o


def kda_forward(q, k, v, beta, g_in, scale, C=C_DEFAULT, dtype=np.float64, S0=None,
                return_state=False):
    """Kimi Delta Attention forward (per-dimension gate), restating kda_reference
    (examples/attention/_kda_full.py:38-77): per chunk, g = per-dimension cumsum,
    A = tril((k e^g)(k e^-g)^T beta_i, -1), T = (I+A)^-1, W = T (k e^g beta), U = T (v beta),
    vc = U - W S, S = e^{g_tot} S + (k e^{g_tot-g})^T vc,
    o = scale ((q e^g) S_c + tril((q e^g)(k e^-g)^T, 0) vc).
    q, k, v [B,H,nc,C,D]; beta [B,H,nc,C]; g_in [B,H,nc,C,D] -> o [B,H,nc,C,D].
    S0 [B,H,D,D] optional initial state (the reference starts from 0); with
    return_state the final state [B,H,D,D] is returned as well."""
    q, k, v, beta, g_in = (_f(x, dtype) for x in (q, k, v, beta, g_in))
    B, H, nc, Cc, D = q.shape
    g = np.cumsum(g_in, axis=3)
    eye = np.eye(Cc, dtype=dtype)
    causal = np.tril(np.ones((Cc, Cc), dtype=dtype))
    o = np.zeros((B, H, nc, Cc, D), dtype=dtype)
    fin = np.zeros((B, H, D, D), dtype=dtype)
    for b in range(B):
        for h in range(H):
            S = np.zeros((D, D), dtype=dtype) if S0 is None else _f(S0[b, h], dtype).copy()
            for c in range(nc):
                gc, kc, bc = g[b, h, c], k[b, h, c], beta[b, h, c]
                ka, kb = kc * np.exp(gc), kc * np.exp(-gc)
                A = np.tril((ka @ kb.T) * bc[:, None], -1)
                T = tri_inv(A, dtype)
                W = T @ (ka * bc[:, None])
                U = T @ (v[b, h, c] * bc[:, None])
                vc = U - W @ S
                qe = q[b, h, c] * np.exp(gc)
                o[b, h, c] = qe @ S + ((qe @ kb.T) * causal) @ vc
                g_tot = gc[-1]
                S = np.exp(g_tot)[:, None] * S + (kc * np.exp(g_tot[None, :] - gc)).T @ vc
            fin[b, h] = S
    return (o * scale, fin) if return_state else o * scale


def segment_scan(A, B, X0, dtype=np.float64):
    """Apply per-segment affine state maps in order (the checker of
    ptof_seg_scan_exec; the reference has no segment split, its scan walks the
    whole sequence, kernels/scan_fused.h:198-262):
    X_0 = X0 (None: 0), X_{j+1} = A_j X_j + B_j (B None: no offset).
    A [H, n, D, D], B [H, n, D, Dv] or None, X0 [H, D, Dv] or None (then Dv from B).
    Returns (entry states [H, n, D, Dv], exit state [H, D, Dv])."""
    A = _f(A, dtype)
    H, n, D = A.shape[:3]
    Dv = (X0.shape[-1] if X0 is not None else B.shape[-1])
    X = np.zeros((H, D, Dv), dtype=dtype) if X0 is None else _f(X0, dtype).copy()
    entries = np.empty((H, n, D, Dv), dtype=dtype)
    for j in range(n):
        entries[:, j] = X
        X = np.einsum("hde,hev->hdv", A[:, j], X)
        if B is not None:
            X = X + _f(B, dtype)[:, j]
    return entries, X
