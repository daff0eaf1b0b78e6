"""Kimi Delta Attention (KDA): the delta-rule forward with a per-dimension gate.

KDA is GDN whose log decay is a vector g [.., C, D] per token (per key dimension)
instead of a scalar, so the gate multiplies the contraction operands instead of the
scores (the reference's examples/attention/_kda_full.py:1-19). Per chunk, with g the
chunk-local cumsum and g_tot its last row:

    A   = tril((k*e^g)(k*e^-g)^T * beta_i, -1)        T = (I + A)^-1
    W   = T (k*e^g*beta)   U = T (v*beta)            vc = U - W S
    S  <- e^{g_tot} * S (row-wise) + (k*e^{g_tot-g})^T vc
    o   = scale * ((q*e^g) S_c + tril((q*e^g)(k*e^-g)^T, 0) vc)

``build_kda_program`` is the canonical staged Program with the reference's node names
(so ``LowerPerDimScan`` can lower its scan onto ``chunk_h_scan`` with a per-dimension
decay); ``prepare_kda_bindings`` precomputes the gate coefficients.
"""
from __future__ import annotations

from typing import Dict

import torch

from ..ir import EinsumNode, OpaqueNode, Program, TensorOp, VecGlueNode


def make_kda_inputs(B, H, nc, C, D, device, dtype=torch.float16, seed=0) -> Dict[str, torch.Tensor]:
    """q, k unit-normalised N(0,1), v ~ N(0,1), beta = sigmoid(N(0,1)), per-dimension
    log decay g = -U(0,1) * 0.05 (the reference's KDA input distributions)."""
    gen = torch.Generator().manual_seed(seed)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, H, nc, C, D, generator=gen), dim=-1)
    k = nrm(torch.randn(B, H, nc, C, D, generator=gen), dim=-1)
    v = torch.randn(B, H, nc, C, D, generator=gen)
    beta = torch.sigmoid(torch.randn(B, H, nc, C, generator=gen))
    g_in = -torch.rand(B, H, nc, C, D, generator=gen) * 0.05
    dev = lambda t, dt=dtype: t.to(device=device, dtype=dt)
    return dict(q=dev(q), k=dev(k), v=dev(v), beta=dev(beta), g_in=dev(g_in, torch.float32))


def prepare_kda_bindings(q, k, v, beta, g_in, work=torch.float16) -> Dict[str, torch.Tensor]:
    """Flattened operands (M = B*H*nc chunks) and the per-dimension gate coefficients:
    e^g, e^-g, e^g*beta (operands), beta, e^{g_tot-g} (scan keys), e^{g_tot} (state rows)."""
    B, H, nc, C, D = q.shape
    M, N = B * H * nc, B * H
    g = g_in.float().cumsum(dim=3)
    bet = beta.float().unsqueeze(-1)
    g_tot = g[:, :, :, -1:, :]
    flat = lambda t, *tail: t.reshape(M, *tail).to(work).contiguous()
    per_head = lambda t, *tail: t.reshape(N, nc, *tail).to(work).contiguous()
    return {
        "qF": flat(q, C, D), "kF": flat(k, C, D), "vF": flat(v, C, D),
        "coef_ag": flat(torch.exp(g), C, D), "coef_bg": flat(torch.exp(-g), C, D),
        "coef_beta": flat(bet.expand(B, H, nc, C, 1), C, 1),
        "coef_wg": flat(torch.exp(g) * bet, C, D),
        "coef_ub": flat(bet.expand(B, H, nc, C, 1), C, 1),
        "coef_krest": per_head(torch.exp(g_tot - g), C, D),
        "coef_S": per_head(torch.exp(g_tot).reshape(B, H, nc, D, 1), D, 1),
    }


def build_kda_program(B, H, nc, C, D, scale, work=torch.float16) -> Program:
    """The canonical KDA forward (scan unrolled, no fused nodes); output o [B,H,nc,C,D]."""
    M, N = B * H * nc, B * H
    nodes: list = []
    E = lambda out, eq, a, b: nodes.append(EinsumNode(eq, [a, b], out, out_dtype=work))
    G = lambda out, op, ins, dt=work, **p: nodes.append(
        VecGlueNode(op, ins if isinstance(ins, list) else [ins], out, params=p, out_dtype=dt))
    Tn = lambda out, op, ins, **p: nodes.append(
        TensorOp(op, ins if isinstance(ins, list) else [ins], out, params=p))

    # kkt: A = tril((k e^g)(k e^-g)^T * beta, -1)
    G("a_op", "mul", ["kF", "coef_ag"])
    G("b_op", "mul", ["kF", "coef_bg"])
    E("Araw", "nid,njd->nij", "a_op", "b_op")
    G("Ag", "mul", ["Araw", "coef_beta"])
    G("A_t", "tril", "Ag", diagonal=-1)
    Tn("A", "contiguous", "A_t")
    # (I + A)^-1: the opaque triangular inverse
    nodes.append(OpaqueNode("tri_inv_rec_unroll", ["A"], "T_raw"))
    Tn("Tm", "cast", "T_raw", dtype=work)
    # WY: W = T (k e^g beta), U = T (v beta)
    G("wk", "mul", ["kF", "coef_wg"])
    G("vb", "mul", ["vF", "coef_ub"])
    E("W_m", "nij,njd->nid", "Tm", "wk")
    E("U_m", "nij,njd->nid", "Tm", "vb")
    Tn("Wb", "reshape", "W_m", shape=[N, nc, C, D])
    Tn("Ub", "reshape", "U_m", shape=[N, nc, C, D])
    Tn("kb5", "reshape", "kF", shape=[N, nc, C, D])
    # chunk scan, per-dimension decay (unrolled)
    Tn("S0", "zeros", "Wb", shape=[N, D, D], dtype=work)
    hs, vns, S = [], [], "S0"
    for c in range(nc):
        hs.append(S)
        Tn(f"Wc{c}_s", "slice", "Wb", axis=1, index=c)
        Tn(f"Wc{c}", "contiguous", f"Wc{c}_s")
        E(f"WS{c}", "nid,nde->nie", f"Wc{c}", S)
        Tn(f"Uc{c}", "slice", "Ub", axis=1, index=c)
        G(f"vn{c}", "sub", [f"Uc{c}", f"WS{c}"])
        vns.append(f"vn{c}")
        Tn(f"kc{c}_s", "slice", "kb5", axis=1, index=c)
        Tn(f"kc{c}", "contiguous", f"kc{c}_s")
        Tn(f"krc{c}", "slice", "coef_krest", axis=1, index=c)
        G(f"krest{c}", "mul", [f"kc{c}", f"krc{c}"])
        E(f"dS{c}", "nid,nie->nde", f"krest{c}", f"vn{c}")
        Tn(f"sc{c}", "slice", "coef_S", axis=1, index=c)
        G(f"Sd{c}", "mul", [S, f"sc{c}"])
        G(f"S{c + 1}", "add", [f"Sd{c}", f"dS{c}"])
        S = f"S{c + 1}"
    Tn("h_bh", "stack", hs, dim=1)
    Tn("h_flat", "reshape", "h_bh", shape=[M, D, D])
    Tn("vn_bh", "stack", vns, dim=1)
    Tn("vn_flat", "reshape", "vn_bh", shape=[M, C, D])
    # chunk_o
    G("q_eff", "mul", ["qF", "coef_ag"])
    E("o_inter", "nid,nde->nie", "q_eff", "h_flat")
    G("k_eff", "mul", ["kF", "coef_bg"])
    E("Aqk", "nid,njd->nij", "q_eff", "k_eff")
    G("Aqk_t", "tril", "Aqk", diagonal=0)
    Tn("Aqk_c", "contiguous", "Aqk_t")
    E("o_intra", "nij,nje->nie", "Aqk_c", "vn_flat")
    G("o_sum", "add", ["o_inter", "o_intra"], dt=torch.float32)
    G("o_s", "scale", "o_sum", dt=torch.float32, scalar=scale)
    Tn("o", "reshape", "o_s", shape=[B, H, nc, C, D])
    inputs = ["qF", "kF", "vF", "coef_ag", "coef_bg", "coef_beta", "coef_wg", "coef_ub",
              "coef_krest", "coef_S"]
    return Program(nodes=nodes, inputs=inputs, outputs=["o"])
