"""Chunked (ungated) DeltaNet forward as an IR program, plus its fp32 torch
reference. Program structure and outputs follow src/pto_fuser/forwards/deltanet.py:23-143:
kkt -> opaque (I+A)^-1 -> W, U -> unrolled state scan -> chunk_o, returning
A, T, W, U, v_new, h_state and o."""
from __future__ import annotations

import torch

from ..ir import Program
from ._build import ProgramBuilder


def build_deltanet_program(B: int, H: int, nc: int, C: int, D: int, scale: float,
                           work=torch.float16) -> Program:
    M, N = B * H * nc, B * H
    b = ProgramBuilder(work)
    b.op("beta_u", "reshape", "beta", shape=[B, H, nc, C, 1])
    b.glue("kb", "mul", ["beta_u", "k"])
    b.glue("vb", "mul", ["beta_u", "v"])
    b.op("k_h", "cast", "k", dtype=work)
    b.op("q_h", "cast", "q", dtype=work)
    for src, dst in (("kb", "kbF"), ("vb", "vbF"), ("k_h", "kF"), ("q_h", "qF")):
        b.op(dst + "_r", "reshape", src, shape=[M, C, D])
        b.op(dst, "contiguous", dst + "_r")
    b.einsum("Araw", "nid,njd->nij", "kbF", "kF")
    b.glue("A_t", "tril", "Araw", diagonal=-1)
    b.op("A", "contiguous", "A_t")
    b.opaque("T_raw", "tri_inv_rec_unroll", "A")
    b.op("T", "cast", "T_raw", dtype=work)
    b.einsum("W_m", "nij,njd->nid", "T", "kbF")
    b.op("W", "reshape", "W_m", shape=[B, H, nc, C, D])
    b.einsum("U_m", "nij,njd->nid", "T", "vbF")
    b.op("U", "reshape", "U_m", shape=[B, H, nc, C, D])
    b.op("Wb", "reshape", "W", shape=[N, nc, C, D])
    b.op("Ub", "reshape", "U", shape=[N, nc, C, D])
    b.op("kb5", "reshape", "kF", shape=[N, nc, C, D])
    b.op("S0", "zeros", "Wb", shape=[N, D, D], dtype=work)
    hs, vns, S = [], [], "S0"
    for c in range(nc):
        hs.append(S)
        b.op(f"Wc{c}_s", "slice", "Wb", axis=1, index=c)
        b.op(f"Wc{c}", "contiguous", f"Wc{c}_s")
        b.einsum(f"WS{c}", "nid,nde->nie", f"Wc{c}", S)
        b.op(f"Uc{c}", "slice", "Ub", axis=1, index=c)
        vns.append(b.glue(f"vn{c}", "sub", [f"Uc{c}", f"WS{c}"]))
        b.op(f"kc{c}_s", "slice", "kb5", axis=1, index=c)
        b.op(f"kc{c}", "contiguous", f"kc{c}_s")
        b.einsum(f"dS{c}", "nid,nie->nde", f"kc{c}", f"vn{c}")
        S = b.glue(f"S{c + 1}", "add", [S, f"dS{c}"])
    b.op("h_bh", "stack", hs, dim=1)
    b.op("h_state", "reshape", "h_bh", shape=[B, H, nc, D, D])
    b.op("vn_bh", "stack", vns, dim=1)
    b.op("v_new", "reshape", "vn_bh", shape=[B, H, nc, C, D])
    b.op("h_flat_r", "reshape", "h_bh", shape=[M, D, D])
    b.op("h_flat", "contiguous", "h_flat_r")
    b.op("vn_flat_r", "reshape", "vn_bh", shape=[M, C, D])
    b.op("vn_flat", "contiguous", "vn_flat_r")
    b.einsum("o_inter", "nid,nde->nie", "qF", "h_flat")
    b.einsum("Aqk_raw", "nid,njd->nij", "qF", "kF")
    b.glue("Aqk_t", "tril", "Aqk_raw", diagonal=0)
    b.op("Aqk", "contiguous", "Aqk_t")
    b.einsum("o_intra", "nij,nje->nie", "Aqk", "vn_flat")
    b.glue("o_sum", "add", ["o_inter", "o_intra"], out_dtype=torch.float32)
    b.glue("o_s", "scale", "o_sum", scalar=scale, out_dtype=torch.float32)
    b.op("o", "reshape", "o_s", shape=[B, H, nc, C, D])
    return Program(nodes=b.nodes, inputs=["q", "k", "v", "beta"],
                   outputs=["A", "T", "W", "U", "v_new", "h_state", "o"])


def make_inputs(B, H, nc, C, D, device="cuda") -> dict:
    """Small-magnitude inputs (v * 0.1, beta in [0, 0.5)) that keep the fp16 staged
    recurrence well conditioned, as the reference's make_inputs does."""
    gen = torch.Generator().manual_seed(0)
    nrm = torch.nn.functional.normalize
    k = nrm(torch.randn(B, H, nc, C, D, generator=gen), dim=-1)
    q = nrm(torch.randn(B, H, nc, C, D, generator=gen), dim=-1)
    v = torch.randn(B, H, nc, C, D, generator=gen) * 0.1
    beta = torch.rand(B, H, nc, C, generator=gen) * 0.5
    return {n: t.half().to(device) for n, t in dict(q=q, k=k, v=v, beta=beta).items()}


def deltanet_reference(q, k, v, beta, B, H, nc, C, D, scale) -> dict:
    """The same pipeline in fp32 torch (the gate reference)."""
    qf, kf, vf, bf = q.float(), k.float(), v.float(), beta.float()
    M = B * H * nc
    kbF = (bf[..., None] * kf).reshape(M, C, D)
    vbF = (bf[..., None] * vf).reshape(M, C, -1)
    kF, qF = kf.reshape(M, C, D), qf.reshape(M, C, D)
    A = torch.tril(kbF @ kF.transpose(-1, -2), -1)
    eye = torch.eye(C, device=q.device).expand(M, C, C)
    T = torch.linalg.solve_triangular(eye + A, eye, upper=False, unitriangular=True)
    W, U = (T @ kbF).reshape(B, H, nc, C, D), (T @ vbF).reshape(B, H, nc, C, -1)
    h = torch.zeros(B, H, nc, D, vf.shape[-1], device=q.device)
    vn = torch.zeros(B, H, nc, C, vf.shape[-1], device=q.device)
    kf5 = kf.reshape(B, H, nc, C, D)
    for bb in range(B):
        for hh in range(H):
            S = torch.zeros(D, vf.shape[-1], device=q.device)
            for c in range(nc):
                h[bb, hh, c] = S
                x = U[bb, hh, c] - W[bb, hh, c] @ S
                vn[bb, hh, c] = x
                S = S + kf5[bb, hh, c].T @ x
    o = (qF @ h.reshape(M, D, -1)
         + torch.tril(qF @ kF.transpose(-1, -2)) @ vn.reshape(M, C, -1)) * scale
    return dict(A=A, T=T, W=W, U=U, h_state=h, v_new=vn, o=o.reshape(B, H, nc, C, -1))
