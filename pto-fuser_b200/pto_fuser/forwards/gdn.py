"""The full gated DeltaNet (GDN) forward as an IR program, its host gate
coefficients, and the fp32 torch reference.

Follows examples/attention/_gdn_full.py of the reference:
  * ``make_gdn_inputs``        (:37-50)  random operands in [B,H,nc,C,D] layout;
  * ``gdn_reference``          (:57-97)  fp32 oracle; here also with an optional
                                         initial state and the final state;
  * ``prepare_gdn_bindings``   (:103-144) host-side gate coefficient tensors;
  * ``build_gdn_program``      (:150-235) the canonical all-staged Program.
The node names of ``build_gdn_program`` are the contract the structural transforms
match on (pto_fuser.transforms, pto_fuser.template). ``gdn_contraction_stages``
gives the four GDN contractions as single-node programs (src/pto_fuser/forwards/gdn.py).
"""
from __future__ import annotations

import torch

from ..ir import EinsumNode, Program
from ._build import ProgramBuilder


def make_gdn_inputs(B, H, nc, C, D, device="cuda", dtype=torch.float16, seed=None) -> dict:
    """q, k L2-normalised N(0,1), v N(0,1), beta U(0,1), g = logsigmoid(N(0,1)) fp32."""
    gen = torch.Generator().manual_seed(0 if seed is None else seed)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, H, nc, C, D, generator=gen), dim=-1)
    k = nrm(torch.randn(B, H, nc, C, D, generator=gen), dim=-1)
    v = torch.randn(B, H, nc, C, D, generator=gen)
    beta = torch.rand(B, H, nc, C, generator=gen)
    g_in = torch.nn.functional.logsigmoid(torch.randn(B, H, nc, C, generator=gen))
    out = {n: t.to(device=device, dtype=dtype) for n, t in dict(q=q, k=k, v=v, beta=beta).items()}
    out["g_in"] = g_in.to(device)
    return out


def _safe_exp(x):
    return torch.where(x <= 0, torch.exp(torch.clamp(x, max=0.0)), torch.zeros_like(x))


def gdn_reference(q, k, v, beta, g_in, scale, S0=None, return_final_state=False):
    """fp32 per-(b, h) chunk loop; q,k,v [B,H,nc,C,D], beta/g_in [B,H,nc,C]."""
    B, H, nc, C, D = q.shape
    Dv = v.shape[-1]
    qf, kf, vf, bf = q.float(), k.float(), v.float(), beta.float()
    gs = g_in.float().cumsum(dim=3)
    dev = q.device
    eye = torch.eye(C, device=dev)
    causal = torch.tril(torch.ones(C, C, device=dev))
    o = torch.zeros(B, H, nc, C, Dv, device=dev)
    fin = torch.zeros(B, H, D, Dv, device=dev)
    for b in range(B):
        for h in range(H):
            S = torch.zeros(D, Dv, device=dev) if S0 is None else S0[b, h].float().clone()
            for c in range(nc):
                g = gs[b, h, c]
                kc, vc, qc, bc = kf[b, h, c], vf[b, h, c], qf[b, h, c], bf[b, h, c]
                A = torch.tril((kc @ kc.T) * _safe_exp(g[:, None] - g[None, :]) * bc[:, None], -1)
                T = torch.linalg.solve_triangular(eye + A, eye, upper=False, unitriangular=True)
                W = T @ (kc * (bc * torch.exp(g))[:, None])
                U = T @ (vc * bc[:, None])
                vn = U - W @ S
                gate = torch.exp(torch.clamp(g[:, None] - g[None, :], max=0.0)) * causal
                o[b, h, c] = (qc @ S) * torch.exp(g)[:, None] + ((qc @ kc.T) * gate) @ vn
                gl = g[-1]
                S = torch.exp(gl) * S + kc.T @ (vn * torch.exp(gl - g)[:, None])
            fin[b, h] = S
    o = o * scale
    return (o, fin) if return_final_state else o


def prepare_gdn_bindings(q, k, v, beta, g_in, work=torch.float16) -> dict:
    """Flatten operands to [M, C, ...] (M = B*H*nc) and precompute every gate
    coefficient on the host, as the canonical program expects."""
    B, H, nc, C, D = q.shape
    M = B * H * nc
    gsum = g_in.float().cumsum(dim=3)
    gi, gj = gsum.unsqueeze(-1), gsum.unsqueeze(-2)
    bet = beta.float()
    gl = gsum[..., -1:]
    causal = torch.tril(torch.ones(C, C, device=q.device))
    flat = lambda t, *tail: t.reshape(M, *tail).to(work).contiguous()
    nflat = lambda t, *tail: t.reshape(B * H, nc, *tail).to(work).contiguous()
    return {
        "qF": flat(q, C, D), "kF": flat(k, C, D), "vF": flat(v, C, v.shape[-1]),
        "coefA": flat(_safe_exp(gi - gj) * bet.unsqueeze(-1), C, C),
        "coef_kb": flat((bet * torch.exp(gsum)).unsqueeze(-1), C, 1),
        "coef_vb": flat(bet.unsqueeze(-1), C, 1),
        "coef_qg": flat(torch.exp(gsum).unsqueeze(-1), C, 1),
        "coef_o": flat(torch.exp(torch.clamp(gi - gj, max=0.0)) * causal, C, C),
        "coef_vcs": nflat(torch.exp(gl.unsqueeze(-1) - gi), C, 1),
        "coef_S": nflat(torch.exp(gl).unsqueeze(-1), 1, 1),
        "g_native": gsum.reshape(M, C).float().contiguous(),
        "beta_native": bet.reshape(M, C).to(work).contiguous(),
        "beta_native_ones": torch.ones(M, C, device=q.device, dtype=work),
    }


GDN_PROGRAM_INPUTS = ["qF", "kF", "vF", "coefA", "coef_kb", "coef_vb", "coef_qg", "coef_o",
                      "coef_vcs", "coef_S", "g_native", "beta_native", "beta_native_ones"]


def build_gdn_program(B, H, nc, C, D, scale, work=torch.float16) -> Program:
    """Canonical all-staged GDN forward: output o [B,H,nc,C,D] (fp32)."""
    M, N = B * H * nc, B * H
    b = ProgramBuilder(work)
    # kkt: A = tril((k k^T) * coefA, -1)
    b.einsum("Araw", "nid,njd->nij", "kF", "kF")
    b.glue("Ag", "mul", ["Araw", "coefA"])
    b.glue("A_t", "tril", "Ag", diagonal=-1)
    b.op("A", "contiguous", "A_t")
    # (I + A)^-1
    b.opaque("T_raw", "tri_inv_rec_unroll", "A")
    b.op("Tm", "cast", "T_raw", dtype=work)
    # WY: W = T (k coef_kb), U = T (v coef_vb)
    b.glue("kb", "mul", ["kF", "coef_kb"])
    b.glue("vb", "mul", ["vF", "coef_vb"])
    b.einsum("W_m", "nij,njd->nid", "Tm", "kb")
    b.einsum("U_m", "nij,njd->nid", "Tm", "vb")
    b.op("Wb", "reshape", "W_m", shape=[N, nc, C, D])
    b.op("Ub", "reshape", "U_m", shape=[N, nc, C, D])
    b.op("kb5", "reshape", "kF", shape=[N, nc, C, D])
    # state scan, unrolled over chunks
    b.op("S0", "zeros", "Wb", shape=[N, D, D], dtype=work)
    hs, vns, S = [], [], "S0"
    for c in range(nc):
        hs.append(S)
        b.op(f"Wc{c}_s", "slice", "Wb", axis=1, index=c)
        b.op(f"Wc{c}", "contiguous", f"Wc{c}_s")
        b.einsum(f"WS{c}", "nid,nde->nie", f"Wc{c}", S)
        b.op(f"Uc{c}", "slice", "Ub", axis=1, index=c)
        vns.append(b.glue(f"vn{c}", "sub", [f"Uc{c}", f"WS{c}"]))
        b.op(f"vcs{c}", "slice", "coef_vcs", axis=1, index=c)
        b.glue(f"vn2{c}", "mul", [f"vn{c}", f"vcs{c}"])
        b.op(f"kc{c}_s", "slice", "kb5", axis=1, index=c)
        b.op(f"kc{c}", "contiguous", f"kc{c}_s")
        b.einsum(f"dS{c}", "nid,nie->nde", f"kc{c}", f"vn2{c}")
        b.op(f"sc{c}", "slice", "coef_S", axis=1, index=c)
        b.glue(f"Sd{c}", "mul", [S, f"sc{c}"])
        S = b.glue(f"S{c + 1}", "add", [f"Sd{c}", f"dS{c}"])
    b.op("h_bh", "stack", hs, dim=1)
    b.op("h_flat", "reshape", "h_bh", shape=[M, D, D])
    b.op("vn_bh", "stack", vns, dim=1)
    b.op("vn_flat", "reshape", "vn_bh", shape=[M, C, D])
    # chunk_o: o = (q h) coef_qg + tril(q k^T coef_o) v_new, scaled
    b.einsum("o_inter_m", "nid,nde->nie", "qF", "h_flat")
    b.glue("o_inter", "mul", ["o_inter_m", "coef_qg"])
    b.einsum("Aqk", "nid,njd->nij", "qF", "kF")
    b.glue("Aqk_g", "mul", ["Aqk", "coef_o"])
    b.op("Aqk_c", "contiguous", "Aqk_g")
    b.einsum("o_intra", "nij,nje->nie", "Aqk_c", "vn_flat")
    b.glue("o_sum", "add", ["o_inter", "o_intra"], out_dtype=torch.float32)
    b.glue("o_s", "scale", "o_sum", scalar=scale, out_dtype=torch.float32)
    b.op("o", "reshape", "o_s", shape=[B, H, nc, C, D])
    return Program(nodes=b.nodes, inputs=list(GDN_PROGRAM_INPUTS), outputs=["o"])


def _stage(eq: str) -> Program:
    a, bb = (s.strip() for s in eq.split("->")[0].split(","))
    out = eq.split("->")[1].strip()
    return Program(nodes=[EinsumNode(eq, [a, bb], out, out_dtype=torch.float16)],
                   inputs=[a, bb], outputs=[out])


def gdn_contraction_stages(B: int = 2, nc: int = 4, H: int = 16, C: int = 64, D: int = 128,
                           device="cuda") -> list:
    """[(name, Program, bindings)] for the kkt / wy / chunk_h / chunk_o contractions."""
    Bn = B * nc
    g = dict(device=device, dtype=torch.float16)
    r = lambda *s: torch.randn(*s, **g)
    return [
        ("kkt", _stage("bihd,bjhd->bihj"), {"bihd": r(Bn, C, H, D), "bjhd": r(Bn, C, H, D)}),
        ("wy_fast", _stage("bihj,bjhd->bihd"), {"bihj": r(Bn, C, H, C), "bjhd": r(Bn, C, H, D)}),
        ("chunk_h", _stage("bvhd,bvhe->bhde"), {"bvhd": r(Bn, C, H, D), "bvhe": r(Bn, C, H, D)}),
        ("chunk_o", _stage("bvhd,bhde->bvhe"), {"bvhd": r(Bn, C, H, D), "bhde": r(Bn, H, D, D)}),
    ]
