"""Staged-versus-fused head-to-head programs of the reference
(src/pto_fuser/forwards/fused_stages.py:34-163): the resident-state scan and the
gated kkt, each as a staged program and as a single FusedNode, with fp32 torch
references. C = D = 128 as in the reference's prototypes."""
from __future__ import annotations

import torch

from ..ir import EinsumNode, FusedNode, Program, TensorOp, VecGlueNode

C = D = 128


def make_scan_inputs(B: int, H: int, nc: int, device="cuda", seed: int = 0) -> dict:
    """Token-major [B,nc,C,H,D] operands with a contractive scale."""
    gen = torch.Generator().manual_seed(seed)
    w = (torch.randn(B, nc, C, H, D, generator=gen) * 0.02).half()
    k = (torch.randn(B, nc, C, H, D, generator=gen) * 0.02).half()
    u = (torch.randn(B, nc, C, H, D, generator=gen) * 0.05).half()
    decay = (0.7 + 0.2 * torch.rand(B, H, nc, generator=gen)).float()
    return {n: t.to(device) for n, t in dict(w=w, u=u, k=k, decay=decay).items()}


def scan_reference(inp: dict, B: int, H: int, nc: int) -> dict:
    w, u, k, d = (inp[n].float() for n in ("w", "u", "k", "decay"))
    dev = w.device
    h_out = torch.zeros(B, nc, H, D, D, device=dev)
    final = torch.zeros(B, H, D, D, device=dev)
    for b in range(B):
        for h in range(H):
            S = torch.zeros(D, D, device=dev)
            for c in range(nc):
                h_out[b, c, h] = S
                vc = u[b, c, :, h, :] - w[b, c, :, h, :] @ S
                S = d[b, h, c] * S + k[b, c, :, h, :].T @ vc
            final[b, h] = S
    return {"h_out": h_out, "final": final}


def build_scan_fused_program(B: int, H: int, nc: int) -> Program:
    node = FusedNode(kernel="chunk_h_scan", inputs=["w", "u", "k", "decay"],
                     outputs=["h_out", "final"], params={"B": B, "H": H, "nc": nc},
                     subsumes=["per-chunk WS / kv contraction pairs + residual glue"])
    return Program(nodes=[node], inputs=["w", "u", "k", "decay"], outputs=["h_out", "final"])


def build_scan_staged_program(B: int, H: int, nc: int) -> Program:
    N, f16 = B * H, torch.float16
    nodes = []
    for name in ("w", "u", "k"):
        nodes.append(TensorOp("permute", [name], f"{name}_p", {"dims": (0, 3, 1, 2, 4)}))
        nodes.append(TensorOp("reshape", [f"{name}_p"], f"{name}_b", {"shape": (N, nc, C, D)}))
    nodes.append(TensorOp("reshape", ["decay"], "decay_b", {"shape": (N, nc)}))
    nodes.append(TensorOp("zeros", ["w_b"], "S0", {"shape": (N, D, D), "dtype": f16}))
    readouts, S = [], "S0"
    for c in range(nc):
        readouts.append(S)
        for nm in ("w", "k", "u"):
            nodes.append(TensorOp("slice", [f"{nm}_b"], f"{nm}_c{c}", {"axis": 1, "index": c}))
        nodes.append(EinsumNode("ncd,nde->nce", [f"w_c{c}", S], f"WS{c}"))
        nodes.append(VecGlueNode("sub", [f"u_c{c}", f"WS{c}"], f"vc{c}", out_dtype=f16))
        nodes.append(EinsumNode("ncd,nce->nde", [f"k_c{c}", f"vc{c}"], f"kv{c}"))
        nodes.append(TensorOp("slice", ["decay_b"], f"dec{c}", {"axis": 1, "index": c}))
        nodes.append(TensorOp("reshape", [f"dec{c}"], f"decr{c}", {"shape": (N, 1, 1)}))
        nodes.append(VecGlueNode("mul", [S, f"decr{c}"], f"Sdec{c}"))
        S = f"S{c + 1}"
        nodes.append(VecGlueNode("add", [f"Sdec{c}", f"kv{c}"], S, out_dtype=f16))
    nodes.append(TensorOp("stack", readouts, "h_b", {"dim": 1}))
    nodes.append(TensorOp("reshape", ["h_b"], "h_bhncdd", {"shape": (B, H, nc, D, D)}))
    nodes.append(TensorOp("permute", ["h_bhncdd"], "h_out", {"dims": (0, 2, 1, 3, 4)}))
    nodes.append(TensorOp("reshape", [S], "final", {"shape": (B, H, D, D)}))
    return Program(nodes=nodes, inputs=["w", "u", "k", "decay"], outputs=["h_out", "final"])


def make_kkt_inputs(nc: int, H: int, device="cuda", seed: int = 0) -> dict:
    """k [1,T,H,D] fp16 (L2-normalised), chunk-local g_sum [1,T,H] fp32, beta fp16."""
    gen = torch.Generator().manual_seed(seed)
    T = nc * C
    k = torch.nn.functional.normalize(torch.randn(1, T, H, D, generator=gen), dim=-1).half()
    beta = torch.rand(1, T, H, generator=gen).half()
    g_in = torch.nn.functional.logsigmoid(torch.randn(1, T, H, generator=gen))
    g_sum = g_in.reshape(1, nc, C, H).cumsum(2).reshape(1, T, H)
    return {n: t.to(device) for n, t in dict(k=k, g_sum=g_sum, beta=beta).items()}


def kkt_reference(inp: dict, nc: int, H: int) -> dict:
    """L = (k k^T) * exp(min(g_i + log beta_i - g_j, 0)) * strict-lower, [T,H,C] fp16."""
    k, g, b = inp["k"], inp["g_sum"], inp["beta"]
    kc = k[0].float().reshape(nc, C, H, D)
    qk = torch.einsum("cihd,cjhd->cihj", kc, kc)
    gs = g[0].reshape(nc, C, H).float()
    gv = gs + torch.log(b[0].reshape(nc, C, H).float())
    coeff = torch.exp(torch.clamp(gv.permute(0, 2, 1)[..., None] - gs.permute(0, 2, 1)[:, :, None, :],
                                  max=0.0)).permute(0, 2, 1, 3)
    r = torch.arange(C, device=k.device)
    mask = (r[:, None] > r[None, :]).float()
    return {"L": (qk * coeff * mask[None, :, None, :]).reshape(nc * C, H, C).half()}


def build_kkt_fused_program(nc: int, H: int) -> Program:
    node = FusedNode(kernel="kkt_gated", inputs=["k", "g_sum", "beta"], outputs=["L"],
                     params={"nc": nc, "H": H}, subsumes=["qk einsum + gated/masked epilogue"])
    return Program(nodes=[node], inputs=["k", "g_sum", "beta"], outputs=["L"])
