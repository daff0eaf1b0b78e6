"""Chunked linear attention: the recurrence behind vanilla linear attention, RetNet,
Mamba-2 (SSD) and GLA, as a canonical pto_fuser ``Program``.

Per head, with state ``S`` [d_k, d_v] and gate ``g_t`` in (0, 1]^{d_k}:

    S_t = diag(g_t) S_{t-1} + k_t^T v_t        o_t = q_t S_t

(examples/attention/_chunked.py:8-20 of the reference). Chunk-parallel form with
``P_i`` the inclusive in-chunk gate product, ``gamma = P_{C-1}``:

    O_c = tril((q*P)(k/P)^T, 0) V_c + (q*P) S_in       S_out = diag(gamma) S_in + (k*gamma/P)^T V_c

The variants differ only in the gate: 1 (vanilla), a per-head constant (RetNet), a
per-token scalar (Mamba-2), a per-channel vector (GLA). The Program keeps the
reference's node kinds, equations and input names, so the ``batch-chunk-intra-score``
transform (``pto_fuser.transforms.chunked``) recognises the per-chunk intra score
``einsum "nid,njd->nij" -> tril(0) -> einsum "nij,nje->nie"`` and batches it into one
fused kernel (``gated_qk_native_v2`` for a scalar gate, ``qk_prologue[_v2]`` for a
per-channel gate).
"""
from __future__ import annotations

from typing import Dict

import torch

from ..ir import EinsumNode, Program, TensorOp, VecGlueNode


def build_chunked_linear_program(N: int, nc: int, C: int, d_k: int, d_v: int,
                                 work=torch.float16) -> Program:
    """Canonical chunked linear attention over N = B*H heads and nc chunks.

    Inputs (chunk-major, batched over N): q, k, P, invP, gammaInvP [N, nc, C, d_k];
    v [N, nc, C, d_v]; gamma [N, nc, d_k]; g_intra [N*nc, C] (log of the scalar
    cumulative gate) and beta_intra [N*nc, C] (ones), read only once the scalar
    intra-score batching applies. Output o [N, nc, C, d_v]."""
    nodes: list = []
    add = nodes.append
    add(TensorOp("zeros", ["q"], "S0", params={"shape": (N, d_k, d_v), "dtype": work}))
    S = "S0"
    outs = []
    for c in range(nc):
        for src in ("q", "k", "v", "P", "invP", "gammaInvP"):
            add(TensorOp("slice", [src], f"{src}{c}", params={"axis": 1, "index": c}))
        add(TensorOp("slice", ["gamma"], f"g{c}", params={"axis": 1, "index": c}))
        # operands with the decay applied: q*P, k/P, k*gamma/P
        add(VecGlueNode("mul", [f"q{c}", f"P{c}"], f"qd{c}", out_dtype=work))
        add(VecGlueNode("mul", [f"k{c}", f"invP{c}"], f"kinv{c}", out_dtype=work))
        add(VecGlueNode("mul", [f"k{c}", f"gammaInvP{c}"], f"kout{c}", out_dtype=work))
        # intra-chunk score and its product with V, then the carried state's term
        add(EinsumNode("nid,njd->nij", [f"qd{c}", f"kinv{c}"], f"A{c}", out_dtype=work))
        add(VecGlueNode("tril", [f"A{c}"], f"Am{c}", params={"diagonal": 0}, out_dtype=work))
        add(EinsumNode("nij,nje->nie", [f"Am{c}", f"v{c}"], f"o_intra{c}", out_dtype=work))
        add(EinsumNode("nid,nde->nie", [f"qd{c}", S], f"o_inter{c}", out_dtype=work))
        add(VecGlueNode("add", [f"o_inter{c}", f"o_intra{c}"], f"o{c}", out_dtype=work))
        outs.append(f"o{c}")
        # state: S' = diag(gamma) S + (k gamma/P)^T V
        add(EinsumNode("nid,nie->nde", [f"kout{c}", f"v{c}"], f"dS{c}", out_dtype=work))
        add(TensorOp("reshape", [f"g{c}"], f"gcol{c}", params={"shape": (N, d_k, 1)}))
        add(VecGlueNode("mul", [S, f"gcol{c}"], f"Sdec{c}", out_dtype=work))
        add(VecGlueNode("add", [f"Sdec{c}", f"dS{c}"], f"S{c + 1}", out_dtype=work))
        S = f"S{c + 1}"
    add(TensorOp("stack", outs, "o", params={"dim": 1}))
    inputs = ["q", "k", "v", "P", "invP", "gammaInvP", "gamma", "g_intra", "beta_intra"]
    return Program(nodes=nodes, inputs=inputs, outputs=["o"])


def prepare_chunked_inputs(q, k, v, gates, *, work=torch.float16) -> Dict[str, torch.Tensor]:
    """Bindings of build_chunked_linear_program from per-token gates [N, nc, C, d_k]
    (in (0, 1]; a scalar gate is broadcast over d_k). P is the inclusive in-chunk
    cumulative product; g_intra is log P averaged over d_k (exact for a scalar gate)."""
    gf = gates.float().clamp_min(1e-6)
    P = torch.cumprod(gf, dim=2)
    gamma = P[:, :, -1, :]
    invP = 1.0 / P
    gammaInvP = gamma.unsqueeze(2) * invP
    N, nc, C = P.shape[:3]
    g_intra = torch.log(P).mean(dim=-1).reshape(N * nc, C).contiguous()
    beta_intra = torch.ones(N * nc, C, device=P.device, dtype=work)
    cast = lambda t: t.to(work).contiguous()
    return dict(q=cast(q), k=cast(k), v=cast(v), P=cast(P), invP=cast(invP),
                gammaInvP=cast(gammaInvP), gamma=cast(gamma), g_intra=g_intra,
                beta_intra=beta_intra)
