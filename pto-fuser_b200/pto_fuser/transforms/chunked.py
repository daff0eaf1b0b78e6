"""Batch the per-chunk intra-chunk scores of a chunked linear-attention program.

The canonical program (``forwards.chunked``) computes ``A_c = tril(q̃_c k̂_c^T, 0)``
once per chunk inside the scan, ``nc`` small einsums. ``BatchChunkIntraScore``
replaces them with one fused kernel over all ``M = N * nc`` chunks, a reshape, and a
per-chunk slice feeding each chunk's ``A V`` einsum (the reference's transform of the
same name, src/pto_fuser/transforms/chunked.py:33-103):

* scalar gate (vanilla LA, RetNet, Mamba-2): the decay factors out of the product,
  so the score is ``gated_qk_native_v2`` on raw q, k with the scalar log-cumgate
  ``g_intra`` (and ``beta_intra`` = 1);
* per-channel gate (GLA): the decay rides on the operands, ``qk_prologue[_v2]``
  computes ``tril((q*P)(k*invP)^T)`` directly.

The gate kind is an option of the transform: the program itself cannot tell them
apart.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

from ..ir import EinsumNode, FusedNode, Program, TensorOp, VecGlueNode
from ..transform import Transform, TransformResult


def select_prologue_kernel(C: int, d_k: int) -> str:
    """The reference picks its L2-ring variant for large tiles (C * d_k >= 4096); both
    keys run the same CUDA kernel here and stay distinct for program compatibility."""
    return "qk_prologue_v2" if C * d_k >= 4096 else "qk_prologue"


def _consumers(program: Program, name: str) -> List[int]:
    return [i for i, n in enumerate(program.nodes) if name in n.inputs]


class BatchChunkIntraScore(Transform):
    name = "batch-chunk-intra-score"
    summary = "nc per-chunk tril(q~ k^^T) intra scores -> one batched fused kernel"

    def __init__(self, N: int, nc: int, C: int, d_k: int, d_v: int,
                 per_dim_gate: bool = False, v2: Optional[bool] = None) -> None:
        self.N, self.nc, self.C, self.d_k, self.d_v = N, nc, C, d_k, d_v
        self.per_dim_gate, self.v2 = per_dim_gate, v2

    def _scores(self, program: Program) -> List[Tuple[int, int, str]]:
        """(score einsum, tril, masked name) per chunk: einsum 'nid,njd->nij' whose only
        consumer is a tril glue whose only consumer is einsum 'nij,nje->nie'."""
        found = []
        nodes = program.nodes
        for i, n in enumerate(nodes):
            if not (isinstance(n, EinsumNode) and n.equation == "nid,njd->nij"):
                continue
            c1 = _consumers(program, n.output)
            if len(c1) != 1 or not (isinstance(nodes[c1[0]], VecGlueNode)
                                    and nodes[c1[0]].op == "tril"):
                continue
            t = c1[0]
            c2 = _consumers(program, nodes[t].output)
            if len(c2) != 1 or not (isinstance(nodes[c2[0]], EinsumNode)
                                    and nodes[c2[0]].equation == "nij,nje->nie"):
                continue
            found.append((i, t, nodes[t].output))
        return found

    def match(self, program: Program) -> int:
        if any(isinstance(n, FusedNode) and n.output == "A_all" for n in program.nodes):
            return 0
        return 1 if self._scores(program) else 0

    def apply(self, program: Program) -> TransformResult:
        found = self._scores(program)
        if not found:
            return TransformResult(program, False, 0, "no per-chunk intra scores")
        params = {"nc": self.nc, "H": self.N, "C": self.C, "D": self.d_k}
        subsumed = [name for _, _, name in found]
        if self.per_dim_gate:
            kernel = ("qk_prologue_v2" if self.v2 else "qk_prologue") if self.v2 is not None \
                else select_prologue_kernel(self.C, self.d_k)
            fused = FusedNode(kernel=kernel, inputs=["q", "k", "P", "invP"], outputs=["A_all"],
                              params=params, subsumes=subsumed)
        else:
            fused = FusedNode(kernel="gated_qk_native_v2",
                              inputs=["q", "k", "g_intra", "beta_intra"], outputs=["A_all"],
                              params=dict(params, causal=True), subsumes=subsumed)
        head = [fused, TensorOp("reshape", ["A_all"], "A_allr",
                                params={"shape": (self.N, self.nc, self.C, self.C)})]
        score_idx = {i for i, _, _ in found}
        chunk_of_tril = {t: c for c, (_, t, _) in enumerate(found)}
        body = []
        for idx, node in enumerate(program.nodes):
            if idx in score_idx:
                continue
            if idx in chunk_of_tril:
                body.append(TensorOp("slice", ["A_allr"], node.output,
                                     params={"axis": 1, "index": chunk_of_tril[idx]}))
                continue
            body.append(node)
        new = Program(nodes=head + body, inputs=list(program.inputs),
                      outputs=list(program.outputs))
        return TransformResult(new, True, 1, f"{len(found)} intra scores -> {fused.kernel}")
