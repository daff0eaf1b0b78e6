"""Small builder for IR programs: appends nodes and returns the output name."""
from __future__ import annotations

from typing import List

import torch

from ..ir import EinsumNode, OpaqueNode, TensorOp, VecGlueNode


class ProgramBuilder:
    def __init__(self, work: torch.dtype) -> None:
        self.work = work
        self.nodes: List = []

    def einsum(self, out, eq, a, b, out_dtype=None):
        self.nodes.append(EinsumNode(eq, [a, b], out, out_dtype=out_dtype or self.work))
        return out

    def glue(self, out, op, ins, out_dtype=None, **params):
        ins = ins if isinstance(ins, list) else [ins]
        self.nodes.append(VecGlueNode(op, ins, out, params=params,
                                      out_dtype=out_dtype or self.work))
        return out

    def opaque(self, out, kernel, a):
        self.nodes.append(OpaqueNode(kernel, [a], out))
        return out

    def op(self, out, op, ins=None, **params):
        ins = [] if ins is None else (ins if isinstance(ins, list) else [ins])
        self.nodes.append(TensorOp(op, ins, out, params=params))
        return out
