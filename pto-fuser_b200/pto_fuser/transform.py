"""Transforms: pure ``Program -> Program`` rewrites (what), separate from the cost
model (whether) and the verifier (is it correct and faster).

Interface as in the reference (src/pto_fuser/transform.py:39-183): a ``Transform``
has a kebab-case ``name``, a one-line ``summary``, ``match(program) -> int`` (number
of rewritable sites, 0 = not applicable) and ``apply(program) -> TransformResult``.
``canonicalize`` produces the all-staged baseline every verification compares
against. The read-mode / fused-store levers are annotation rewrites; on B200 they
do not change execution (torch's contraction has no read modes) and the policy
proposes them only when the cost model says they can pay.
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Dict, List

from .ir import EinsumNode, Node, Program, node_outputs


@dataclass
class TransformResult:
    program: Program
    changed: bool
    sites: int
    note: str = ""


class Transform:
    name: str = "transform"
    summary: str = ""

    def match(self, program: Program) -> int:  # pragma: no cover - abstract
        raise NotImplementedError

    def apply(self, program: Program) -> TransformResult:  # pragma: no cover - abstract
        raise NotImplementedError

    def __str__(self) -> str:
        return self.name


def producer_index(program: Program) -> Dict[str, int]:
    """name -> index of the node that writes it (the last writer)."""
    out: Dict[str, int] = {}
    for i, node in enumerate(program.nodes):
        for n in node_outputs(node):
            out[n] = i
    return out


def consumer_map(program: Program) -> Dict[str, List[int]]:
    """name -> indices of the nodes that read it."""
    out: Dict[str, List[int]] = {}
    for i, node in enumerate(program.nodes):
        for n in node.inputs:
            out.setdefault(n, []).append(i)
    return out


def splice(program: Program, drop: set, insert_at: int, new_nodes: List[Node]) -> Program:
    """Remove the nodes at ``drop`` and insert ``new_nodes`` before the original node
    ``insert_at``; the result is re-validated by Program construction."""
    nodes: List[Node] = []
    placed = False
    for i, node in enumerate(program.nodes):
        if i == insert_at:
            nodes.extend(new_nodes)
            placed = True
        if i not in drop:
            nodes.append(node)
    if not placed:
        nodes.extend(new_nodes)
    return Program(nodes=nodes, inputs=list(program.inputs), outputs=list(program.outputs))


def _rewrite_einsums(program: Program, pred, **changes) -> (Program, int):
    nodes, n = [], 0
    for node in program.nodes:
        if isinstance(node, EinsumNode) and pred(node):
            node = replace(node, **changes)
            n += 1
        nodes.append(node)
    return Program(nodes=nodes, inputs=list(program.inputs), outputs=list(program.outputs)), n


def canonicalize(program: Program) -> Program:
    """Every einsum on the baseline read (NN, no fused store)."""
    prog, _ = _rewrite_einsums(program, lambda n: True, read_mode="NN", fuse_out=False)
    return prog


class EnableDirectReads(Transform):
    name = "enable-direct-reads"
    summary = "EinsumNode read_mode NN -> auto"

    def match(self, program: Program) -> int:
        return sum(isinstance(n, EinsumNode) and n.read_mode == "NN" for n in program.nodes)

    def apply(self, program: Program) -> TransformResult:
        prog, n = _rewrite_einsums(program, lambda e: e.read_mode == "NN", read_mode="auto")
        return TransformResult(prog, n > 0, n, f"{n} einsum(s) -> direct read")


class EnableFusedStore(Transform):
    name = "enable-fused-store"
    summary = "EinsumNode fuse_out False -> True"

    def match(self, program: Program) -> int:
        return sum(isinstance(n, EinsumNode) and not n.fuse_out for n in program.nodes)

    def apply(self, program: Program) -> TransformResult:
        prog, n = _rewrite_einsums(program, lambda e: not e.fuse_out, fuse_out=True)
        return TransformResult(prog, n > 0, n, f"{n} einsum(s) -> fused store permitted")
