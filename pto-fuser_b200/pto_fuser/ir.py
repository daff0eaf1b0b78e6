"""The pto-fuser IR: an ordered program of named-tensor steps.

Same node kinds and semantics as the reference IR (src/pto_fuser/ir.py:29-180):

  * ``EinsumNode``  — one contraction (two operands, einsum equation);
  * ``OpaqueNode``  — a foreign kernel the contraction core cannot express (tri-inv);
  * ``VecGlueNode`` — a standalone elementwise op (mul / sub / add / tril / scale);
  * ``FusedNode``   — a sub-chain collapsed into one hosted kernel (several outputs);
  * ``TensorOp``    — host plumbing (reshape, slice, stack, cast, zeros, ...), no kernel.

On B200 every node runs on the current CUDA stream: einsums and glue through torch,
opaque and fused nodes through the sm_100a kernel library. ``read_mode`` /
``fuse_out`` on an ``EinsumNode`` are the reference planner's read-mode annotations;
they are kept (transforms set them) but carry no meaning for torch's contraction.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, List, Optional


@dataclass(frozen=True)
class TensorRef:
    """A named handle; ``shape`` / ``dtype`` are advisory documentation."""
    name: str
    shape: Optional[tuple] = None
    dtype: Optional[Any] = None

    def __str__(self) -> str:
        return self.name


class Node:
    """Base of every program step."""
    inputs: List[str]
    output: str


@dataclass
class EinsumNode(Node):
    equation: str
    inputs: List[str]
    output: str
    out_dtype: Optional[Any] = None     # result is computed in fp32, then cast
    read_mode: str = "auto"             # "auto" | "NN" (reference planner annotation)
    fuse_out: bool = True
    epilogue: Optional[list] = None
    prologue: Optional[list] = None


@dataclass
class OpaqueNode(Node):
    """A hosted foreign kernel; the registry entry owns its dtype contract."""
    kernel: str
    inputs: List[str]
    output: str
    params: dict = field(default_factory=dict)


@dataclass
class VecGlueNode(Node):
    """Elementwise glue computed in fp32: tril | add | sub | mul | scale."""
    op: str
    inputs: List[str]
    output: str
    params: dict = field(default_factory=dict)
    out_dtype: Optional[Any] = None


@dataclass
class FusedNode(Node):
    """A sub-chain replaced by one kernel from the fused-kernel registry. The only
    node kind with several outputs; ``output`` names the first."""
    kernel: str
    inputs: List[str]
    outputs: List[str]
    params: dict = field(default_factory=dict)
    subsumes: List[str] = field(default_factory=list)

    @property
    def output(self) -> str:
        return self.outputs[0]


@dataclass
class TensorOp(Node):
    """reshape | contiguous | transpose | permute | cast | slice | stack | zeros."""
    op: str
    inputs: List[str]
    output: str
    params: dict = field(default_factory=dict)


def node_outputs(node: Node) -> List[str]:
    """Every name a step binds (a FusedNode binds its whole output list)."""
    outs = getattr(node, "outputs", None)
    return list(outs) if outs is not None else [node.output]


@dataclass
class Program:
    """Ordered steps plus the names bound at run time (``inputs``) and returned
    (``outputs``). Construction checks use-before-definition."""
    nodes: List[Node]
    inputs: List[str]
    outputs: List[str]

    def __post_init__(self) -> None:
        known = set(self.inputs)
        for node in self.nodes:
            for name in node.inputs:
                if name not in known:
                    raise ValueError(f"step producing {node.output!r} reads {name!r} before "
                                     "it is produced or bound as an input")
            known.update(node_outputs(node))
        missing = [o for o in self.outputs if o not in known]
        if missing:
            raise ValueError(f"declared outputs never produced: {missing}")
