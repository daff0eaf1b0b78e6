"""Template emission: a contraction plus its local glue -> one proven fused kernel.

Interface of the reference generator (src/pto_fuser/template.py:42-436):
``extract_epilogue_unit`` grows the single-consumer glue chain after an einsum and
the per-operand prescale ``mul`` before it; each ``Template`` recognises one proven
kernel shape; ``FuseContractionEpilogue`` rewrites every unit some template matches
and leaves the rest staged; ``FuseChunkOFlash`` fuses the chunk_o score -> output
chain into one ``qkv_flash_native_v2`` node; ``epilogue_report`` explains each
contraction's fate. Proven-only: a template exists only where a kernel backs it.
The per-dim (KDA) chunk_o score is backed by the ``qk_prologue`` kernel
(``PerDimPrologueTemplate``) and its score -> output chain by ``qkvp_flash_native_v2``
(``FusePerDimChunkOFlash``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

from .ir import EinsumNode, FusedNode, Program, TensorOp, VecGlueNode
from .transform import Transform, TransformResult, producer_index, splice


@dataclass
class EpilogueUnit:
    anchor_idx: int
    anchor: EinsumNode
    epilogue: List[Tuple[int, object]]
    prologue: Dict[str, Tuple[int, List[str]]]
    boundary_out: str

    @property
    def epilogue_ops(self) -> List[str]:
        return [n.op for _, n in self.epilogue]


def _only_consumer(program: Program, name: str) -> Optional[int]:
    hits = [i for i, n in enumerate(program.nodes) if name in n.inputs]
    return hits[0] if len(hits) == 1 else None


def extract_epilogue_unit(program: Program, anchor_idx: int) -> EpilogueUnit:
    anchor = program.nodes[anchor_idx]
    chain: List[Tuple[int, object]] = []
    cur = anchor.output
    while True:
        c = _only_consumer(program, cur)
        if c is None:
            break
        nd = program.nodes[c]
        glue = isinstance(nd, VecGlueNode) and nd.op in ("mul", "scale", "tril")
        plumb = isinstance(nd, TensorOp) and nd.op == "contiguous"
        if not (glue or plumb):
            break
        chain.append((c, nd))
        cur = nd.output
    prod = producer_index(program)
    pro: Dict[str, Tuple[int, List[str]]] = {}
    for operand in anchor.inputs:
        p = prod.get(operand)
        if p is not None and isinstance(program.nodes[p], VecGlueNode) and program.nodes[p].op == "mul":
            pro[operand] = (p, list(program.nodes[p].inputs))
    return EpilogueUnit(anchor_idx, anchor, chain, pro, cur)


@dataclass
class Dims:
    B: int
    H: int
    nc: int
    C: int
    D: int
    v2: Optional[bool] = None

    @property
    def N(self) -> int:
        return self.B * self.H

    @property
    def M(self) -> int:
        return self.B * self.H * self.nc


class Template:
    name: str = "template"
    family: str = ""

    def matches(self, program: Program, unit: EpilogueUnit) -> bool:  # pragma: no cover
        raise NotImplementedError

    def emit(self, program: Program, unit: EpilogueUnit, dims: Dims) -> Tuple[FusedNode, set]:
        raise NotImplementedError  # pragma: no cover


def _coef(unit: EpilogueUnit, op: str) -> Optional[str]:
    for _, n in unit.epilogue:
        if isinstance(n, VecGlueNode) and n.op == op:
            rest = [x for x in n.inputs if x != unit.anchor.output]
            return rest[0] if rest else None
    return None


class GatedKKTTemplate(Template):
    """A = tril((k k^T) * coefA, -1)  ->  kkt_gated_native[_v2]."""
    name = "kkt-gated-native"
    family = "scalar-gate"

    def matches(self, program, unit) -> bool:
        a, b = unit.anchor.inputs
        return (unit.anchor.equation == "nid,njd->nij" and a == b == "kF"
                and unit.epilogue_ops == ["mul", "tril", "contiguous"])

    def emit(self, program, unit, dims):
        node = FusedNode(kernel="kkt_gated_native_v2" if dims.v2 else "kkt_gated_native",
                         inputs=["kF", "g_native", "beta_native"], outputs=[unit.boundary_out],
                         params={"nc": dims.nc, "H": dims.H, "B": dims.B},
                         subsumes=["kkt einsum + coefA mul + tril"])
        return node, {unit.anchor_idx} | {i for i, _ in unit.epilogue}


class GatedChunkOTemplate(Template):
    """Aqk = (q k^T) * coef_o  ->  gated_qk_native[_v2] (causal, beta = 1)."""
    name = "chunk-o-gated-native"
    family = "scalar-gate"

    def matches(self, program, unit) -> bool:
        a, b = unit.anchor.inputs
        return (unit.anchor.equation == "nid,njd->nij" and (a, b) == ("qF", "kF")
                and unit.epilogue_ops == ["mul", "contiguous"] and _coef(unit, "mul") == "coef_o")

    def emit(self, program, unit, dims):
        node = FusedNode(kernel="gated_qk_native_v2" if dims.v2 else "gated_qk_native",
                         inputs=["qF", "kF", "g_native", "beta_native_ones"],
                         outputs=[unit.boundary_out],
                         params={"nc": dims.nc, "H": dims.H, "B": dims.B, "causal": True},
                         subsumes=["chunk_o Aqk einsum + coef_o mul + contiguous"])
        return node, {unit.anchor_idx} | {i for i, _ in unit.epilogue}


class PerDimPrologueTemplate(Template):
    """KDA chunk_o score with the per-dimension gate on its operands:
    ``Aqk = tril((qF * coef_ag)(kF * coef_bg)^T, 0)`` -> ``qk_prologue[_v2]``, which
    applies the two operand scales while loading (the reference's template of the same
    name, src/pto_fuser/template.py:174-203). The unit is the score einsum whose two
    operands come from those prescale muls, followed by ``tril -> contiguous``. The
    q-side product also feeds the inter-chunk output, so it stays; the k-side product
    is dropped when the score einsum is its only consumer."""
    name = "qk-prologue"
    family = "per-dim-prologue"

    def matches(self, program, unit) -> bool:
        pa = unit.prologue.get(unit.anchor.inputs[0])
        pb = unit.prologue.get(unit.anchor.inputs[1])
        return (pa is not None and pb is not None
                and unit.anchor.equation == "nid,njd->nij"
                and pa[1] == ["qF", "coef_ag"] and pb[1] == ["kF", "coef_bg"]
                and unit.epilogue_ops == ["tril", "contiguous"])

    def emit(self, program, unit, dims):
        from .transforms.chunked import select_prologue_kernel
        if dims.v2 is None:
            kernel = select_prologue_kernel(dims.C, dims.D)
        else:
            kernel = "qk_prologue_v2" if dims.v2 else "qk_prologue"
        node = FusedNode(kernel=kernel, inputs=["qF", "kF", "coef_ag", "coef_bg"],
                         outputs=[unit.boundary_out],
                         params={"nc": dims.nc, "H": dims.N, "C": dims.C, "D": dims.D},
                         subsumes=["chunk_o k-side gate mul + Aqk einsum + tril + contiguous"])
        drop = {unit.anchor_idx} | {i for i, _ in unit.epilogue}
        k_mul = unit.prologue[unit.anchor.inputs[1]][0]
        if _only_consumer(program, program.nodes[k_mul].output) == unit.anchor_idx:
            drop.add(k_mul)
        return node, drop


def default_templates() -> List[Template]:
    return [GatedKKTTemplate(), GatedChunkOTemplate(), PerDimPrologueTemplate()]


class FuseContractionEpilogue(Transform):
    name = "fuse-contraction-epilogue"
    summary = "contraction + epilogue glue -> proven gated-matmul FusedNode (template)"

    def __init__(self, B, H, nc, C, D, v2: Optional[bool] = None,
                 templates: Optional[List[Template]] = None) -> None:
        self.dims = Dims(B, H, nc, C, D, v2)
        self.templates = templates if templates is not None else default_templates()

    def _hits(self, program: Program):
        out = []
        for i, n in enumerate(program.nodes):
            if isinstance(n, EinsumNode):
                unit = extract_epilogue_unit(program, i)
                t = next((t for t in self.templates if t.matches(program, unit)), None)
                if t is not None:
                    out.append((i, t))
        return out

    def match(self, program: Program) -> int:
        return len(self._hits(program))

    def apply(self, program: Program) -> TransformResult:
        fired, prog = [], program
        while True:
            hits = self._hits(prog)
            if not hits:
                break
            i, t = hits[0]
            node, drop = t.emit(prog, extract_epilogue_unit(prog, i), self.dims)
            prog = splice(prog, drop, min(drop), [node])
            fired.append(t.name)
        return TransformResult(prog, bool(fired), len(fired),
                               "emitted: " + (", ".join(fired) if fired else "none"))


class FuseChunkOFlash(Transform):
    """chunk_o q k^T -> gate/mask -> v as one qkv_flash_native_v2 node."""
    name = "fuse-chunk-o-flash"
    summary = "chunk_o q k^T -> gate/mask -> v -> one qkv_flash_native_v2"

    def __init__(self, B, H, nc, C, D) -> None:
        self.dims = Dims(B, H, nc, C, D)

    def _site(self, program: Program):
        for i, n in enumerate(program.nodes):
            if not (isinstance(n, EinsumNode) and n.equation == "nid,njd->nij"
                    and n.inputs == ["qF", "kF"]):
                continue
            unit = extract_epilogue_unit(program, i)
            if unit.epilogue_ops != ["mul", "contiguous"] or _coef(unit, "mul") != "coef_o":
                continue
            c = _only_consumer(program, unit.boundary_out)
            if c is None:
                continue
            cn = program.nodes[c]
            if isinstance(cn, EinsumNode) and cn.equation == "nij,nje->nie" \
                    and cn.inputs[0] == unit.boundary_out:
                return i, unit, c
        return None

    def match(self, program: Program) -> int:
        return int(self._site(program) is not None)

    def apply(self, program: Program) -> TransformResult:
        site = self._site(program)
        if site is None:
            return TransformResult(program, False, 0, "no chunk_o score -> output chain")
        i, unit, c = site
        o_intra = program.nodes[c]
        d = self.dims
        node = FusedNode(kernel="qkv_flash_native_v2",
                         inputs=["qF", "kF", o_intra.inputs[1], "g_native", "beta_native_ones"],
                         outputs=[o_intra.output],
                         params={"nc": d.nc, "H": d.H, "B": d.B, "C": d.C, "D": d.D, "DV": d.D,
                                 "causal": True},
                         subsumes=["Aqk einsum + coef_o mul + contiguous + o_intra A v"])
        drop = {i, c} | {j for j, _ in unit.epilogue}
        return TransformResult(splice(program, drop, min(drop), [node]), True, 1,
                               "emitted qkv_flash_native_v2")


class FusePerDimChunkOFlash(Transform):
    """Per-dim (KDA) chunk_o score -> output in one ``qkvp_flash_native_v2`` launch: the
    gated score ``tril((qF coef_ag)(kF coef_bg)^T, 0)`` never reaches HBM (the
    reference's transform of that name, src/pto_fuser/template.py:335-397). The site is
    the per-dim prologue unit (as ``PerDimPrologueTemplate`` matches it) whose only
    consumer is the o_intra ``nij,nje->nie`` contraction; the score einsum, its
    ``tril -> contiguous`` epilogue and that contraction are replaced, the k-side
    prescale too when nothing else reads it (the q-side one feeds o_inter)."""
    name = "fuse-perdim-chunk-o-flash"
    summary = "per-dim chunk_o prescale, q k^T, tril, A v -> one qkvp_flash_native_v2"

    def __init__(self, B, H, nc, C, D) -> None:
        self.dims = Dims(B, H, nc, C, D)

    def _site(self, program: Program):
        probe = PerDimPrologueTemplate()
        for i, n in enumerate(program.nodes):
            if not isinstance(n, EinsumNode):
                continue
            unit = extract_epilogue_unit(program, i)
            if not probe.matches(program, unit):
                continue
            c = _only_consumer(program, unit.boundary_out)
            if c is None:
                continue
            cn = program.nodes[c]
            if (isinstance(cn, EinsumNode) and cn.equation == "nij,nje->nie"
                    and cn.inputs[0] == unit.boundary_out):
                return i, unit, c
        return None

    def match(self, program: Program) -> int:
        return int(self._site(program) is not None)

    def apply(self, program: Program) -> TransformResult:
        site = self._site(program)
        if site is None:
            return TransformResult(program, False, 0, "no per-dim chunk_o score -> output chain")
        i, unit, c = site
        o_intra = program.nodes[c]
        d = self.dims
        node = FusedNode(kernel="qkvp_flash_native_v2",
                         inputs=["qF", "kF", o_intra.inputs[1], "coef_ag", "coef_bg"],
                         outputs=[o_intra.output],
                         params={"nc": d.nc, "H": d.N, "C": d.C, "D": d.D, "DV": d.D,
                                 "causal": True},
                         subsumes=["chunk_o k-side gate mul + Aqk einsum + tril + contiguous + "
                                   "o_intra A v"])
        drop = {i, c} | {j for j, _ in unit.epilogue}
        k_mul = unit.prologue[unit.anchor.inputs[1]][0]
        if _only_consumer(program, program.nodes[k_mul].output) == i:
            drop.add(k_mul)
        return TransformResult(splice(program, drop, min(drop), [node]), True, 1,
                               "emitted qkvp_flash_native_v2")


@dataclass
class EpilogueReport:
    rows: List[Tuple[str, str, str]] = field(default_factory=list)

    def __str__(self) -> str:
        lines = ["contraction-epilogue units (template = proven fused kernel):"]
        for anchor, epi, verdict in self.rows:
            lines.append(f"  {anchor:<12} epilogue[{epi:<22}] -> {verdict}")
        hit = sum(v.startswith("template ") for _, _, v in self.rows)
        lines.append(f"  -- {hit}/{len(self.rows)} contractions match a proven template")
        return "\n".join(lines)


def epilogue_report(program: Program, templates: Optional[List[Template]] = None) -> EpilogueReport:
    templates = templates if templates is not None else default_templates()
    rep = EpilogueReport()
    for i, n in enumerate(program.nodes):
        if not isinstance(n, EinsumNode):
            continue
        unit = extract_epilogue_unit(program, i)
        t = next((t for t in templates if t.matches(program, unit)), None)
        rep.rows.append((n.output, "+".join(unit.epilogue_ops) or "(none)",
                         f"template {t.name}" if t else "staged (no matching template)"))
    return rep
