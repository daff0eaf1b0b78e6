"""GDN structural transforms over the canonical program of ``build_gdn_program``.

* ``LowerResidentScan`` — the reference's resident-state rewrite
  (src/pto_fuser/transforms/gdn.py:30-102): the unrolled nc-chunk scan becomes one
  ``chunk_h_scan`` FusedNode plus the parallel ``v_new = U - W h`` recompute.
* ``FuseGDNForward`` — the B200 lowering: the whole forward (cumsum'd gates in,
  ``o`` out) becomes one ``gdn_chunk_fwd`` FusedNode, the fused tcgen05 kernel that
  keeps A, T, W, U, the state and the masked scores on chip.

Both key on the node names the canonical builder documents, as the reference does.
"""
from __future__ import annotations

import torch

from ..ir import EinsumNode, FusedNode, Program, TensorOp, VecGlueNode, node_outputs
from ..transform import Transform, TransformResult, producer_index, splice


def _has_fused(program: Program, prefix: str) -> bool:
    return any(isinstance(n, FusedNode) and n.kernel.startswith(prefix) for n in program.nodes)


class LowerResidentScan(Transform):
    name = "lower-resident-scan"
    summary = "unrolled chunk_h scan -> chunk_h_scan FusedNode (resident S)"

    def __init__(self, B: int, H: int, nc: int, C: int, D: int,
                 work: torch.dtype = torch.float16) -> None:
        self.B, self.H, self.nc, self.C, self.D, self.work = B, H, nc, C, D, work

    def _region(self, program: Program):
        if _has_fused(program, "chunk_h_scan") or "coef_vcs" not in program.inputs:
            return None
        prod = producer_index(program)
        if not {"S0", "h_flat", "vn_flat"} <= set(prod):
            return None
        names = {"S0", "h_bh", "h_flat", "vn_bh", "vn_flat"}
        for c in range(self.nc):
            names |= {f"Wc{c}_s", f"Wc{c}", f"WS{c}", f"Uc{c}", f"vn{c}", f"vcs{c}", f"vn2{c}",
                      f"kc{c}_s", f"kc{c}", f"dS{c}", f"sc{c}", f"Sd{c}", f"S{c + 1}"}
        drop = {i for i, n in enumerate(program.nodes) if set(node_outputs(n)) & names}
        return (drop, min(drop)) if drop else None

    def match(self, program: Program) -> int:
        return int(self._region(program) is not None)

    def apply(self, program: Program) -> TransformResult:
        region = self._region(program)
        if region is None:
            return TransformResult(program, False, 0, "no canonical scan region")
        drop, at = region
        B, H, nc, C, D, w = self.B, self.H, self.nc, self.C, self.D, self.work
        M = B * H * nc
        new = [VecGlueNode("mul", ["kb5", "coef_vcs"], "k_vcs", out_dtype=w)]
        # the scan kernel takes token-major [B, nc, C, H, D] operands
        for nm, src in (("sw", "Wb"), ("su", "Ub"), ("sk", "k_vcs")):
            new.append(TensorOp("reshape", [src], f"{nm}5", params={"shape": [B, H, nc, C, D]}))
            new.append(TensorOp("permute", [f"{nm}5"], nm, params={"dims": (0, 2, 3, 1, 4)}))
        new += [
            TensorOp("reshape", ["coef_S"], "sdecay", params={"shape": [B, H, nc]}),
            FusedNode(kernel="chunk_h_scan", inputs=["sw", "su", "sk", "sdecay"],
                      outputs=["h_out_k", "final_k"], params={"B": B, "H": H, "nc": nc},
                      subsumes=["nc per-chunk WS / kv contraction pairs + residual glue"]),
            TensorOp("permute", ["h_out_k"], "h_bhn", params={"dims": (0, 2, 1, 3, 4)}),
            TensorOp("reshape", ["h_bhn"], "h_flat", params={"shape": [M, D, D]}),
            EinsumNode("nid,nde->nie", ["W_m", "h_flat"], "WS_all", out_dtype=w,
                       read_mode="NN", fuse_out=False),
            VecGlueNode("sub", ["U_m", "WS_all"], "vn_flat", out_dtype=w),
        ]
        return TransformResult(splice(program, drop, at, new), True, 1,
                               f"scan of {nc} chunks -> chunk_h_scan (resident state)")


# names the canonical GDN builder emits for each stage (its documented contract)
_GDN_MARKERS = ("Araw", "A", "T_raw", "W_m", "U_m", "Aqk", "o_intra", "o_s")
_GDN_INPUTS = ("qF", "kF", "vF", "g_native", "beta_native")


class FuseGDNForward(Transform):
    """The whole canonical GDN forward -> one ``gdn_chunk_fwd`` FusedNode.

    Applies to the canonical program and to any partially lowered form of it whose
    only output is ``o`` (every intermediate stays on chip, so no other output may be
    requested). Inputs: qF, kF, vF [M,C,D], g_native [M,C] (chunk-local cumsum),
    beta_native [M,C]; the scale is read from the program's final ``scale`` glue."""

    name = "fuse-gdn-forward"
    summary = "whole GDN forward -> gdn_chunk_fwd FusedNode (one tcgen05 launch)"

    def __init__(self, B: int, H: int, nc: int, C: int, D: int) -> None:
        self.B, self.H, self.nc, self.C, self.D = B, H, nc, C, D

    def _scale(self, program: Program):
        if program.outputs != ["o"] or _has_fused(program, "gdn_chunk_fwd"):
            return None
        if not all(n in program.inputs for n in _GDN_INPUTS):
            return None
        prod = producer_index(program)
        produced = set(prod)
        # the canonical or a lowered form: the score and output stages must be present
        if "o_s" not in produced or not ({"Aqk", "qkv_o"} & produced or "o_intra" in produced):
            return None
        node = program.nodes[prod["o_s"]]
        if not (isinstance(node, VecGlueNode) and node.op == "scale"):
            return None
        return float(node.params["scalar"])

    def match(self, program: Program) -> int:
        return int(self._scale(program) is not None)

    def apply(self, program: Program) -> TransformResult:
        scale = self._scale(program)
        if scale is None:
            return TransformResult(program, False, 0, "no whole GDN forward")
        B, H, nc, C, D = self.B, self.H, self.nc, self.C, self.D
        node = FusedNode(kernel="gdn_chunk_fwd", inputs=list(_GDN_INPUTS), outputs=["o"],
                         params={"B": B, "H": H, "nc": nc, "scale": scale,
                                 "out_dtype": torch.float32},
                         subsumes=["kkt", "tri_inv", "wy", "chunk_h scan", "chunk_o"])
        prog = Program(nodes=[node], inputs=list(program.inputs), outputs=["o"])
        return TransformResult(prog, True, 1, "whole forward -> gdn_chunk_fwd")
