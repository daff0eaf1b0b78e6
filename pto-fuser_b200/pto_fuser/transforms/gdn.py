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


class _ResidentScanRewrite(Transform):
    """Shared rewrite of an unrolled chunk scan into one resident-state scan key.

    The canonical builders unroll the inter-chunk recurrence: per chunk c they emit
    W S_c, v_new = U - W S_c, a key scaling, the (k')^T v_new update and the decayed
    state S_{c+1}, then stack the states (``h_flat``) and the v_new (``vn_flat``). On
    the device the recurrence belongs in one kernel that keeps S on chip, so the whole
    per-chunk block is replaced by:

      k' = kb5 * <key coefficient>        (the decay from each token to the chunk end)
      [W, U, k'] -> token-major [B, nc, C, H, D] views
      chunk_h_scan(W, U, k', decay)     -> every chunk's entry state and the final one
      h_flat = entry states as [M, D, D]; vn_flat = U - W h_flat (all chunks at once)

    Subclasses name the program input that identifies the forward, the per-chunk node
    names to drop (format strings of the chunk index c and c1 = c + 1), the key coefficient, the decay's shape and whether it is per key
    dimension."""

    key_coef: str
    chunk_names: tuple
    perdim: bool

    def __init__(self, B: int, H: int, nc: int, C: int, D: int,
                 work: torch.dtype = torch.float16) -> None:
        self.B, self.H, self.nc, self.C, self.D, self.work = B, H, nc, C, D, work

    def _region(self, program: Program):
        if _has_fused(program, "chunk_h_scan") or self.key_coef not in program.inputs:
            return None
        made = set(producer_index(program))
        if not {"S0", "h_flat", "vn_flat"} <= made:
            return None
        doomed = {"S0", "h_bh", "h_flat", "vn_bh", "vn_flat"}
        doomed.update(n.format(c=c, c1=c + 1) for c in range(self.nc) for n in self.chunk_names)
        drop = {i for i, n in enumerate(program.nodes) if doomed.intersection(node_outputs(n))}
        return (drop, min(drop)) if drop else None

    def match(self, program: Program) -> int:
        return int(self._region(program) is not None)

    def apply(self, program: Program) -> TransformResult:
        region = self._region(program)
        if region is None:
            return TransformResult(program, False, 0, f"{self.name}: no unrolled scan")
        drop, at = region
        B, H, nc, C, D, w = self.B, self.H, self.nc, self.C, self.D, self.work
        tok_major = lambda src, dst: [
            TensorOp("reshape", [src], dst + "_5d", params={"shape": [B, H, nc, C, D]}),
            TensorOp("permute", [dst + "_5d"], dst, params={"dims": (0, 2, 3, 1, 4)})]
        decay_shape = [B, H, nc, D] if self.perdim else [B, H, nc]
        params = {"B": B, "H": H, "nc": nc}
        if self.perdim:
            params["perdim_decay"] = True
        body = [VecGlueNode("mul", ["kb5", self.key_coef], "scan_k", out_dtype=w)]
        body += tok_major("Wb", "scan_w") + tok_major("Ub", "scan_u") + tok_major("scan_k", "scan_kt")
        body += [
            TensorOp("reshape", ["coef_S"], "scan_decay", params={"shape": decay_shape}),
            FusedNode(kernel="chunk_h_scan", inputs=["scan_w", "scan_u", "scan_kt", "scan_decay"],
                      outputs=["scan_h", "scan_final"], params=params,
                      subsumes=[f"the {nc} unrolled state updates and their glue"]),
            TensorOp("permute", ["scan_h"], "scan_h_bh", params={"dims": (0, 2, 1, 3, 4)}),
            TensorOp("reshape", ["scan_h_bh"], "h_flat", params={"shape": [B * H * nc, D, D]}),
            EinsumNode("nid,nde->nie", ["W_m", "h_flat"], "WS_all", out_dtype=w,
                       read_mode="NN", fuse_out=False),
            VecGlueNode("sub", ["U_m", "WS_all"], "vn_flat", out_dtype=w),
        ]
        kind = "per-dimension " if self.perdim else ""
        return TransformResult(splice(program, drop, at, body), True, 1,
                               f"{nc}-chunk {kind}scan -> chunk_h_scan (state resident)")


class LowerResidentScan(_ResidentScanRewrite):
    """GDN: scalar per-chunk decay (the reference's rewrite of the same name,
    src/pto_fuser/transforms/gdn.py:30-102)."""
    name = "lower-resident-scan"
    summary = "unrolled chunk_h scan -> chunk_h_scan FusedNode (resident S)"
    key_coef = "coef_vcs"
    chunk_names = ("Wc{c}_s", "Wc{c}", "WS{c}", "Uc{c}", "vn{c}", "vcs{c}", "vn2{c}", "kc{c}_s",
                   "kc{c}", "dS{c}", "sc{c}", "Sd{c}", "S{c1}")
    perdim = False


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
