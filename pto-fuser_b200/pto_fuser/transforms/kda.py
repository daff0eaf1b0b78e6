"""KDA's resident-state scan lowering: the unrolled per-chunk scan of
``build_kda_program`` becomes one ``chunk_h_scan`` FusedNode with a per-dimension
decay, plus the parallel ``v_new = U - W h`` recompute — the per-channel counterpart of
``LowerResidentScan`` (the reference's transforms/kda.py:19-70)."""
from __future__ import annotations

import torch

from ..ir import EinsumNode, FusedNode, Program, TensorOp, VecGlueNode, node_outputs
from ..transform import Transform, TransformResult, producer_index, splice
from .gdn import _has_fused


class LowerPerDimScan(Transform):
    name = "lower-perdim-scan"
    summary = "unrolled KDA scan -> chunk_h_scan FusedNode (resident S, per-dim decay)"

    def __init__(self, B: int, H: int, nc: int, C: int, D: int,
                 work: torch.dtype = torch.float16) -> None:
        self.B, self.H, self.nc, self.C, self.D, self.work = B, H, nc, C, D, work

    def _region(self, program: Program):
        if _has_fused(program, "chunk_h_scan") or "coef_krest" not in program.inputs:
            return None
        prod = producer_index(program)
        if not {"S0", "h_flat", "vn_flat"} <= set(prod):
            return None
        names = {"S0", "h_bh", "h_flat", "vn_bh", "vn_flat"}
        for c in range(self.nc):
            names |= {f"Wc{c}_s", f"Wc{c}", f"WS{c}", f"Uc{c}", f"vn{c}", f"kc{c}_s", f"kc{c}",
                      f"krc{c}", f"krest{c}", f"dS{c}", f"sc{c}", f"Sd{c}", f"S{c + 1}"}
        drop = {i for i, n in enumerate(program.nodes) if set(node_outputs(n)) & names}
        return (drop, min(drop)) if drop else None

    def match(self, program: Program) -> int:
        return int(self._region(program) is not None)

    def apply(self, program: Program) -> TransformResult:
        region = self._region(program)
        if region is None:
            return TransformResult(program, False, 0, "no canonical KDA scan region")
        drop, at = region
        B, H, nc, C, D, w = self.B, self.H, self.nc, self.C, self.D, self.work
        M = B * H * nc
        new = [VecGlueNode("mul", ["kb5", "coef_krest"], "k_krest", out_dtype=w)]
        # the scan kernel takes token-major [B, nc, C, H, D] operands
        for nm, src in (("sw", "Wb"), ("su", "Ub"), ("sk", "k_krest")):
            new.append(TensorOp("reshape", [src], f"{nm}5", params={"shape": [B, H, nc, C, D]}))
            new.append(TensorOp("permute", [f"{nm}5"], nm, params={"dims": (0, 2, 3, 1, 4)}))
        new += [
            TensorOp("reshape", ["coef_S"], "sdecay", params={"shape": [B, H, nc, D]}),
            FusedNode(kernel="chunk_h_scan", inputs=["sw", "su", "sk", "sdecay"],
                      outputs=["h_out_k", "final_k"],
                      params={"B": B, "H": H, "nc": nc, "perdim_decay": True},
                      subsumes=["nc per-chunk WS / kv contraction pairs + residual glue"]),
            TensorOp("permute", ["h_out_k"], "h_bhn", params={"dims": (0, 2, 1, 3, 4)}),
            TensorOp("reshape", ["h_bhn"], "h_flat", params={"shape": [M, D, D]}),
            EinsumNode("nid,nde->nie", ["W_m", "h_flat"], "WS_all", out_dtype=w,
                       read_mode="NN", fuse_out=False),
            VecGlueNode("sub", ["U_m", "WS_all"], "vn_flat", out_dtype=w),
        ]
        return TransformResult(splice(program, drop, at, new), True, 1,
                               f"per-dim scan of {nc} chunks -> chunk_h_scan (resident state)")
