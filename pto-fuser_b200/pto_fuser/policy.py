"""Policy: cost model + program -> ordered pipeline of proposed transforms
(interface of src/pto_fuser/policy.py:27-86). Structural fusions come first, the
whole-forward fusion before the partial ones (if it is kept nothing else matches)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

from .cost import CostModel, Features, Prediction
from .ir import Program
from .transform import EnableDirectReads, EnableFusedStore, Transform

_ORDER = {"fuse-gdn-forward": 0, "lower-resident-scan": 1, "lower-perdim-scan": 1,
          "fuse-chunk-o-flash": 2, "fuse-perdim-chunk-o-flash": 2,
          "fuse-contraction-epilogue": 3, "batch-chunk-intra-score": 3,
          "enable-direct-reads": 4, "enable-fused-store": 5}


@dataclass
class PlannedTransform:
    transform: Transform
    prediction: Prediction

    @property
    def name(self) -> str:
        return self.transform.name


class Policy:
    def __init__(self, cost: Optional[CostModel] = None) -> None:
        self.cost = cost or CostModel()

    def candidates(self, feat: Features) -> List[Transform]:
        from .template import FuseChunkOFlash, FuseContractionEpilogue, FusePerDimChunkOFlash
        from .transforms import (BatchChunkIntraScore, FuseGDNForward, LowerPerDimScan,
                                 LowerResidentScan)
        B, H, nc, C, D = feat.B, feat.H, feat.nc, feat.C, feat.D
        v2 = self.cost.predict("fuse-contraction-epilogue", feat).v2
        intra_v2 = self.cost.predict("batch-chunk-intra-score", feat).v2
        return [FuseGDNForward(B, H, nc, C, D), LowerResidentScan(B, H, nc, C, D, feat.dtype),
                LowerPerDimScan(B, H, nc, C, D, feat.dtype),
                FuseChunkOFlash(B, H, nc, C, D), FusePerDimChunkOFlash(B, H, nc, C, D),
                FuseContractionEpilogue(B, H, nc, C, D, v2=v2),
                BatchChunkIntraScore(feat.N, nc, C, D, D, per_dim_gate=feat.per_dim_gate,
                                     v2=intra_v2 if feat.per_dim_gate else None),
                EnableDirectReads(), EnableFusedStore()]

    def pipeline(self, program: Program, feat: Features) -> List[PlannedTransform]:
        plan = []
        for t in self.candidates(feat):
            if t.match(program) == 0:
                continue
            pred = self.cost.predict(t.name, feat)
            if pred.worth_trying:
                plan.append(PlannedTransform(t, pred))
        plan.sort(key=lambda p: _ORDER.get(p.name, 99))
        return plan
