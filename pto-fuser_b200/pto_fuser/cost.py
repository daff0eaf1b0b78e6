"""Cost model: predicts whether a transform is worth trying on a problem shape.

``Features`` / ``Prediction`` / ``CostModel.predict`` keep the reference interface
(src/pto_fuser/cost.py:29-139). The seeds are set for B200, where the
numbers that matter are:
  * the whole-forward fusion (``fuse-gdn-forward``) replaces ~130 staged nodes with
    one tcgen05 launch that reads q, k, v, beta, g once and writes o once: it is
    HBM-bound and always the first candidate;
  * the partial fusions (resident scan, gated epilogue, chunk_o flash) each remove an
    HBM round trip of an intermediate in the staged chain; they matter only when the
    whole-forward fusion is refused by the verifier;
  * the read-mode / fused-store levers were pto-einsum lowering choices and have no
    effect on B200, so they are predicted not to pay and are not proposed.
The verifier (``compile.py``) measures every proposal; the report records predicted
versus measured so these seeds can be refitted.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass(frozen=True)
class Features:
    B: int
    H: int
    nc: int
    C: int
    D: int
    dtype: torch.dtype = torch.float16
    per_dim_gate: bool = False

    @property
    def T(self) -> int:
        return self.nc * self.C

    @property
    def M(self) -> int:
        return self.B * self.H * self.nc

    @property
    def N(self) -> int:
        return self.B * self.H

    @property
    def regime(self) -> str:
        """launch-bound when there are too few (b, h) pairs to fill the 148 SMs with
        one resident scan each, bandwidth-bound when every SM has a pair, crossover
        between (B200: one pair per SM in the fused forward)."""
        if self.N * 4 < 148:
            return "launch-bound"
        if self.N >= 128:
            return "bandwidth-bound"
        return "crossover"


@dataclass
class Prediction:
    benefit: float
    rationale: str
    v2: Optional[bool] = None

    @property
    def worth_trying(self) -> bool:
        return self.benefit > 0


class CostModel:
    def predict(self, transform_name: str, feat: Features) -> Prediction:
        n = transform_name
        if n == "fuse-gdn-forward":
            ok = feat.C == 64 and feat.D in (64, 128) and not feat.per_dim_gate
            return Prediction(10.0 if ok else 0.0,
                              "one tcgen05 launch for the whole forward (q,k,v,beta,g read once)"
                              if ok else "fused forward supports C=64, D in {64,128}")
        if n in ("lower-resident-scan", "lower-perdim-scan"):
            return Prediction(1.0 + 0.05 * feat.nc,
                              f"keeps S on chip across {feat.nc} chunks")
        if n == "batch-chunk-intra-score":
            return Prediction(0.5 + 0.05 * feat.nc,
                              f"{feat.nc} per-chunk intra scores -> one batched kernel",
                              v2=feat.C * feat.D >= 4096)
        if n == "fuse-chunk-o-flash":
            return Prediction(0.4, "masked score never reaches HBM")
        if n == "fuse-contraction-epilogue":
            return Prediction(0.3 + 0.02 * feat.H, "gated score stays on chip",
                              v2=feat.C * feat.D >= 4096)
        if n in ("enable-direct-reads", "enable-fused-store"):
            return Prediction(0.0, "read-mode levers have no effect on B200 (torch contraction)")
        if n == "fuse-perdim-chunk-o-flash":
            return Prediction(0.4, "per-dim masked score never reaches HBM")
        return Prediction(0.0, "unknown transform - no prediction")
