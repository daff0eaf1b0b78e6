"""Cost model: predicts whether a transform is worth trying on a problem shape.

``Features`` / ``Prediction`` / ``CostModel.predict`` keep the reference interface
(src/pto_fuser/cost.py:29-139). The reference seeds its predictions by hand and
records predicted against measured speed-ups so they can be refitted; here the
predictions ARE the refit: ``pto_fuser.calibrate`` measures every transform alone on
the canonical program of a grid of shapes on a B200 (CUDA-graph replays, CUDA-event
timing, as the verifier does) and fits per transform

    ln(speed-up) = a + b ln(nc) + c ln(N) + d ln(C D / 4096)

into ``cost_table.json`` beside this file. ``predict`` returns that fitted
ln(speed-up) plus the fit's rms residual as the benefit, i.e. a transform is proposed
when it could plausibly pay within the fit's error; the verifier (``compile.py``)
still measures every proposal. What stays hand-written is what the kernels support
(the whole-forward kernel needs C = 64 and D in {64, 128} with a scalar gate), the
``v2`` kernel hints, and the two pto-einsum read-mode levers, which have no effect
on B200 and are never proposed. A transform the table does not cover falls back to
a neutral seed.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass
from typing import Dict, Optional

import torch

TABLE_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "cost_table.json")


def load_table(path: str = TABLE_PATH) -> Optional[Dict]:
    """The committed calibration table, or None when it is absent."""
    try:
        with open(path) as f:
            return json.load(f)
    except OSError:
        return None


def design_row(nc: int, N: int, C: int, D: int):
    """Regressors of the fitted log speed-up (the calibration's ``design_row``)."""
    return [1.0, math.log(nc), math.log(N), math.log(C * D / 4096.0)]


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


# the transforms the policy can propose (policy.Policy.candidates)
_LIBRARY = frozenset({"fuse-gdn-forward", "lower-resident-scan", "lower-perdim-scan",
                      "fuse-chunk-o-flash", "fuse-perdim-chunk-o-flash",
                      "fuse-contraction-epilogue", "batch-chunk-intra-score",
                      "enable-direct-reads", "enable-fused-store"})


class CostModel:
    """Fitted predictor over the transform library (see the module docstring)."""

    def __init__(self, table: Optional[Dict] = None) -> None:
        self.table = load_table() if table is None else table

    def fitted(self, transform_name: str) -> Optional[Dict]:
        return (self.table or {}).get("fits", {}).get(transform_name)

    def predicted_log_speedup(self, transform_name: str, feat: "Features") -> Optional[float]:
        """The calibration fit's ln(speed-up) for this shape, or None if the table
        does not cover the transform."""
        fit = self.fitted(transform_name)
        if fit is None:
            return None
        x = design_row(feat.nc, feat.N, feat.C, feat.D)
        lo, hi = fit.get("x_min"), fit.get("x_max")
        if lo and hi:      # no extrapolation beyond the measured shapes
            x = [min(max(v, a), b) for v, a, b in zip(x, lo, hi)]
        return sum(c * v for c, v in zip(fit["coef"], x))

    def predict(self, transform_name: str, feat: "Features") -> Prediction:
        n = transform_name
        v2 = None
        if n == "fuse-gdn-forward":
            if not (feat.C == 64 and feat.D in (64, 128) and not feat.per_dim_gate):
                return Prediction(0.0, "the fused forward takes C=64, D in {64,128}, scalar gate")
        elif n in ("enable-direct-reads", "enable-fused-store"):
            return Prediction(0.0, "read-mode levers have no effect on B200 (no pto-einsum)")
        elif n in ("batch-chunk-intra-score", "fuse-contraction-epilogue"):
            v2 = feat.C * feat.D >= 4096
        ln_s = self.predicted_log_speedup(n, feat)
        if ln_s is None:
            if n not in _LIBRARY:
                return Prediction(0.0, "unknown transform: no prediction")
            return Prediction(0.05, "not in the calibration table: neutral seed, verifier decides",
                              v2=v2)
        fit = self.fitted(n)
        resid = fit["rms_log_residual"]
        return Prediction(ln_s + resid,
                          f"B200 fit over {fit['points']} measurements: predicted "
                          f"x{math.exp(ln_s):.2f} (rms log residual {resid:.2f})", v2=v2)
