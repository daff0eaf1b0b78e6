"""Calibration of the cost model from B200 measurements.

The reference's cost model ranks transforms from seeded numbers and its compilation
report records predicted against measured speed-ups so the seeds can be refitted
(src/pto_fuser/cost.py:29-139, src/pto_fuser/report.py:15-63). This module closes
that loop on B200:

1. ``measure`` runs, on the GPU, every transform the policy can propose ALONE on the
   canonical program of a grid of shapes (GDN with a scalar gate and KDA with a
   per-dimension gate, C in {32, 64}): canonical and rewritten program are each
   captured as a CUDA graph and their replays timed with CUDA events, exactly as a
   verified ``compile_program`` does. Each point is one measured speed-up.
2. ``fit`` fits, per transform, ``ln(speed-up) = a + b ln(nc) + c ln(N) + d ln(C D)``
   (least squares with a small ridge; N = B H scan chains, nc chunks) to its points,
   and records the box of regressor values it saw (predictions do not extrapolate
   beyond it).
3. ``main`` writes the points and the coefficients to ``cost_table.json`` beside
   this file, which ``CostModel`` loads: a transform's benefit is its predicted
   ln(speed-up), so ``worth_trying`` means "predicted faster than the program
   without it".

Run on a B200: ``python -m pto_fuser.calibrate [--quick]`` (from ``pto-fuser_b200/``).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import time
from typing import Dict, List, Optional, Sequence, Tuple

from .cost import TABLE_PATH, design_row

# (family, B, H, nc, C, D): GDN covers the whole-forward fusion (C = 64) and the
# partial lowerings (every C); KDA covers the per-dimension scan and chunk_o keys.
GRID: Tuple[Tuple[str, int, int, int, int, int], ...] = (
    ("gdn", 1, 2, 4, 64, 128), ("gdn", 1, 4, 8, 64, 128), ("gdn", 2, 8, 8, 64, 128),
    ("gdn", 1, 16, 16, 64, 128), ("gdn", 2, 16, 4, 64, 64), ("gdn", 1, 2, 32, 64, 64),
    ("gdn", 1, 32, 8, 64, 128), ("gdn", 1, 4, 8, 32, 128), ("gdn", 2, 8, 16, 32, 64),
    ("gdn", 4, 8, 8, 32, 128), ("gdn", 1, 2, 16, 32, 64),
    ("kda", 1, 2, 4, 64, 64), ("kda", 1, 8, 8, 64, 64), ("kda", 2, 8, 16, 64, 64),
    ("kda", 1, 16, 4, 64, 128), ("kda", 1, 4, 16, 32, 64), ("kda", 2, 4, 8, 32, 128),
    ("gdn", 1, 4, 8, 128, 128), ("gdn", 2, 8, 4, 128, 64),
    ("kda", 1, 16, 8, 128, 128), ("kda", 1, 4, 4, 128, 64),
)
QUICK = GRID[:3] + GRID[7:8] + GRID[11:13]


def _case(family: str, B: int, H: int, nc: int, C: int, D: int):
    """Canonical program and device bindings of one grid shape."""
    from .forwards import (build_gdn_program, build_kda_program, make_gdn_inputs,
                           make_kda_inputs, prepare_gdn_bindings, prepare_kda_bindings)
    if family == "gdn":
        inp = make_gdn_inputs(B, H, nc, C, D, device="cuda")
        binds = prepare_gdn_bindings(inp["q"], inp["k"], inp["v"], inp["beta"], inp["g_in"])
        return build_gdn_program(B, H, nc, C, D, D ** -0.5), binds
    inp = make_kda_inputs(B, H, nc, C, D, device="cuda")
    return build_kda_program(B, H, nc, C, D, D ** -0.5), prepare_kda_bindings(**inp)


def measure(grid: Sequence[Tuple] = GRID, iters: int = 20, warmup: int = 3,
            log=print) -> List[Dict]:
    """One point per (shape, transform that matches its canonical program): the
    canonical and the rewritten program's replay times, their ratio and the
    rewritten program's error against the canonical outputs."""
    from .compile import _Measured, _worst_error
    from .cost import Features
    from .policy import Policy
    from .transform import canonicalize
    points = []
    for family, B, H, nc, C, D in grid:
        prog, binds = _case(family, B, H, nc, C, D)
        feat = Features(B, H, nc, C, D, per_dim_gate=(family == "kda"))
        canon = canonicalize(prog)
        base = _Measured(canon, binds, iters, warmup)
        for tr in Policy().candidates(feat):
            if tr.match(canon) == 0 or tr.name in ("enable-direct-reads", "enable-fused-store"):
                continue
            try:
                cand = _Measured(tr.apply(canon).program, binds, iters, warmup)
            except (RuntimeError, ValueError) as e:   # a kernel that does not take the shape
                log(f"{family} B{B} H{H} nc{nc} C{C} D{D} {tr.name:<28} unsupported: {e}")
                continue
            pt = {"family": family, "B": B, "H": H, "nc": nc, "C": C, "D": D,
                  "transform": tr.name, "base_ms": base.ms, "cand_ms": cand.ms,
                  "speedup": base.ms / cand.ms,
                  "frob": _worst_error(cand.outputs, base.outputs)}
            points.append(pt)
            log(f"{family} B{B} H{H} nc{nc} C{C} D{D} {tr.name:<28} "
                f"{base.ms:.3f} -> {cand.ms:.3f} ms  x{pt['speedup']:.2f}  err {pt['frob']:.1e}")
    return points


def fit(points: Sequence[Dict], ridge: float = 1e-2) -> Dict[str, Dict]:
    """Per transform: coefficients of ln(speed-up) over ``design_row``, with the
    fit's residual and the number of points."""
    import numpy as np
    by: Dict[str, List[Dict]] = {}
    for p in points:
        by.setdefault(p["transform"], []).append(p)
    out = {}
    for name, pts in sorted(by.items()):
        X = np.array([design_row(p["nc"], p["B"] * p["H"], p["C"], p["D"]) for p in pts])
        y = np.array([math.log(p["speedup"]) for p in pts])
        # ridge on the slopes only (not the intercept): few points per transform
        reg = ridge * np.eye(X.shape[1])
        reg[0, 0] = 0.0
        coef = np.linalg.solve(X.T @ X + reg, X.T @ y)
        resid = float(np.sqrt(np.mean((X @ coef - y) ** 2)))
        out[name] = {"coef": [float(c) for c in coef], "rms_log_residual": resid,
                     "points": len(pts),
                     # the measured box: predictions clamp the regressors to it
                     "x_min": [float(v) for v in X.min(axis=0)],
                     "x_max": [float(v) for v in X.max(axis=0)]}
    return out


def main(argv: Optional[Sequence[str]] = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--quick", action="store_true", help="six shapes instead of the grid")
    ap.add_argument("--out", default=TABLE_PATH)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args(argv)
    import torch
    t0 = time.time()
    points = measure(QUICK if a.quick else GRID, iters=a.iters)
    table = {"how": ("each transform alone on the canonical program, CUDA-graph replays "
                     "timed with CUDA events on one B200 (pto_fuser.calibrate)"),
             "device": torch.cuda.get_device_name(0),
             "regressors": ["1", "ln nc", "ln N", "ln(C D / 4096)"],
             "fits": fit(points), "points": points,
             "seconds": round(time.time() - t0, 1)}
    with open(a.out, "w") as f:
        json.dump(table, f, indent=1)
    print(f"wrote {a.out}: {len(points)} points, {len(table['fits'])} transforms")


if __name__ == "__main__":
    main()
