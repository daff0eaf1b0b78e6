"""The cost model's predictions come from B200 measurements.

``pto_fuser/cost_table.json`` was written by ``python -m pto_fuser.calibrate`` on a
B200: every transform alone on the canonical program of a grid of shapes, timed as
the verifier times it, and a per-transform fit of ln(speed-up). These CPU tests check
that the table is the model's source and that the ordering it implies matches the
measured one (the calibration loop the reference's report exists for:
src/pto_fuser/report.py:15-63, src/pto_fuser/cost.py:29-139)."""
import math

import pytest

from pto_fuser.calibrate import fit
from pto_fuser.cost import CostModel, Features, load_table
from pto_fuser.policy import Policy

TABLE = load_table()
pytestmark = pytest.mark.skipif(TABLE is None, reason="no calibration table")


def _feat(p):
    return Features(p["B"], p["H"], p["nc"], p["C"], p["D"], per_dim_gate=p["family"] == "kda")


def test_table_covers_the_gdn_transforms():
    fits = TABLE["fits"]
    for name in ("fuse-gdn-forward", "lower-resident-scan", "fuse-chunk-o-flash",
                 "fuse-contraction-epilogue", "lower-perdim-scan"):
        assert name in fits and fits[name]["points"] >= 3, name
    assert len(TABLE["points"]) >= 30
    assert "B200" in TABLE["device"]


def test_fit_is_reproducible_from_the_points():
    again = fit(TABLE["points"])
    for name, f in TABLE["fits"].items():
        assert again[name]["coef"] == pytest.approx(f["coef"], rel=1e-6, abs=1e-9)


def test_predictions_come_from_the_table():
    m = CostModel()
    p = next(p for p in TABLE["points"] if p["transform"] == "fuse-gdn-forward")
    pred = m.predict("fuse-gdn-forward", _feat(p))
    ln_s = m.predicted_log_speedup("fuse-gdn-forward", _feat(p))
    assert pred.benefit == pytest.approx(ln_s + TABLE["fits"]["fuse-gdn-forward"]["rms_log_residual"])
    assert "B200 fit" in pred.rationale


def test_predicted_best_transform_matches_measured_per_shape():
    """For every measured shape, the transform the fit ranks first is the one that
    measured fastest (or within 10% of it)."""
    m = CostModel()
    shapes = {}
    for p in TABLE["points"]:
        key = (p["family"], p["B"], p["H"], p["nc"], p["C"], p["D"])
        shapes.setdefault(key, []).append(p)
    checked = 0
    for key, pts in shapes.items():
        if len(pts) < 2:
            continue
        best_meas = max(pts, key=lambda p: p["speedup"])
        best_pred = max(pts, key=lambda p: m.predicted_log_speedup(p["transform"], _feat(p)))
        assert best_pred["speedup"] >= 0.9 * best_meas["speedup"], (key, best_pred["transform"],
                                                                    best_meas["transform"])
        checked += 1
    assert checked >= 8


def test_predicted_sign_matches_clear_measurements():
    """Where a transform measured clearly faster (>1.15x) or clearly slower (<0.87x),
    the fit predicts the same direction."""
    m = CostModel()
    clear = [p for p in TABLE["points"] if p["speedup"] > 1.15 or p["speedup"] < 0.87]
    agree = sum((m.predicted_log_speedup(p["transform"], _feat(p)) > 0) == (p["speedup"] > 1)
                for p in clear)
    assert clear and agree >= 0.9 * len(clear), (agree, len(clear))


def test_policy_puts_the_fused_forward_first_on_config_shapes():
    from pto_fuser.forwards import build_gdn_program
    for B, H, nc, D in ((1, 4, 8, 128), (2, 16, 4, 64)):
        prog = build_gdn_program(B, H, nc, 64, D, D ** -0.5)
        plan = Policy().pipeline(prog, Features(B, H, nc, 64, D))
        assert plan and plan[0].name == "fuse-gdn-forward"
        assert math.exp(plan[0].prediction.benefit) > 2.0
