"""Correctness gates of the compile loop.

A rewritten program only replaces the canonical one when two checks pass on the same
inputs (the contract of the reference's gates, src/pto_fuser/gate.py:25-69):

* closeness: the relative Frobenius norm of the difference to the canonical outputs
  stays under a tolerance;
* determinism: two replays of the candidate give bit-identical outputs.

On B200 both run on the device tensors the candidate produced; only the scalars come
back to the host.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List

import torch


def frob_rel(got: torch.Tensor, ref: torch.Tensor) -> float:
    """||got - ref||_F / ||ref||_F, computed in fp32 (the denominator floored at 1e-9
    so an all-zero reference does not divide by zero)."""
    diff = torch.linalg.vector_norm(got.float() - ref.float())
    base = torch.linalg.vector_norm(ref.float()).clamp_min(1e-9)
    return float(diff / base)


@dataclass
class GateResult:
    """Outcome of one check: which tensor or property, pass/fail, and the numbers."""
    name: str
    passed: bool
    detail: str

    def __str__(self) -> str:
        mark = "pass" if self.passed else "FAIL"
        return f"{self.name:<16} {mark}  {self.detail}"


def gate_frob_rel(name: str, got: torch.Tensor, ref: torch.Tensor, tol: float) -> GateResult:
    """Closeness check of one tensor against its reference."""
    err = frob_rel(got, ref)
    worst = float((got.float() - ref.float()).abs().max()) if got.numel() else 0.0
    return GateResult(name, err < tol,
                      f"rel Frobenius error {err:.2e} (limit {tol:.1e}), largest |diff| {worst:.2e}")


def gate_outputs(got: Dict[str, torch.Tensor], ref: Dict[str, torch.Tensor],
                 tol: float) -> List[GateResult]:
    """Closeness check of every output the two runs have in common (in the
    reference's order)."""
    common = [n for n in ref if n in got]
    return [gate_frob_rel(n, got[n], ref[n], tol) for n in common]


def gate_determinism(run_fn: Callable[[], Dict[str, torch.Tensor]]) -> GateResult:
    """Replay twice; every output must match bit for bit."""
    first = run_fn()
    second = run_fn()
    differing = {}
    for name, a in first.items():
        b = second[name]
        if not torch.equal(a, b):
            differing[name] = float((a.float() - b.float()).abs().max())
    if not differing:
        return GateResult("determinism", True, "2 replays agree bit for bit")
    listing = "; ".join(f"{n} max |diff| {d:.2e}" for n, d in differing.items())
    return GateResult("determinism", False, f"replays differ: {listing}")
