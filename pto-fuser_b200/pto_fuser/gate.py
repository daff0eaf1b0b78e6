"""Correctness gates: relative Frobenius error under a tolerance, and determinism
(two runs on identical input must be bit-identical). Same contract as the
reference (src/pto_fuser/gate.py:25-69)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict

import torch


def frob_rel(got: torch.Tensor, ref: torch.Tensor) -> float:
    g, r = got.float(), ref.float()
    return (g - r).norm().item() / max(r.norm().item(), 1e-9)


@dataclass
class GateResult:
    name: str
    passed: bool
    detail: str

    def __str__(self) -> str:
        return f"[{'OK' if self.passed else 'FAIL'}] {self.name}: {self.detail}"


def gate_frob_rel(name: str, got: torch.Tensor, ref: torch.Tensor, tol: float) -> GateResult:
    rel = frob_rel(got, ref)
    amax = (got.float() - ref.float()).abs().max().item()
    return GateResult(name, rel < tol, f"frob_rel={rel:.3e} (tol {tol:.1e})  max_abs={amax:.3e}")


def gate_outputs(got: Dict[str, torch.Tensor], ref: Dict[str, torch.Tensor],
                 tol: float) -> list:
    return [gate_frob_rel(n, got[n], ref[n], tol) for n in ref if n in got]


def gate_determinism(run_fn: Callable[[], Dict[str, torch.Tensor]]) -> GateResult:
    a, b = run_fn(), run_fn()
    bad = []
    for n in a:
        if not torch.equal(a[n], b[n]):
            bad.append(f"{n}(d={(a[n].float() - b[n].float()).abs().max().item():.3e})")
    return GateResult("determinism", not bad,
                      "bit-identical across 2 runs" if not bad else "NDET: " + ", ".join(bad))
