"""What ``compile_program`` did with each proposal.

One ``TransformRecord`` per transform the policy proposed: the cost model's
prediction, whether the rewrite matched, and (verified compiles) the measured error,
determinism and replay times that decided it. ``CompilationReport`` collects them.
Field names follow the reference's report (src/pto_fuser/report.py:15-63), which
callers read; the text rendering is this package's own.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional


@dataclass
class TransformRecord:
    name: str
    summary: str
    predicted_benefit: float
    predicted_rationale: str
    matched: bool
    attempted: bool
    kept: bool
    frob: Optional[float] = None
    deterministic: Optional[bool] = None
    faster: Optional[bool] = None
    t_base_ms: Optional[float] = None
    t_cand_ms: Optional[float] = None
    note: str = ""

    @property
    def speedup(self) -> Optional[float]:
        """Replay time of the program before the rewrite over the time after it."""
        if not (self.t_base_ms and self.t_cand_ms):
            return None
        return self.t_base_ms / self.t_cand_ms

    @property
    def outcome(self) -> str:
        if self.kept:
            return "kept"
        return "rejected" if self.attempted else "skipped"

    def __str__(self) -> str:
        parts = [f"{self.outcome:<8}", f"{self.name:<28}",
                 f"predicted {self.predicted_benefit:+.2f}"]
        if self.speedup is not None:
            parts.append(f"measured {self.t_base_ms:.3f} -> {self.t_cand_ms:.3f} ms "
                         f"(x{self.speedup:.2f})")
            parts.append(f"err {self.frob:.1e}")
            parts.append("deterministic" if self.deterministic else "NOT deterministic")
        elif self.note:
            parts.append(f"({self.note})")
        return "  ".join(parts)


@dataclass
class CompilationReport:
    features: object
    records: List[TransformRecord] = field(default_factory=list)
    verified: bool = False

    @property
    def kept(self) -> List[TransformRecord]:
        return [r for r in self.records if r.kept]

    def __str__(self) -> str:
        mode = "measured on the device" if self.verified else "not verified"
        lines = [f"compilation ({mode}): kept {len(self.kept)} of {len(self.records)} "
                 f"proposed transforms"]
        lines += ["  " + str(r) for r in self.records]
        return "\n".join(lines)
