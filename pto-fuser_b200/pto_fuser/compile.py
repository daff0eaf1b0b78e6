"""``compile_program``: lower a program by the transforms a policy proposes, keeping
each one only when it is measured to be correct, deterministic and faster.

Contract (the reference's compile driver, src/pto_fuser/compile.py:46-102): the
program is first put in canonical form, which is always correct; the policy orders
the transforms it proposes from the cost model's predictions; every proposal that
matches is tried on top of the best program so far. In a verified compile (device
bindings given) a proposal survives only if

* its outputs are within ``tol`` (relative Frobenius) of the CANONICAL program's,
  never of the previous candidate's, so errors cannot accumulate step by step;
* two replays of it agree bit for bit;
* its replay time beats the best program's.

Here each candidate is captured once as a CUDA graph and its replays are timed with
CUDA events. Without bindings, or with ``verify=False``, matching proposals are
applied as they come and the report says they were not verified.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, Optional, Tuple

from .cost import Features
from .gate import frob_rel, gate_determinism
from .ir import Program
from .policy import Policy
from .report import CompilationReport, TransformRecord
from .transform import canonicalize


@dataclass
class CompileResult:
    program: Program
    report: CompilationReport


class _Measured:
    """A program captured as one CUDA graph: its outputs after warm-up, the mean
    replay time, and a function that replays the same graph (for the determinism
    check of exactly this capture)."""

    def __init__(self, program: Program, bindings: Dict, iters: int, warmup: int) -> None:
        import torch
        from .graph import GraphReplayExecutor
        graph = GraphReplayExecutor().capture(program, bindings)
        outputs = None
        for _ in range(max(1, warmup)):
            outputs = graph.replay(bindings)
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record()
        for _ in range(iters):
            graph.replay(bindings, clone=False)
        stop.record()
        torch.cuda.synchronize()
        self.outputs: Dict = outputs
        self.ms: float = start.elapsed_time(stop) / iters
        self.replay: Callable[[], Dict] = lambda: graph.replay(bindings)


def _worst_error(got: Dict, ref: Dict) -> float:
    shared = [n for n in ref if n in got]
    if not shared:
        return float("inf")          # a candidate that lost every output never passes
    return max(frob_rel(got[n], ref[n]) for n in shared)


def compile_program(program: Program, features: Features, *, policy: Optional[Policy] = None,
                    bindings: Optional[Dict] = None, verify: bool = True, tol: float = 2e-2,
                    iters: int = 30, warmup: int = 5) -> CompileResult:
    policy = policy or Policy()
    canonical = canonicalize(program)
    proposals = policy.pipeline(canonical, features)
    measuring = bool(verify and bindings is not None)

    current = canonical
    reference: Optional[_Measured] = None
    best_ms = float("inf")
    if measuring:
        reference = _Measured(canonical, bindings, iters, warmup)
        best_ms = reference.ms

    records = []
    for proposal in proposals:
        tr = proposal.transform
        rec = TransformRecord(name=tr.name, summary=tr.summary,
                              predicted_benefit=proposal.prediction.benefit,
                              predicted_rationale=proposal.prediction.rationale,
                              matched=tr.match(current) > 0, attempted=False, kept=False)
        records.append(rec)
        if not rec.matched:
            rec.note = "does not match the program at this point"
            continue
        candidate = tr.apply(current).program
        rec.attempted = True
        if not measuring:
            rec.kept = True
            rec.note = "applied without verification"
            current = candidate
            continue
        trial = _Measured(candidate, bindings, iters, warmup)
        rec.frob = _worst_error(trial.outputs, reference.outputs)
        rec.deterministic = gate_determinism(trial.replay).passed
        rec.t_base_ms, rec.t_cand_ms = best_ms, trial.ms
        rec.faster = trial.ms < best_ms
        rec.kept = rec.frob < tol and rec.deterministic and rec.faster
        if rec.kept:
            current, best_ms = candidate, trial.ms
    return CompileResult(current, CompilationReport(features, records, measuring))
