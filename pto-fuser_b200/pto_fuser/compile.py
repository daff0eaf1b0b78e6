"""compile_program: propose (policy) / verify (gate + timing) / dispose.

Same contract as src/pto_fuser/compile.py:46-123: the program is canonicalized,
the policy proposes an ordered pipeline, and each proposed rewrite is kept only if
its outputs are within ``tol`` (relative Frobenius) of the canonical program's,
bit-deterministic across two replays, and faster than the current best. Timing runs
each candidate captured as one CUDA graph and measures replays with CUDA events.
Without bindings (or with ``verify=False``) every matching proposal is applied
unverified — the structural path the CPU tests exercise.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

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


def compile_program(program: Program, features: Features, *, policy: Optional[Policy] = None,
                    bindings: Optional[Dict] = None, verify: bool = True, tol: float = 2e-2,
                    iters: int = 30, warmup: int = 5) -> CompileResult:
    policy = policy or Policy()
    canon = canonicalize(program)
    plan = policy.pipeline(canon, features)
    do_verify = verify and bindings is not None
    records, prog = [], canon
    if do_verify:
        ref_out, base_ms, _ = _run_and_time(canon, bindings, iters, warmup)
    for planned in plan:
        t, pred = planned.transform, planned.prediction
        rec = TransformRecord(name=t.name, summary=t.summary, predicted_benefit=pred.benefit,
                              predicted_rationale=pred.rationale, matched=t.match(prog) > 0,
                              attempted=False, kept=False)
        if not rec.matched:
            rec.note = "no match after prior transforms"
            records.append(rec)
            continue
        cand = t.apply(prog).program
        if not do_verify:
            prog = cand
            rec.attempted = rec.kept = True
            rec.note = "applied (unverified)"
            records.append(rec)
            continue
        got, cand_ms, replay = _run_and_time(cand, bindings, iters, warmup)
        worst = max((frob_rel(got[n], ref_out[n]) for n in ref_out if n in got),
                    default=float("inf"))
        det = gate_determinism(replay)
        rec.attempted = True
        rec.frob, rec.deterministic = worst, det.passed
        rec.faster = cand_ms < base_ms
        rec.t_base_ms, rec.t_cand_ms = base_ms, cand_ms
        rec.kept = worst < tol and det.passed and rec.faster
        if rec.kept:
            prog, base_ms = cand, cand_ms
        records.append(rec)
    return CompileResult(prog, CompilationReport(features, records, do_verify))


def _run_and_time(program: Program, bindings: Dict, iters: int, warmup: int):
    """Capture ``program`` as one CUDA graph; (outputs, ms per replay, replay_fn)."""
    import torch
    from .graph import GraphReplayExecutor
    gr = GraphReplayExecutor().capture(program, bindings)
    out = None
    for _ in range(warmup):
        out = gr.replay(bindings)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        gr.replay(bindings, clone=False)
    e1.record()
    torch.cuda.synchronize()
    return out, e0.elapsed_time(e1) / iters, (lambda: gr.replay(bindings))
