"""Graph-replay backend: capture a Program into one CUDA graph, replay it.

Interface of the reference's NPU-graph backend (src/pto_fuser/graph.py:45-138):
``CaptureExecutor`` and ``GraphReplayExecutor.capture(program, bindings, warmup)`` /
``replay(bindings, clone=True)`` with static input buffers, a shape check that raises
``ValueError``, and ``RuntimeError`` for a replay before capture. On B200 the capture
is a ``torch.cuda.CUDAGraph`` recorded on a side stream after eager warm-up runs
(which also create every persistent kernel runner, so the captured region holds only
kernel launches).
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

from . import registry as _registry
from .executor import StagedExecutor
from .ir import Program
from .registry import OpaqueRegistry


class CaptureExecutor(StagedExecutor):
    """A StagedExecutor used inside capture (every runner is persistent already)."""

    def __init__(self, registry: Optional[OpaqueRegistry] = None) -> None:
        super().__init__(registry)


class GraphReplayExecutor:
    def __init__(self, registry: Optional[OpaqueRegistry] = None) -> None:
        self._exec = CaptureExecutor(registry)
        self._graph: Optional[torch.cuda.CUDAGraph] = None
        self._static_in: Dict[str, torch.Tensor] = {}
        self._out: Dict[str, torch.Tensor] = {}
        self.program: Optional[Program] = None

    def capture(self, program: Program, bindings: Dict[str, torch.Tensor],
                warmup: int = 3) -> "GraphReplayExecutor":
        missing = [n for n in program.inputs if n not in bindings]
        if missing:
            raise ValueError(f"missing bindings for inputs: {missing}")
        self._static_in = {k: bindings[k].clone() for k in program.inputs}
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                self._exec.run(program, self._static_in, return_env=True)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            with _registry.capture_mode():
                env = self._exec.run(program, self._static_in, return_env=True)
        torch.cuda.synchronize()
        self._graph, self.program = graph, program
        self._out = {n: env[n] for n in program.outputs}
        return self

    def replay(self, bindings: Dict[str, torch.Tensor], clone: bool = True) -> Dict[str, torch.Tensor]:
        if self._graph is None:
            raise RuntimeError("capture() must be called before replay()")
        for name, buf in self._static_in.items():
            src = bindings[name]
            if src.shape != buf.shape:
                raise ValueError(f"replay shape {tuple(src.shape)} for {name!r} != captured "
                                 f"{tuple(buf.shape)} (a new shape needs a new capture)")
            buf.copy_(src)
        self._graph.replay()
        return {k: v.clone() for k, v in self._out.items()} if clone else dict(self._out)
