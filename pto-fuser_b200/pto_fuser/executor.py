"""Staged executor: runs a Program node by node on the current CUDA stream.

Same interface as the reference (src/pto_fuser/executor.py:87-181). Einsum nodes
are contractions computed by torch in fp32 and cast to ``out_dtype`` (the reference
library also returns fp32, executor.py:123-127); glue accumulates in fp32; opaque and
fused nodes dispatch to the registries (sm_100a kernels). This is the canonical
floor every transformed program is gated against.
"""
from __future__ import annotations

import contextlib
from typing import Callable, Dict, Optional

import torch

from .fused import FusedKernelRegistry, shared_fused_registry
from .ir import EinsumNode, FusedNode, OpaqueNode, Program, TensorOp, VecGlueNode
from .registry import OpaqueRegistry, default_registry

_TRIL_MASKS: Dict[tuple, torch.Tensor] = {}


def _tril_mask(rows: int, cols: int, diagonal: int, device, dtype) -> torch.Tensor:
    key = (rows, cols, diagonal, device, dtype)
    m = _TRIL_MASKS.get(key)
    if m is None:
        r = torch.arange(rows, device=device).unsqueeze(1)
        c = torch.arange(cols, device=device).unsqueeze(0)
        m = (c <= r + diagonal).to(dtype)
        _TRIL_MASKS[key] = m
    return m


@contextlib.contextmanager
def library_modes(read_mode: str = "auto", fuse_out: bool = True):
    """Kept for interface compatibility with the reference (executor.py:47-71),
    where it toggled the pto-einsum read-mode environment. torch's CUDA contraction
    has no such modes, so this context changes nothing."""
    yield


def _torch_einsum(eq: str, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return torch.einsum(eq, a.float(), b.float())


def _cast(t: torch.Tensor, dtype) -> torch.Tensor:
    return t if dtype is None or t.dtype == dtype else t.to(dtype)


class StagedExecutor:
    def __init__(self, registry: Optional[OpaqueRegistry] = None,
                 einsum_fn: Optional[Callable] = None,
                 fused: Optional[FusedKernelRegistry] = None) -> None:
        self.registry = registry or default_registry()
        self.fused = fused or shared_fused_registry()
        self.einsum = einsum_fn or _torch_einsum

    def run(self, program: Program, bindings: Dict[str, torch.Tensor],
            return_env: bool = False) -> Dict[str, torch.Tensor]:
        missing = [n for n in program.inputs if n not in bindings]
        if missing:
            raise ValueError(f"missing bindings for inputs: {missing}")
        env: Dict[str, torch.Tensor] = dict(bindings)
        for node in program.nodes:
            res = self._exec(node, env)
            if isinstance(res, dict):
                env.update(res)
            else:
                env[node.output] = res
        return env if return_env else {n: env[n] for n in program.outputs}

    def _exec(self, node, env):
        if isinstance(node, EinsumNode):
            a, b = (env[n] for n in node.inputs)
            return _cast(self.einsum(node.equation, a, b), node.out_dtype)
        if isinstance(node, OpaqueNode):
            return self.registry.run(node.kernel, [env[n] for n in node.inputs], node.params)
        if isinstance(node, FusedNode):
            outs = self.fused.run(node.kernel, [env[n] for n in node.inputs], node.params)
            return dict(zip(node.outputs, outs))
        if isinstance(node, VecGlueNode):
            return self._glue(node, env)
        if isinstance(node, TensorOp):
            return self._tensorop(node, env)
        raise TypeError(f"unknown node type: {type(node).__name__}")

    def _glue(self, node: VecGlueNode, env):
        ins = [env[n].float() for n in node.inputs]
        op, p = node.op, node.params
        if op == "tril":
            x = ins[0]
            out = x * _tril_mask(x.shape[-2], x.shape[-1], p.get("diagonal", 0), x.device, x.dtype)
        elif op == "add":
            out = ins[0] + ins[1]
        elif op == "sub":
            out = ins[0] - ins[1]
        elif op == "mul":
            out = ins[0] * ins[1]
        elif op == "scale":
            out = ins[0] * p["scalar"]
        else:
            raise ValueError(f"unknown glue op {op!r}")
        return _cast(out, node.out_dtype)

    def _tensorop(self, node: TensorOp, env):
        op, p = node.op, node.params
        if op == "zeros":
            ref = env[node.inputs[0]] if node.inputs else None
            dev = p.get("device") or (ref.device if ref is not None else None)
            return torch.zeros(p["shape"], dtype=p["dtype"], device=dev)
        x = env[node.inputs[0]]
        if op == "reshape":
            return x.reshape(p["shape"])
        if op == "contiguous":
            return x.contiguous()
        if op == "transpose":
            return x.transpose(*p["dims"])
        if op == "permute":
            return x.permute(*p["dims"]).contiguous()
        if op == "cast":
            return x.to(p["dtype"])
        if op == "slice":
            return x.select(p["axis"], p["index"])
        if op == "stack":
            return torch.stack([env[n] for n in node.inputs], dim=p["dim"])
        raise ValueError(f"unknown tensor op {op!r}")
