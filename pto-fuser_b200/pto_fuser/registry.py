"""Opaque-kernel registry: foreign kernels hosted by key with a pinned contract.

Mirrors the reference interface (src/pto_fuser/registry.py:37-90): ``register`` /
``contract`` / ``run``, ``KeyError`` for an unknown key, ``ValueError`` for a
duplicate, and the ``capture_mode()`` context. The seed entry
``tri_inv_rec_unroll`` — (I + A)^-1 of a strictly-lower A — runs the sm_100a
``ptof_tri_inv_exec`` kernel on the current CUDA stream. The reference needed host
synchronisations around its raw launch (registry.py:122-126); a CUDA launch on the
torch stream is already ordered, so the lowering never synchronises and
``capture_mode`` only records that a graph capture is in progress.
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional

import torch

from . import native as nv

_CAPTURE_MODE = False


@contextlib.contextmanager
def capture_mode():
    """Mark a region as graph capture (nests; restored on exit or exception)."""
    global _CAPTURE_MODE
    prev = _CAPTURE_MODE
    _CAPTURE_MODE = True
    try:
        yield
    finally:
        _CAPTURE_MODE = prev


@dataclass
class OpaqueContract:
    in_dtypes: List[Any]
    out_dtype: Any
    notes: str = ""


@dataclass
class _Entry:
    factory: Callable[[], Callable]
    lowering: Callable
    contract: OpaqueContract
    _raw: Optional[Callable] = field(default=None, repr=False)

    def callable(self) -> Callable:
        if self._raw is None:
            self._raw = self.factory()
        return self._raw


class OpaqueRegistry:
    def __init__(self) -> None:
        self._entries: Dict[str, _Entry] = {}

    def register(self, key: str, *, factory: Callable, lowering: Callable,
                 contract: OpaqueContract) -> None:
        if key in self._entries:
            raise ValueError(f"opaque kernel {key!r} already registered")
        self._entries[key] = _Entry(factory, lowering, contract)

    def contract(self, key: str) -> OpaqueContract:
        return self._entries[key].contract

    def run(self, key: str, inputs: List[torch.Tensor], params: dict) -> torch.Tensor:
        if key not in self._entries:
            raise KeyError(f"no opaque kernel registered under {key!r}")
        e = self._entries[key]
        return e.lowering(e.callable(), inputs, params)


# ----------------------------------------------------------- tri_inv_rec_unroll ----
def _tri_inv_factory() -> Callable:
    return nv.lib().ptof_tri_inv_exec


def _tri_inv_lowering(tri_inv: Callable, inputs: List[torch.Tensor], params: dict) -> torch.Tensor:
    """(I + A)^-1 per matrix for strictly-lower A [M, C, C]; fp16 in (the contract
    cast, as the reference applies it), fp32 out."""
    (A,) = inputs
    A = A.half().contiguous()
    M, C, _ = A.shape
    out = torch.empty(M, C, C, device=A.device, dtype=torch.float32)
    nv.check(tri_inv(None, A.data_ptr(), nv.F16, out.data_ptr(), M, C,
                     nv.stream_handle(A.device)))
    return out


def default_registry() -> OpaqueRegistry:
    reg = OpaqueRegistry()
    reg.register("tri_inv_rec_unroll", factory=_tri_inv_factory, lowering=_tri_inv_lowering,
                 contract=OpaqueContract(
                     in_dtypes=[torch.float16], out_dtype=torch.float32,
                     notes="strictly-lower A [M,C,C] -> (I+A)^-1 fp32; C <= 128 (sm_100a)"))
    return reg
