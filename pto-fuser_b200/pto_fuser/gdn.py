"""Host side of the fused chunked Gated DeltaNet forward on B200.

``GDNChunkForward`` is a persistent runner bound to one shape: its constructor
calls ``ptof_gdn_fwd_setup`` (library-owned workspace, as ``FusedKernel`` does in
the reference, fused.py:93-115) and ``__call__`` only launches on the current
CUDA stream, so it can be captured in a CUDA graph. ``chunk_gdn_forward`` is the
functional entry point with a per-shape runner cache.

Semantics: gdn_reference (examples/attention/_gdn_full.py:57-97) with the output
scale folded in, plus an optional initial state and the final state.
"""
from __future__ import annotations

import ctypes
from typing import Dict, Optional, Tuple

import torch

from . import native as nv

_LAYOUTS = {"bhtd": nv.LAYOUT_BHTD, "bthd": nv.LAYOUT_BTHD}
_GATES = {"raw": nv.GATE_RAW, "cumsum": nv.GATE_CUMSUM, "none": nv.GATE_NONE}


class GDNChunkForward:
    """One-shape persistent runner of the fused GDN chunk forward."""

    def __init__(self, B: int, H: int, T: int, Dk: int, Dv: int, *,
                 in_dtype=torch.bfloat16, beta_dtype=None, out_dtype=None,
                 gate: str = "raw", layout: str = "bhtd", scale: Optional[float] = None,
                 chunk: int = 64, device=None) -> None:
        self.device = nv.cuda_device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        beta_dtype = beta_dtype or in_dtype
        out_dtype = out_dtype or in_dtype
        self.shape = (B, H, T, Dk, Dv)
        self.in_dtype, self.beta_dtype, self.out_dtype = in_dtype, beta_dtype, out_dtype
        self.gate, self.layout = gate, layout
        self.scale = Dk ** -0.5 if scale is None else float(scale)
        p = nv.GdnParams(B, H, T, chunk, Dk, Dv, nv.dtype_code(in_dtype),
                         nv.dtype_code(beta_dtype), nv.dtype_code(out_dtype),
                         _GATES[gate], _LAYOUTS[layout], self.scale)
        L = nv.lib()
        with torch.cuda.device(self.device):
            self._ws = L.ptof_gdn_fwd_setup(ctypes.byref(p))
        if not self._ws:
            raise nv.NativeError(nv.EINVAL, nv.last_error())

    # logical shapes of the operands in the chosen layout
    def _qshape(self, D):
        B, H, T = self.shape[:3]
        return (B, H, T, D) if self.layout == "bhtd" else (B, T, H, D)

    def _gshape(self):
        B, H, T = self.shape[:3]
        return (B, H, T) if self.layout == "bhtd" else (B, T, H)

    def _check(self, name, t, shape, dtype):
        if t is None:
            raise ValueError(f"{name} is required")
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name} shape {tuple(t.shape)} != expected {tuple(shape)}")
        if t.dtype != dtype:
            raise TypeError(f"{name} dtype {t.dtype} != contract dtype {dtype}")
        if t.device != self.device:
            raise ValueError(f"{name} on {t.device}, runner on {self.device}")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")

    def __call__(self, q, k, v, beta, g, initial_state=None, *, o=None,
                 final_state=None, output_final_state: bool = True
                 ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        B, H, T, Dk, Dv = self.shape
        self._check("q", q, self._qshape(Dk), self.in_dtype)
        self._check("k", k, self._qshape(Dk), self.in_dtype)
        self._check("v", v, self._qshape(Dv), self.in_dtype)
        self._check("beta", beta, self._gshape(), self.beta_dtype)
        if self.gate != "none":
            self._check("g", g, self._gshape(), torch.float32)
        else:
            g = None
        if initial_state is not None:
            self._check("initial_state", initial_state, (B, H, Dk, Dv), torch.float32)
        if o is None:
            o = torch.empty(self._qshape(Dv), device=self.device, dtype=self.out_dtype)
        if output_final_state and final_state is None:
            final_state = torch.empty(B, H, Dk, Dv, device=self.device, dtype=torch.float32)
        rc = nv.lib().ptof_gdn_fwd_exec(
            self._ws, q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr(), nv.ptr(g),
            nv.ptr(initial_state), o.data_ptr(), nv.ptr(final_state),
            nv.stream_handle(self.device))
        nv.check(rc)
        return o, final_state

    def check_status(self) -> None:
        """Synchronise and raise if a bounded device wait of the last launch gave up."""
        nv.check(nv.lib().ptof_check_status(self._ws, nv.stream_handle(self.device)))

    def set_view(self, qk: Tuple[int, int], v: Tuple[int, int], o: Tuple[int, int]) -> None:
        """Strided views for later ``call_view`` launches (ptof_gdn_fwd_set_view): head
        (b, h) of q/k/beta/g starts at token ``b * qk[0] + h * qk[1]`` of its buffer, of v
        at ``b * v[0] + h * v[1]``, of o at ``b * o[0] + h * o[1]``. (0, 0) x 3 restores
        the dense layout."""
        nv.check(nv.lib().ptof_gdn_fwd_set_view(self._ws, int(qk[0]), int(qk[1]), int(v[0]),
                                                 int(v[1]), int(o[0]), int(o[1])))

    def call_view(self, q, k, v, beta, g, initial_state, o, final_state) -> None:
        """Launch on strided views set with ``set_view``: the tensors' data pointers are
        the first tokens of head (0, 0); shapes are the caller's responsibility (the
        runner's B, H, T and the view strides address every element)."""
        for name, t in (("q", q), ("k", k), ("v", v), ("beta", beta), ("o", o)):
            if t.device != self.device:
                raise ValueError(f"{name} on {t.device}, runner on {self.device}")
        rc = nv.lib().ptof_gdn_fwd_exec(
            self._ws, q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr(), nv.ptr(g),
            nv.ptr(initial_state), o.data_ptr(), nv.ptr(final_state),
            nv.stream_handle(self.device))
        nv.check(rc)

    def set_wait_limit(self, ns: int) -> None:
        """Limit of every bounded device wait of later launches, in ns (default 2 s).
        A launch whose wait runs out ends early; ``check_status`` then raises."""
        nv.check(nv.lib().ptof_ws_set_wait_limit(self._ws, int(ns)))

    def close(self) -> None:
        if getattr(self, "_ws", None):
            nv.lib().ptof_gdn_fwd_teardown(self._ws)
            self._ws = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


class KDAChunkForward:
    """One-shape persistent runner of the fused KDA (per-dimension gate) chunk forward
    on the tensor cores: ``ptof_kda_fwd_setup`` once, ``ptof_kda_fwd_exec`` per call
    on the current stream. Semantics of kda_reference (examples/attention/
    _kda_full.py:38-77) with the output scale folded in, plus an optional initial
    state and the final state. q, k, v bf16 [B,H,T,64]; beta [B,H,T]; g fp32
    [B,H,T,64] (per-token, per-dimension log decay)."""

    def __init__(self, B: int, H: int, T: int, D: int = 64, *, beta_dtype=torch.bfloat16,
                 out_dtype=torch.bfloat16, scale: Optional[float] = None, device=None) -> None:
        self.device = nv.cuda_device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.shape = (B, H, T, D)
        self.beta_dtype, self.out_dtype = beta_dtype, out_dtype
        self.scale = D ** -0.5 if scale is None else float(scale)
        p = nv.GdnParams(B, H, T, 64, D, D, nv.BF16, nv.dtype_code(beta_dtype),
                         nv.dtype_code(out_dtype), nv.GATE_RAW, nv.LAYOUT_BHTD, self.scale)
        with torch.cuda.device(self.device):
            self._ws = nv.lib().ptof_kda_fwd_setup(ctypes.byref(p))
        if not self._ws:
            raise nv.NativeError(nv.EUNSUPPORTED, nv.last_error())

    def __call__(self, q, k, v, beta, g, initial_state=None, *, o=None, final_state=None):
        B, H, T, D = self.shape
        for name, t, shape, dt in (("q", q, (B, H, T, D), torch.bfloat16),
                                   ("k", k, (B, H, T, D), torch.bfloat16),
                                   ("v", v, (B, H, T, D), torch.bfloat16),
                                   ("beta", beta, (B, H, T), self.beta_dtype),
                                   ("g", g, (B, H, T, D), torch.float32)):
            if tuple(t.shape) != shape or t.dtype != dt or not t.is_contiguous() \
                    or t.device != self.device:
                raise ValueError(f"{name}: expected contiguous {dt} {shape} on {self.device}, "
                                 f"got {t.dtype} {tuple(t.shape)} on {t.device}")
        if o is None:
            o = torch.empty(B, H, T, D, device=self.device, dtype=self.out_dtype)
        if final_state is None:
            final_state = torch.empty(B, H, D, D, device=self.device, dtype=torch.float32)
        rc = nv.lib().ptof_kda_fwd_exec(
            self._ws, q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr(), g.data_ptr(),
            nv.ptr(initial_state), o.data_ptr(), final_state.data_ptr(),
            nv.stream_handle(self.device))
        nv.check(rc)
        return o, final_state

    def check_status(self) -> None:
        nv.check(nv.lib().ptof_check_status(self._ws, nv.stream_handle(self.device)))

    def close(self) -> None:
        if getattr(self, "_ws", None):
            nv.lib().ptof_gdn_fwd_teardown(self._ws)
            self._ws = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


_RUNNERS: Dict[tuple, GDNChunkForward] = {}


def chunk_gdn_forward(q, k, v, beta, g, *, scale: Optional[float] = None,
                      initial_state=None, output_final_state: bool = True,
                      gate: str = "raw", layout: str = "bhtd", out_dtype=None):
    """Fused chunked GDN forward on the current CUDA device.

    q, k [B,H,T,Dk] and v [B,H,T,Dv] (or [B,T,H,D] with layout="bthd"), beta like
    g [B,H,T]; g fp32 per-token log decay (gate="raw"), chunk-local cumsum
    (gate="cumsum") or ignored (gate="none"). Returns (o, final_state)."""
    if layout == "bhtd":
        B, H, T, Dk = q.shape
    else:
        B, T, H, Dk = q.shape
    Dv = v.shape[-1]
    out_dtype = out_dtype or q.dtype
    sc = Dk ** -0.5 if scale is None else float(scale)
    key = (B, H, T, Dk, Dv, q.dtype, beta.dtype, out_dtype, gate, layout, sc, q.device)
    r = _RUNNERS.get(key)
    if r is None:
        r = GDNChunkForward(B, H, T, Dk, Dv, in_dtype=q.dtype, beta_dtype=beta.dtype,
                            out_dtype=out_dtype, gate=gate, layout=layout, scale=sc,
                            device=q.device)
        _RUNNERS[key] = r
    return r(q, k, v, beta, g, initial_state, output_final_state=output_final_state)


class GDNChunkForwardVarlen:
    """Persistent runner of the variable-length, grouped-query GDN forward.

    Sequences are packed token-major: q, k [T_total, Hg, Dk]; v, o [T_total, H, Dv];
    beta, g [T_total, H]; cu_seqlens int32 [N+1] on the device (every length at most
    ``max_len``). Value head h reads query/key head h // (H // Hg). The workspace is
    sized for N sequences of up to ``max_len`` tokens; ``T_total`` is fixed per runner.
    """

    def __init__(self, N: int, H: int, Hg: int, T_total: int, max_len: int, Dk: int,
                 Dv: int, *, in_dtype=torch.bfloat16, beta_dtype=None, out_dtype=None,
                 gate: str = "raw", scale: Optional[float] = None, device=None) -> None:
        self.device = nv.cuda_device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        beta_dtype = beta_dtype or in_dtype
        out_dtype = out_dtype or in_dtype
        self.dims = (N, H, Hg, T_total, max_len, Dk, Dv)
        self.in_dtype, self.beta_dtype, self.out_dtype, self.gate = (
            in_dtype, beta_dtype, out_dtype, gate)
        self.scale = Dk ** -0.5 if scale is None else float(scale)
        p = nv.GdnVarlenParams(N, H, Hg, T_total, max_len, Dk, Dv, nv.dtype_code(in_dtype),
                               nv.dtype_code(beta_dtype), nv.dtype_code(out_dtype),
                               _GATES[gate], self.scale)
        with torch.cuda.device(self.device):
            self._ws = nv.lib().ptof_gdn_fwd_varlen_setup(ctypes.byref(p))
        if not self._ws:
            raise nv.NativeError(nv.EINVAL, nv.last_error())

    def __call__(self, q, k, v, beta, g, cu_seqlens, initial_state=None, *, o=None,
                 final_state=None) -> Tuple[torch.Tensor, torch.Tensor]:
        N, H, Hg, T_total, _, Dk, Dv = self.dims
        for name, t, shape, dt in (("q", q, (T_total, Hg, Dk), self.in_dtype),
                                   ("k", k, (T_total, Hg, Dk), self.in_dtype),
                                   ("v", v, (T_total, H, Dv), self.in_dtype),
                                   ("beta", beta, (T_total, H), self.beta_dtype),
                                   ("cu_seqlens", cu_seqlens, (N + 1,), torch.int32)):
            if tuple(t.shape) != shape or t.dtype != dt or not t.is_contiguous() \
                    or t.device != self.device:
                raise ValueError(f"{name}: expected contiguous {dt} {shape} on {self.device}, "
                                 f"got {t.dtype} {tuple(t.shape)} on {t.device}")
        if self.gate != "none":
            if g is None or tuple(g.shape) != (T_total, H) or g.dtype != torch.float32:
                raise ValueError("g: expected float32 [T_total, H]")
        else:
            g = None
        if o is None:
            o = torch.empty(T_total, H, Dv, device=self.device, dtype=self.out_dtype)
        if final_state is None:
            final_state = torch.empty(N, H, Dk, Dv, device=self.device, dtype=torch.float32)
        rc = nv.lib().ptof_gdn_fwd_varlen_exec(
            self._ws, q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr(), nv.ptr(g),
            cu_seqlens.data_ptr(), nv.ptr(initial_state), o.data_ptr(), final_state.data_ptr(),
            nv.stream_handle(self.device))
        nv.check(rc)
        return o, final_state

    def check_status(self) -> None:
        nv.check(nv.lib().ptof_check_status(self._ws, nv.stream_handle(self.device)))

    def close(self) -> None:
        if getattr(self, "_ws", None):
            nv.lib().ptof_gdn_fwd_teardown(self._ws)
            self._ws = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass
