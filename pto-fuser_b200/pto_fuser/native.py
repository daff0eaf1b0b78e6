"""ctypes binding of the in-tree CUDA library ``_native/libptofuser_gdn.so``.

The library is the B200 replacement of the per-shape Ascend ``.so`` files the
reference compiles and loads in ``fused.py:58-77``: one prebuilt sm_100a library,
shapes passed at run time. There is no fallback: if the library is missing or a
GPU call fails, the caller gets an exception.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_native", "libptofuser_gdn.so")

# status codes / dtype / layout / gate enums (include/pto_fuser_gdn.h)
OK, EINVAL, EALIGN, ECUDA, EUNSUPPORTED, ETIMEOUT = range(6)
F32, F16, BF16 = 0, 1, 2
LAYOUT_BHTD, LAYOUT_BTHD = 0, 1
GATE_RAW, GATE_CUMSUM, GATE_NONE = 0, 1, 2

_DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}


class NativeError(RuntimeError):
    """A non-zero status from the CUDA library (message from ptof_last_error)."""

    def __init__(self, code: int, msg: str) -> None:
        super().__init__(f"[ptof status {code}] {msg}")
        self.code = code


class GdnParams(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int32), ("H", ctypes.c_int32), ("T", ctypes.c_int32),
                ("C", ctypes.c_int32), ("Dk", ctypes.c_int32), ("Dv", ctypes.c_int32),
                ("in_dtype", ctypes.c_int32), ("beta_dtype", ctypes.c_int32),
                ("out_dtype", ctypes.c_int32), ("gate_mode", ctypes.c_int32),
                ("layout", ctypes.c_int32), ("scale", ctypes.c_float)]


class GdnVarlenParams(ctypes.Structure):
    _fields_ = [("N", ctypes.c_int32), ("H", ctypes.c_int32), ("Hg", ctypes.c_int32),
                ("T_total", ctypes.c_int32), ("max_len", ctypes.c_int32),
                ("Dk", ctypes.c_int32), ("Dv", ctypes.c_int32),
                ("in_dtype", ctypes.c_int32), ("beta_dtype", ctypes.c_int32),
                ("out_dtype", ctypes.c_int32), ("gate_mode", ctypes.c_int32),
                ("scale", ctypes.c_float)]


_vp = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_SIGNATURES = {
    "ptof_gdn_fwd_setup": (_vp, [ctypes.POINTER(GdnParams)]),
    "ptof_gdn_fwd_exec": (_i32, [_vp] * 10),
    "ptof_gdn_fwd_teardown": (None, [_vp]),
    "ptof_gdn_fwd_varlen_setup": (_vp, [ctypes.POINTER(GdnVarlenParams)]),
    "ptof_gdn_fwd_varlen_exec": (_i32, [_vp] * 11),
    "ptof_kda_fwd_setup": (_vp, [ctypes.POINTER(GdnParams)]),
    "ptof_kda_fwd_exec": (_i32, [_vp] * 10),
    "ptof_gdn_fwd_exec_noalloc": (_i32, [ctypes.POINTER(GdnParams)] + [_vp] * 9),
    "ptof_gdn_fwd_noalloc_status": (_i32, [_vp]),
    "ptof_seg_scan_exec": (_i32, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _i64,
                                  _vp, _i64, _i32, _i32, _i32, _i32, _vp]),
    "ptof_seg_fix_exec": (_i32, [_vp] * 4 + [_i32] * 4 + [_vp]),
    "ptof_check_status": (_i32, [_vp, _vp]),
    "ptof_gdn_fwd_set_trace": (_i32, [_vp, _vp, _i32]),
    "ptof_ws_set_wait_limit": (_i32, [_vp, ctypes.c_ulonglong]),
    "ptof_gdn_fwd_inject_stall": (_i32, [_vp, _i32]),
    "ptof_gdn_fwd_set_view": (_i32, [_vp] + [ctypes.c_longlong] * 6),
    "ptof_seg_fix_exec_view": (_i32, [_vp] * 4 + [_i32] * 5 + [ctypes.c_longlong] * 2 + [_vp]),
    "ptof_last_error": (ctypes.c_char_p, []),
    "ptof_ws_setup": (_vp, []),
    "ptof_ws_teardown": (None, [_vp]),
    "ptof_gated_qk_exec": (_i32, [_vp] * 6 + [_i32] * 6 + [_vp]),
    "ptof_kkt_inv_exec": (_i32, [_vp] * 5 + [_i32] * 8 + [_vp]),
    "ptof_chunk_h_scan_perdim_exec": (_i32, [_vp] * 7 + [_i32] * 8 + [_vp]),
    "ptof_qk_prologue_exec": (_i32, [_vp] * 6 + [_i32] * 4 + [_vp]),
    "ptof_qkvp_flash_exec": (_i32, [_vp] * 7 + [_i32] * 5 + [_vp]),
    "ptof_tri_inv_exec": (_i32, [_vp, _vp, _i32, _vp, _i32, _i32, _vp]),
    "ptof_chunk_h_scan_exec": (_i32, [_vp] * 7 + [_i32] * 8 + [_vp]),
    "ptof_qkv_flash_exec": (_i32, [_vp] * 6 + [_i32] * 5 + [_vp]),
    "ptof_selftest_umma": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp]),
    "ptof_selftest_umma_rate": (_i32, [_i32, _i32, _i32, _i32, _vp, _vp, _vp]),
    "ptof_selftest_tma": (_i32, [_vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp]),
}

_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load (once) and bind the CUDA library; raise if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"CUDA library not built: {LIB_PATH} is missing "
                        "(build it with `make -C pto-fuser_b200/csrc` or "
                        "`python -c 'import __graft_entry__ as g; g.build()'`)")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def bind(name: str, restype, argtypes) -> None:
    """Declare the signature of an additional exported symbol."""
    _SIGNATURES[name] = (restype, argtypes)
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.restype = restype
        fn.argtypes = argtypes


def last_error() -> str:
    return lib().ptof_last_error().decode(errors="replace")


def check(code: int) -> None:
    if code != OK:
        raise NativeError(code, last_error())


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def cuda_device(device) -> torch.device:
    """``device`` as a torch.device with an explicit index ("cuda" -> the current
    CUDA device), so it compares equal to the devices of tensors allocated on it."""
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return d


def stream_handle(device: Optional[torch.device] = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream
