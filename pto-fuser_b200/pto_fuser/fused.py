"""Fused-kernel registry: FusedNode keys -> persistent CUDA runners.

Keeps the reference interface (src/pto_fuser/fused.py:83-162): ``FusedContract``,
``FusedKernel`` (workspace set up once, ``run`` only launches on the current stream,
so it can be captured), ``FusedKernelRegistry.register / contract / kernel / run /
close`` with ``KeyError`` for an unknown key and ``ValueError`` for a duplicate, and
``default_fused_registry`` / ``shared_fused_registry``. The difference is the build
model: the reference compiles one Ascend ``.so`` per shape at first use
(fused.py:58-77); here one prebuilt sm_100a library takes shapes at run time, so a
kernel is cached per (key, device) only.

Registered keys (contract slots as in fused.py:446-569) plus the B200 whole-forward key:

  chunk_h_scan                 resident-state recurrence
  kkt_gated, gated_qk          gated a b^T epilogue, token-major [1,T,H,D] operands
  kkt_gated_native[_v2]        gated k k^T, strict lower, native [M,C,D]
  gated_qk_native[_v2]         gated q k^T, causal, native [M,C,D]
  qkv_flash_native[_v2]        chunk_o score -> output in one launch
  gdn_chunk_fwd                the whole chunked GDN forward in one launch (tcgen05)

The ``_v2`` keys name the reference's second on-chip scheduling of the same math;
on B200 they share the kernel of their base key.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Tuple

import torch

from . import native as nv


@dataclass
class FusedContract:
    in_slots: List[str]
    in_dtypes: List[Any]
    out_names: List[str]
    out_dtype: Any
    notes: str = ""


class FusedKernel:
    """A registered kernel bound to one device with its workspace set up once."""

    def __init__(self, launch: Callable, device: torch.device) -> None:
        self._launch = launch
        self.device = device
        self._ws = nv.lib().ptof_ws_setup()
        if not self._ws:
            raise nv.NativeError(nv.ECUDA, nv.last_error())

    def run(self, inputs: List[torch.Tensor], params: dict) -> List[torch.Tensor]:
        return self._launch(self._ws, inputs, params)

    def close(self) -> None:
        if self._ws:
            nv.lib().ptof_ws_teardown(self._ws)
            self._ws = None


@dataclass
class _Recipe:
    launch: Callable              # (ws, inputs, params) -> [outputs]
    contract: FusedContract


class FusedKernelRegistry:
    def __init__(self) -> None:
        self._recipes: Dict[str, _Recipe] = {}
        self._cache: Dict[Tuple, FusedKernel] = {}

    def register(self, key: str, recipe: _Recipe) -> None:
        if key in self._recipes:
            raise ValueError(f"fused kernel {key!r} already registered")
        self._recipes[key] = recipe

    def keys(self) -> List[str]:
        return list(self._recipes)

    def contract(self, key: str) -> FusedContract:
        return self._recipes[key].contract

    def kernel(self, key: str, params: dict, device=None) -> FusedKernel:
        if key not in self._recipes:
            raise KeyError(f"no fused kernel registered under {key!r}")
        dev = nv.cuda_device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        ck = (key, dev)
        if ck not in self._cache:
            self._cache[ck] = FusedKernel(self._recipes[key].launch, dev)
        return self._cache[ck]

    def run(self, key: str, inputs: List[torch.Tensor], params: dict) -> List[torch.Tensor]:
        dev = inputs[0].device if inputs else None
        return self.kernel(key, params, dev).run(inputs, params)

    def close(self) -> None:
        for k in self._cache.values():
            k.close()
        self._cache.clear()


# ------------------------------------------------------------------ launchers ----
def _c(t: torch.Tensor, dtype=None) -> torch.Tensor:
    t = t if dtype is None or t.dtype == dtype else t.to(dtype)
    return t.contiguous()


def _scan_launch(ws, inputs, params) -> List[torch.Tensor]:
    """w, u, k [B,nc,C,H,D] (cast fp16 per contract), decay [B,H,nc] fp32, or
    [B,H,nc,D] with params perdim_decay (the KDA scan)."""
    w, u, k, decay = inputs
    B, H, nc = params["B"], params["H"], params["nc"]
    w, u, k = _c(w, torch.float16), _c(u, torch.float16), _c(k, torch.float16)
    C, D, Dv = w.shape[2], w.shape[4], u.shape[4]
    perdim = bool(params.get("perdim_decay", False))
    decay = _c(decay.reshape((B, H, nc, D) if perdim else (B, H, nc)), torch.float32)
    h_out = torch.empty(B, nc, H, D, Dv, device=w.device, dtype=torch.float16)
    final = torch.empty(B, H, D, Dv, device=w.device, dtype=torch.float16)
    fn = nv.lib().ptof_chunk_h_scan_perdim_exec if perdim else nv.lib().ptof_chunk_h_scan_exec
    nv.check(fn(
        ws, w.data_ptr(), u.data_ptr(), k.data_ptr(), decay.data_ptr(), h_out.data_ptr(),
        final.data_ptr(), B, H, nc, C, D, Dv, nv.F16, nv.F16, nv.stream_handle(w.device)))
    return [h_out, final]


def _gated_qk(ws, a, b, g, beta, M, C, D, causal) -> torch.Tensor:
    a, b = _c(a, torch.float16).reshape(M, C, D), _c(b, torch.float16).reshape(M, C, D)
    g = _c(g, torch.float32).reshape(M, C)
    beta = _c(beta, torch.float16).reshape(M, C)
    L = torch.empty(M, C, C, device=a.device, dtype=torch.float16)
    nv.check(nv.lib().ptof_gated_qk_exec(ws, a.data_ptr(), b.data_ptr(), g.data_ptr(),
                                         beta.data_ptr(), L.data_ptr(), M, C, D, nv.F16, nv.F16,
                                         int(causal), nv.stream_handle(a.device)))
    return L


def _to_native(x: torch.Tensor, nc: int, C: int) -> torch.Tensor:
    """token-major [1, T, H, ...] -> native [H*nc, C, ...] (heads outer)."""
    T, H = x.shape[1], x.shape[2]
    rest = x.shape[3:]
    return x[0].reshape(nc, C, H, *rest).permute(2, 0, 1, *range(3, 3 + len(rest))) \
        .reshape(H * nc, C, *rest).contiguous()


def _mega_launch(ws, inputs, params, causal) -> List[torch.Tensor]:
    if len(inputs) == 3:
        a, g_sum, beta = inputs
        b = a
    else:
        a, b, g_sum, beta = inputs
    nc, H = params["nc"], params["H"]
    C = a.shape[1] // nc
    D = a.shape[-1]
    L = _gated_qk(ws, _to_native(a, nc, C), _to_native(b, nc, C), _to_native(g_sum, nc, C),
                  _to_native(beta, nc, C), H * nc, C, D, causal)
    # [H*nc, C, C] -> [T, H, C] (the reference's mega output layout)
    return [L.reshape(H, nc, C, C).permute(1, 2, 0, 3).reshape(nc * C, H, C).contiguous()]


def _native_launch(ws, inputs, params, causal) -> List[torch.Tensor]:
    if len(inputs) == 3:
        a, g, beta = inputs
        b = a
    else:
        a, b, g, beta = inputs
    C, D = a.shape[-2], a.shape[-1]
    M = a.numel() // (C * D)
    return [_gated_qk(ws, a, b, g, beta, M, C, D, causal)]


def _qkv_launch(ws, inputs, params) -> List[torch.Tensor]:
    q, k, v, g, _beta = inputs
    C, D, Dv = q.shape[-2], q.shape[-1], v.shape[-1]
    M = q.numel() // (C * D)
    q, k = _c(q, torch.float16).reshape(M, C, D), _c(k, torch.float16).reshape(M, C, D)
    v = _c(v, torch.float16).reshape(M, C, Dv)
    g = _c(g, torch.float32).reshape(M, C)
    o = torch.empty(M, C, Dv, device=q.device, dtype=torch.float32)
    nv.check(nv.lib().ptof_qkv_flash_exec(ws, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                          g.data_ptr(), o.data_ptr(), M, C, D, Dv, nv.F16,
                                          nv.stream_handle(q.device)))
    return [o]


def _prologue_launch(ws, inputs, params) -> List[torch.Tensor]:
    """q, k, P, invP [., C, D] over M = nc * H chunks -> L = tril((q*P)(k*invP)^T) [M,C,C]
    fp16 (the per-channel-gate intra score; reference fused.py:303-311)."""
    q, k, P, invP = inputs
    C, D = params.get("C", q.shape[-2]), params.get("D", q.shape[-1])
    M = params["nc"] * params["H"]
    rs = lambda t: _c(t, torch.float16).reshape(M, C, D)
    q, k, P, invP = rs(q), rs(k), rs(P), rs(invP)
    L = torch.empty(M, C, C, device=q.device, dtype=torch.float16)
    nv.check(nv.lib().ptof_qk_prologue_exec(ws, q.data_ptr(), k.data_ptr(), P.data_ptr(),
                                            invP.data_ptr(), L.data_ptr(), M, C, D, nv.F16,
                                            nv.stream_handle(q.device)))
    return [L]


def _qkvp_launch(ws, inputs, params) -> List[torch.Tensor]:
    """q, k, v, coef_ag, coef_bg over M = nc * H chunks -> o = tril((q*coef_ag)
    (k*coef_bg)^T) v [M, C, DV] fp32 (the per-dim chunk_o flash; reference
    fused.py:414-433)."""
    q, k, v, ag, bg = inputs
    C, D = params.get("C", q.shape[-2]), params.get("D", q.shape[-1])
    DV = params.get("DV", v.shape[-1])
    M = params["nc"] * params["H"]
    rs = lambda t, d: _c(t, torch.float16).reshape(M, C, d)
    q, k, ag, bg, v = rs(q, D), rs(k, D), rs(ag, D), rs(bg, D), rs(v, DV)
    o = torch.empty(M, C, DV, device=q.device, dtype=torch.float32)
    nv.check(nv.lib().ptof_qkvp_flash_exec(ws, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                           ag.data_ptr(), bg.data_ptr(), o.data_ptr(), M, C, D,
                                           DV, nv.F16, nv.stream_handle(q.device)))
    return [o]


_GDN_RUNNERS: Dict[tuple, Any] = {}


def _gdn_launch(ws, inputs, params) -> List[torch.Tensor]:
    """qF, kF, vF [M,C,D] (M = B*H*nc, heads outer), g_native [M,C] chunk-local
    cumsum, beta_native [M,C] -> o [B,H,nc,C,Dv] (out_dtype, default fp32)."""
    from .gdn import GDNChunkForward
    q, k, v, g, beta = inputs
    B, H, nc = params["B"], params["H"], params["nc"]
    C, D, Dv = q.shape[-2], q.shape[-1], v.shape[-1]
    T = nc * C
    dt = q.dtype if q.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.bfloat16
    out_dtype = params.get("out_dtype", torch.float32)
    key = (B, H, T, D, Dv, dt, beta.dtype, out_dtype, params.get("scale"), q.device)
    r = _GDN_RUNNERS.get(key)
    if r is None:
        r = GDNChunkForward(B, H, T, D, Dv, in_dtype=dt, beta_dtype=beta.dtype,
                            out_dtype=out_dtype, gate="cumsum", scale=params.get("scale"),
                            chunk=C, device=q.device)
        _GDN_RUNNERS[key] = r
    shp = lambda x, d: _c(x, dt).reshape(B, H, T, d)
    o, _ = r(shp(q, D), shp(k, D), shp(v, Dv), _c(beta).reshape(B, H, T),
             _c(g, torch.float32).reshape(B, H, T), output_final_state=False)
    return [o.reshape(B, H, nc, C, Dv)]


def default_fused_registry() -> FusedKernelRegistry:
    reg = FusedKernelRegistry()
    f16, f32 = torch.float16, torch.float32
    reg.register("chunk_h_scan", _Recipe(_scan_launch, FusedContract(
        in_slots=["w", "u", "k", "decay"], in_dtypes=[f16, f16, f16, f32],
        out_names=["h_out", "final"], out_dtype=f16,
        notes="resident-state chunk recurrence; w/u/k [B,nc,C,H,D], decay [B,H,nc] "
              "(or [B,H,nc,D] with perdim_decay)")))
    mega = lambda causal: (lambda ws, ins, p: _mega_launch(ws, ins, p, p.get("causal", causal)))
    native = lambda causal: (lambda ws, ins, p: _native_launch(ws, ins, p, p.get("causal", causal)))
    reg.register("kkt_gated", _Recipe(mega(False), FusedContract(
        in_slots=["k", "g_sum", "beta"], in_dtypes=[f16, f32, f16], out_names=["L"],
        out_dtype=f16, notes="gated k k^T, strict lower; k [1,T,H,D] -> L [T,H,C]")))
    reg.register("gated_qk", _Recipe(mega(True), FusedContract(
        in_slots=["a", "b", "g_sum", "beta"], in_dtypes=[f16, f16, f32, f16], out_names=["L"],
        out_dtype=f16, notes="gated a b^T (causal by default); a,b [1,T,H,D]")))
    for key in ("kkt_gated_native", "kkt_gated_native_v2"):
        reg.register(key, _Recipe(native(False), FusedContract(
            in_slots=["k", "g_native", "beta_native"], in_dtypes=[f16, f32, f16],
            out_names=["L"], out_dtype=f16,
            notes="native [M,C,D] gated k k^T, strict lower, L [M,C,C]")))
    for key in ("gated_qk_native", "gated_qk_native_v2"):
        reg.register(key, _Recipe(native(True), FusedContract(
            in_slots=["a", "b", "g_native", "beta_native"], in_dtypes=[f16, f16, f32, f16],
            out_names=["L"], out_dtype=f16,
            notes="native [M,C,D] gated a b^T (causal unless params causal=False)")))
    qkv = FusedContract(in_slots=["q", "k", "v", "g_native", "beta_native"],
                        in_dtypes=[f16, f16, f16, f32, f16], out_names=["o"], out_dtype=f32,
                        notes="o = tril(q k^T * exp(min(g_i-g_j,0))) v in one launch")
    for key in ("qkv_flash_native", "qkv_flash_native_v2"):
        reg.register(key, _Recipe(_qkv_launch, qkv))
    pro = FusedContract(in_slots=["q", "k", "P", "invP"], in_dtypes=[f16, f16, f16, f16],
                        out_names=["L"], out_dtype=f16,
                        notes="per-channel-gate intra score tril((q*P)(k*invP)^T, 0); "
                              "q/k/P/invP [M,C,D], L [M,C,C]")
    for key in ("qk_prologue", "qk_prologue_v2"):
        reg.register(key, _Recipe(_prologue_launch, pro))
    qkvp = FusedContract(in_slots=["q", "k", "v", "coef_ag", "coef_bg"],
                         in_dtypes=[f16] * 5, out_names=["o"], out_dtype=f32,
                         notes="per-dim chunk_o flash o = tril((q*coef_ag)(k*coef_bg)^T) v; "
                               "q/k/coef [M,C,D], v [M,C,DV], o [M,C,DV] f32")
    for key in ("qkvp_flash_native", "qkvp_flash_native_v2"):
        reg.register(key, _Recipe(_qkvp_launch, qkvp))
    reg.register("gdn_chunk_fwd", _Recipe(_gdn_launch, FusedContract(
        in_slots=["q", "k", "v", "g_native", "beta_native"],
        in_dtypes=[torch.bfloat16, torch.bfloat16, torch.bfloat16, f32, torch.bfloat16],
        out_names=["o"], out_dtype=f32,
        notes="whole chunked GDN forward (kkt, (I+A)^-1, WY, state scan, chunk_o) in one "
              "tcgen05 launch; fp16/bf16/fp32 operands accepted as given")))
    return reg


_DEFAULT: Optional[FusedKernelRegistry] = None


def shared_fused_registry() -> FusedKernelRegistry:
    """Process-wide registry, so runners persist across executors and captures."""
    global _DEFAULT
    if _DEFAULT is None:
        _DEFAULT = default_fused_registry()
    return _DEFAULT
