"""Chunk-segment scan: the GDN forward of few heads over a very long sequence,
split along the token axis across ranks (and into sub-segments within a rank).

Over a chunk-aligned token segment the gated delta-rule state map is affine in the
entry state, ``S_out = A S_in + B`` (each chunk applies
``S <- (e^{g_last} I - K_dec^T W) S + K_dec^T U``, a left multiplication plus an
offset). ``A`` [Dk, Dk] is the final state of the forward started from ``S0 = I``
with ``v = 0``; ``B`` [Dk, Dv] the final state started from ``S0 = 0``. So a rank
that owns tokens ``[r T_local, (r+1) T_local)`` of every (b, h) pair:

1. runs the fused forward twice over its ``s`` sub-segments (both runs share k,
   beta, g): the ``A`` run and the ``B`` run, ``pairs * s`` CTAs each;
2. composes its sub-segment maps into one ``(A_r, B_r)`` (``ptof_seg_scan_exec``);
3. all-gathers ``(A_r, B_r)`` over the process group (the one exchange);
4. applies the maps of ranks ``0..r-1`` to the global initial state for its entry
   state, then its own sub-segment maps for every sub-segment's entry state X and
   its exit state (on the last rank, the final state);
5. fixes the outputs up in place: the output is affine in the entry state too,
   ``o = o^B + o^A X`` with ``o^B`` the B run's output and ``o^A`` the A run's
   (``ptof_seg_fix_exec``, a tensor-core product per 128-token tile).

The reference runs each head serially over the whole sequence (its resident scan,
kernels/scan_fused.h:198-262); its design notes place few-head long contexts outside
the regime it wins (docs/DESIGN.md:336-340). This is the exchange-step extension of
that recurrence; the result equals the serial forward (examples/attention/
_gdn_full.py:57-97 with an initial state) up to rounding.

Chain work per token is two forwards instead of one (run side by side), spread over
``world * s`` times more CTAs, plus one bandwidth-bound fix-up pass, so it pays when
the serial chain leaves SMs idle: few (b, h) pairs, many GPUs.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch

from . import native as nv
from .gdn import GDNChunkForward

CHUNK = 64


def split_tokens(T: int, world: int, chunk: int = CHUNK) -> Tuple[int, ...]:
    """Token count of each rank's contiguous range: whole chunks, as even as possible
    (the first ranks take the extra chunks)."""
    if T % chunk:
        raise ValueError(f"T={T} is not a multiple of the chunk length {chunk}")
    if world < 1:
        raise ValueError("world must be >= 1")
    base, extra = divmod(T // chunk, world)
    return tuple((base + (1 if r < extra else 0)) * chunk for r in range(world))


def seg_scan(A: Optional[torch.Tensor], B: Optional[torch.Tensor], X0: Optional[torch.Tensor],
             Xout: Optional[torch.Tensor], Xf: Optional[torch.Tensor], heads: int, nseg: int,
             D: int, Dv: int) -> None:
    """Apply segment maps in order on the current CUDA stream (ptof_seg_scan_exec):
    ``X_0 = X0 (None: 0), X_{j+1} = A_j X_j + B_j (B None: no offset)``; entry states
    to ``Xout`` [heads, nseg, D, Dv], exit state to ``Xf`` [heads, D, Dv]. Operands
    are fp32 views whose two innermost dimensions are contiguous rows; the head and
    segment strides are taken from the views."""
    def hs(t, i=0):
        return 0 if t is None else t.stride(i)

    for name, t in (("A", A), ("B", B), ("X0", X0), ("Xout", Xout), ("Xf", Xf)):
        if t is not None:
            if t.dtype != torch.float32 or not t.is_cuda:
                raise TypeError(f"seg_scan {name}: fp32 CUDA tensor required")
            if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1]:
                raise ValueError(f"seg_scan {name}: rows must be contiguous")
    dev = next(t for t in (A, B, X0, Xout, Xf) if t is not None).device
    rc = nv.lib().ptof_seg_scan_exec(
        nv.ptr(A), hs(A), hs(A, 1) if A is not None and A.dim() == 4 else 0,
        nv.ptr(B), hs(B), hs(B, 1) if B is not None and B.dim() == 4 else 0,
        nv.ptr(X0), hs(X0),
        nv.ptr(Xout), hs(Xout), hs(Xout, 1) if Xout is not None else 0,
        nv.ptr(Xf), hs(Xf), heads, nseg, D, Dv, nv.stream_handle(dev))
    nv.check(rc)


def seg_fix(ws, o: torch.Tensor, oa: torch.Tensor, X: torch.Tensor, units: int, Tseg: int,
            D: int) -> None:
    """o[u, t] += oa[u, t] @ X[u] in place on the current stream (ptof_seg_fix_exec):
    o, oa [units, Tseg, D] 16-bit, X [units, D, D] fp32, all contiguous."""
    for name, t in (("o", o), ("oa", oa), ("X", X)):
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"seg_fix {name}: contiguous CUDA tensor required")
    if oa.dtype != o.dtype or X.dtype != torch.float32:
        raise TypeError("seg_fix: o and oa share a 16-bit dtype, X is fp32")
    nv.check(nv.lib().ptof_seg_fix_exec(ws, o.data_ptr(), oa.data_ptr(), X.data_ptr(), units,
                                        Tseg, D, nv.dtype_code(o.dtype),
                                        nv.stream_handle(o.device)))


class GDNSegmentScan:
    """Segment-parallel GDN forward of ``pairs`` (b, h) recurrences over one rank's
    token range of ``T_local`` tokens, split into ``segments`` local sub-segments.

    Operands are the rank's range of every pair, heads-outer: q, k [pairs, T_local,
    Dk], v [pairs, T_local, Dv], beta, g [pairs, T_local]; ``initial_state``
    [pairs, Dk, Dv] fp32 is the state before token 0 of the WHOLE sequence (the same
    on every rank). ``__call__`` returns (o [pairs, T_local, Dv], the state after
    this rank's range [pairs, Dk, Dv]; on the last rank the final state).

    Sub-segments are whole 128-token tiles (``T_local`` a multiple of
    ``128 * segments``).

    ``group``: the torch.distributed process group the sequence is split over (None:
    this process holds the whole sequence). ``forward``/``scan``/``fix`` are
    injection points for the CPU multi-process tests; by default the fused CUDA
    forward, ``ptof_seg_scan_exec`` and ``ptof_seg_fix_exec`` run, and they fail
    loudly when the library is missing.
    """

    def __init__(self, pairs: int, T_local: int, D: int, *, segments: int = 2, group=None,
                 in_dtype=torch.bfloat16, beta_dtype=None, out_dtype=None, gate: str = "raw",
                 scale: Optional[float] = None, device=None,
                 forward: Optional[Callable] = None, scan: Optional[Callable] = None,
                 fix: Optional[Callable] = None) -> None:
        if segments < 1 or T_local % (segments * 2 * CHUNK):
            raise ValueError(f"T_local={T_local} is not {segments} sub-segments of whole "
                             f"128-token tiles")
        self.pairs, self.T_local, self.D, self.s = pairs, T_local, D, segments
        self.Tseg = T_local // segments
        self.group = group
        import torch.distributed as dist
        self._dist = dist if group is not None else None
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        self.in_dtype = in_dtype
        self.beta_dtype = beta_dtype or in_dtype
        self.out_dtype = out_dtype or in_dtype
        self.gate = gate
        self.scale = D ** -0.5 if scale is None else float(scale)
        if forward is None:
            self.device = nv.cuda_device(device) if device is not None else torch.device(
                "cuda", torch.cuda.current_device())
            mk = lambda: GDNChunkForward(pairs, segments, self.Tseg, D, D, in_dtype=in_dtype,
                                         beta_dtype=self.beta_dtype, out_dtype=self.out_dtype,
                                         gate=gate, scale=self.scale, device=self.device)
            run_main, run_side = mk(), mk()
            self._runners = (run_main, run_side)

            def forward(which, q, k, v, beta, g, S0, o, S_out):
                r = run_main if which == "main" else run_side
                r(q, k, v, beta, g, S0, o=o, final_state=S_out)
            self._side = torch.cuda.Stream(self.device)
            self._ws = nv.lib().ptof_ws_setup()
            if not self._ws:
                raise nv.NativeError(nv.EINVAL, nv.last_error())
            ws = self._ws
            fix = lambda o, oa, X, units, Tseg, D_: seg_fix(ws, o, oa, X, units, Tseg, D_)
        else:
            self.device = torch.device(device or "cpu")
            self._runners = ()
            self._side = None
            self._ws = None
        self._forward = forward
        self._scan = scan or seg_scan
        self._fix = fix
        P, s, dev = pairs, segments, self.device
        f32 = dict(device=dev, dtype=torch.float32)
        # constant operands of the transition run
        self._v0 = torch.zeros(P, s, self.Tseg, D, device=dev, dtype=in_dtype)
        self._eye = torch.eye(D, **f32).expand(P, s, D, D).contiguous()
        self._o_side = torch.empty(P, s, self.Tseg, D, device=dev, dtype=self.out_dtype)
        self._A = torch.empty(P, s, D, D, **f32)
        self._B = torch.empty(P, s, D, D, **f32)
        self._send = torch.empty(2, P, D, D, **f32)            # this rank's (A_r, B_r)
        self._gath = torch.empty(self.world, 2, P, D, D, **f32)
        self._S_in = torch.empty(P, D, D, **f32)
        self._entry = torch.empty(P, s, D, D, **f32)
        self._S_out = torch.empty(P, D, D, **f32)

    def _views(self, q, k, v, beta, g):
        P, s, Ts, D = self.pairs, self.s, self.Tseg, self.D
        for name, t, shape in (("q", q, (P, self.T_local, D)), ("k", k, (P, self.T_local, D)),
                               ("v", v, (P, self.T_local, D)), ("beta", beta, (P, self.T_local))):
            if tuple(t.shape) != shape:
                raise ValueError(f"{name} shape {tuple(t.shape)} != {shape}")
        q4, k4, v4 = (t.reshape(P, s, Ts, D) for t in (q, k, v))
        b3 = beta.reshape(P, s, Ts)
        g3 = None if g is None else g.reshape(P, s, Ts)
        return q4, k4, v4, b3, g3

    def __call__(self, q, k, v, beta, g, initial_state=None, *, o=None
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
        P, s, D, W, r = self.pairs, self.s, self.D, self.world, self.rank
        q4, k4, v4, b3, g3 = self._views(q, k, v, beta, g)
        if o is None:
            o = torch.empty(P, self.T_local, D, device=q.device, dtype=self.out_dtype)
        o4 = o.view(P, s, self.Tseg, D)
        fwd, scan, fix = self._forward, self._scan, self._fix
        # 1. segment maps: B run on the current stream, A run on the side stream
        if self._side is not None:
            main = torch.cuda.current_stream(self.device)
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                fwd("side", q4, k4, self._v0, b3, g3, self._eye, self._o_side, self._A)
            fwd("main", q4, k4, v4, b3, g3, None, o4, self._B)
            main.wait_stream(self._side)
        else:
            fwd("side", q4, k4, self._v0, b3, g3, self._eye, self._o_side, self._A)
            fwd("main", q4, k4, v4, b3, g3, None, o4, self._B)
        # 2. this rank's composite map (A_r, B_r) = maps of sub-segments s-1 o ... o 0
        if W > 1:
            scan(self._A[:, 1:], None, self._A[:, 0], None, self._send[0], P, s - 1, D, D)
            scan(self._A[:, 1:], self._B[:, 1:], self._B[:, 0], None, self._send[1], P, s - 1,
                 D, D)
            # 3. the exchange
            self._dist.all_gather_into_tensor(self._gath.view(-1), self._send.view(-1),
                                              group=self.group)
        # 4. entry state of this rank (maps of ranks 0..r-1 on the initial state), then
        #    the entry state of every local sub-segment and the exit state
        if r > 0:
            g4 = self._gath.permute(2, 0, 1, 3, 4)          # [P, W, 2, D, D] view
            scan(g4[:, :r, 0], g4[:, :r, 1], initial_state, None, self._S_in, P, r, D, D)
            S_in = self._S_in
        else:
            S_in = initial_state
        scan(self._A, self._B, S_in, self._entry, self._S_out, P, s, D, D)
        # 5. o = o^B + o^A X, in place
        fix(o, self._o_side, self._entry, P * s, self.Tseg, D)
        return o, self._S_out

    def check_status(self) -> None:
        """Synchronise and raise if a bounded device wait of the last call gave up."""
        for run in self._runners:
            run.check_status()
        if self._ws:
            nv.check(nv.lib().ptof_check_status(self._ws, nv.stream_handle(self.device)))

    def close(self) -> None:
        for run in self._runners:
            run.close()
        self._runners = ()
        if self._ws:
            nv.lib().ptof_ws_teardown(self._ws)
            self._ws = None


# --------------------------------------------------------------------------------
# Chunk-segment scan inside one GPU, with a long head segment
# --------------------------------------------------------------------------------
def plan_local_split(pairs: int, T: int, sms: int, *, chunk_us: float = 3.0,
                     serial_chunk_us: float = 2.4, fix_gbs: float = 4000.0,
                     fixed_us: float = 40.0, cta_us: float = 15.0, max_rounds: int = 1,
                     D: int = 128
                     ) -> Optional[Tuple[int, int, int]]:
    """Head/tail split of ``pairs`` sequences of T tokens on ``sms`` SMs, or None when
    the plain forward is predicted faster.

    The forward is one CTA per chain walking its chunks in order, so with fewer pairs
    than SMs the chains, not the SMs, set the time: ≈ ``serial_chunk_us`` per chunk when
    one chain per pair runs, ≈ ``chunk_us`` once the split fills every SM (both
    measured on B200: a split of 64 pairs x 16,384 tokens never beat the serial 0.61 ms;
    16 pairs ran in 0.224 ms against 0.594 serial and 0.237 for four equal segments,
    32 pairs in 0.386 against 0.601 and 0.420 for two; config 4 in 4.0 against 4.7 ms
    with tails in many rounds, a plan this model does not propose). Each
    pair's head segment of L0 tokens runs from the true initial state (one chain,
    output final); its tail is cut into s segments of Ls tokens that run as A and B
    chains (2 s chains per pair) on the SMs the heads leave free, composed by
    ``seg_scan`` and fixed up by ``seg_fix``. Modelled time: max(head chain, rounds of
    tail chains, each round with a CTA start-up) plus the fix-up's bytes and a fixed
    cost; by default every tail chain must start in the first round (plans with a
    second round measured slower at 32 pairs: 0.459 against 0.386 ms). Returns
    (L0, s, Ls)."""
    nchunks = T // CHUNK
    plain_us = nchunks * serial_chunk_us
    free = sms - pairs
    if free <= 0 or T % (2 * CHUNK):
        return None
    best = None
    for s in range(1, 9):
        for tiles in range(1, T // (2 * CHUNK * s) + 1):
            Ls = tiles * 2 * CHUNK            # whole 128-token fix-up tiles
            L0 = T - s * Ls
            if L0 < CHUNK:
                break
            rounds = -(-2 * pairs * s // free)
            if rounds > max_rounds:   # later rounds start late: measured, not modelled
                continue
            # each round of tail CTAs also pays a CTA's start-up (TMEM, barriers, the
            # first loads)
            t = max(L0 // CHUNK * chunk_us, rounds * (Ls // CHUNK * chunk_us + cta_us))
            t += pairs * s * Ls * D * 2 * 3 / (fix_gbs * 1e3) + fixed_us
            if best is None or t < best[0]:
                best = (t, L0, s, Ls)
    if best is None or best[0] >= 0.95 * plain_us:
        return None
    return best[1], best[2], best[3]


class GDNLocalSplit:
    """GDN forward of ``pairs`` (b, h) sequences of T tokens on one GPU, each split into
    a head of L0 tokens and s tail segments of Ls tokens (``plan_local_split``).

    The head runs from the true initial state and writes its output in place; the tail
    segments run twice side by side — the B run from a zero state (its output, written
    in place into o, is o^B) and the A run from S0 = I with v = 0 (o^A into a scratch
    buffer) — then ``seg_scan`` applies the tail maps in order from the head's final
    state (the entry state X of every tail segment and the final state) and
    ``ptof_seg_fix_exec_view`` adds o^A X into o. Every launch reads the caller's
    tensors in place through strided views (``GDNChunkForward.set_view``). Operands:
    q, k, v [pairs, T, D] bf16, beta [pairs, T], g [pairs, T] fp32 (per-token log
    decay), initial_state [pairs, D, D] fp32 or None. Returns (o, final state).
    Same result as the serial forward up to rounding (the affine algebra of the module
    docstring)."""

    def __init__(self, pairs: int, T: int, D: int, L0: int, segments: int, Ls: int, *,
                 in_dtype=torch.bfloat16, scale: Optional[float] = None, device=None) -> None:
        if L0 + segments * Ls != T or L0 % CHUNK or Ls % (2 * CHUNK) or L0 < CHUNK:
            raise ValueError(f"split L0={L0} + {segments} x {Ls} does not tile T={T}")
        self.pairs, self.T, self.D, self.L0, self.s, self.Ls = pairs, T, D, L0, segments, Ls
        self.device = nv.cuda_device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.dtype = in_dtype
        self.scale = D ** -0.5 if scale is None else float(scale)
        P, s, dev = pairs, segments, self.device
        mk = lambda H, TT: GDNChunkForward(P, H, TT, D, D, in_dtype=in_dtype, scale=self.scale,
                                           device=dev)
        self._head, self._tb, self._ta = mk(1, L0), mk(s, Ls), mk(s, Ls)
        self._head.set_view((T, T), (T, T), (T, T))
        self._tb.set_view((T, Ls), (T, Ls), (T, Ls))
        self._ta.set_view((T, Ls), (s * Ls, Ls), (s * Ls, Ls))   # v = 0 and o^A dense
        f32 = dict(device=dev, dtype=torch.float32)
        self._v0 = torch.zeros(P, s, Ls, D, device=dev, dtype=in_dtype)
        self._oa = torch.empty(P, s, Ls, D, device=dev, dtype=in_dtype)
        self._eye = torch.eye(D, **f32).expand(P, s, D, D).contiguous()
        self._A = torch.empty(P, s, D, D, **f32)
        self._B = torch.empty(P, s, D, D, **f32)
        self._S_head = torch.empty(P, D, D, **f32)
        self._entry = torch.empty(P, s, D, D, **f32)
        self._S_out = torch.empty(P, D, D, **f32)
        self._streams = (torch.cuda.Stream(dev), torch.cuda.Stream(dev),
                         torch.cuda.Stream(dev, priority=-1))
        self._ws = nv.lib().ptof_ws_setup()
        if not self._ws:
            raise nv.NativeError(nv.EINVAL, nv.last_error())

    def __call__(self, q, k, v, beta, g, initial_state=None, *, o=None):
        P, T, D, L0 = self.pairs, self.T, self.D, self.L0
        for name, t, shape in (("q", q, (P, T, D)), ("k", k, (P, T, D)), ("v", v, (P, T, D)),
                               ("beta", beta, (P, T)), ("g", g, (P, T))):
            if tuple(t.shape) != shape or not t.is_contiguous():
                raise ValueError(f"{name}: expected contiguous {shape}, got {tuple(t.shape)}")
        if o is None:
            o = torch.empty(P, T, D, device=q.device, dtype=self.dtype)
        main = torch.cuda.current_stream(self.device)
        sa, sb, sh = self._streams
        # the heads (the longest chains) on a high-priority stream so that their CTAs
        # take SMs first, the tail runs on two side streams
        sa.wait_stream(main)
        sb.wait_stream(main)
        sh.wait_stream(main)
        with torch.cuda.stream(sh):
            self._head.call_view(q, k, v, beta, g, initial_state, o, self._S_head)
        tq, tk, tv, tb, tg, to = (t[:, L0:] for t in (q, k, v, beta, g, o))
        with torch.cuda.stream(sb):
            self._tb.call_view(tq, tk, tv, tb, tg, None, to, self._B)
        with torch.cuda.stream(sa):
            self._ta.call_view(tq, tk, self._v0, tb, tg, self._eye, self._oa, self._A)
        main.wait_stream(sa)
        main.wait_stream(sb)
        main.wait_stream(sh)
        seg_scan(self._A, self._B, self._S_head, self._entry, self._S_out, P, self.s, D, D)
        nv.check(nv.lib().ptof_seg_fix_exec_view(
            self._ws, to.data_ptr(), self._oa.data_ptr(), self._entry.data_ptr(), P, self.s,
            self.Ls, D, nv.dtype_code(self.dtype), T, self.Ls, nv.stream_handle(self.device)))
        return o, self._S_out

    def check_status(self) -> None:
        for r in (self._head, self._tb, self._ta):
            r.check_status()
        nv.check(nv.lib().ptof_check_status(self._ws, nv.stream_handle(self.device)))

    def close(self) -> None:
        for r in (self._head, self._tb, self._ta):
            r.close()
        if self._ws:
            nv.lib().ptof_ws_teardown(self._ws)
            self._ws = None
