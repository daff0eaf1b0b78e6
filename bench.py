"""Benchmark of the fused chunked Gated DeltaNet forward on B200.

Workload (one "step"): BASELINE config 2 — the full GDN chunk forward, bf16,
B=4, H=32, T=16384, Dk=Dv=128, C=64 — with its 128 independent (batch, head)
pairs sharded over the N GPUs (strong scaling: 128/64/32/16 pairs per GPU; no
collective on the data path). A rank with fewer pairs than it has SMs also splits
every pair's sequence into segments (the chunk-segment scan) so its SMs stay busy.
At N > 1 the line also carries `weak_value`: every rank its own whole config-2 batch. Inputs are synthetic with the benchmark distributions (q, k
L2-normalised N(0,1); v N(0,1); beta = sigmoid(N(0,1)); g = logsigmoid(N(2,1))).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  (N > 1: launched by torch.distributed.run, one rank per GPU)

Prints one JSON line (rank 0). `value` is whole-job tokens/s with inputs resident
in HBM (device-timed with CUDA events, max over ranks); `e2e` is the same metric
through the public API with pinned host buffers and every step's host<->device copies
inside the timed region (uploads, kernels and downloads pipelined over three streams); `roofline` is the fused kernel's achieved HBM bandwidth on its
algorithmic bytes against the measured copy peak; `cpu_baseline` is the CPU oracle
timed on this host on a bounded sample. `--impl reference` times the reference's
forward on the host cores: its fp32 torch `gdn_reference` chunk loop (the reference's
device path is Ascend/CANN code with no CPU or CUDA build), restated in
pto_fuser.forwards.gdn, with all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "pto-fuser_b200"))
sys.path.insert(0, ROOT)

METRIC = "GDN chunk-forward tokens/s per GPU and whole box at 1/2/4/8 B200; % roofline"
CFG = dict(B=4, H=32, T=16384, D=128, C=64)
PEAK_FALLBACK_GBS = 6650.0


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return PEAK_FALLBACK_GBS, "fallback"


def _algo_bytes(B, H, T, D):
    """Algorithmic HBM bytes of one forward: q, k, v (bf16), beta (bf16), g (fp32),
    o (bf16) per head-token, plus the fp32 final state per (b, h)."""
    return B * H * T * (3 * D * 2 + 2 + 4 + D * 2) + B * H * D * D * 4


def _algo_flops(B, H, T, D, C=64):
    return B * H * T * (2 * C * C * (3 * D + 2 * D) + 6 * C * D * D) // C


class ClockSampler:
    """SM clock and throttle-reason sampling (NVML, ~5 ms period) in a background
    thread during the timed region. Reads only; changes no GPU setting."""

    def __init__(self, device, period_s: float = 0.001):
        self.dev = device
        self.period = period_s
        self.rows = []
        self._stop = threading.Event()
        self._t = None
        self._nv = None

    def _sample(self, h, mx):
        nv = self._nv
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        try:
            rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        except Exception:
            rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
        self.rows.append((sm, mx, rs))

    def _run(self, h, mx):
        while not self._stop.is_set():
            try:
                self._sample(h, mx)
            except Exception as e:  # keep sampling; report the first failure
                self.error = self.error or repr(e)
            self._stop.wait(self.period)

    def __enter__(self):
        self.error = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            self._nv = nv
            h, self.ident = _nvml_handle(nv, self.dev)
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self._sample(h, mx)          # the calls work before the timed region starts
            self.rows.clear()
            self._t = threading.Thread(target=self._run, args=(h, mx), daemon=True)
            self._t.start()
        except Exception as e:
            self._nv = None
            self.error = repr(e)
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0,
                    "error": self.error}
        import statistics
        nv = self._nv
        bits = {"hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
                "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
                "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
                "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4)}
        reasons = sorted({n for _, _, r in self.rows for n, b in bits.items() if r & b})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows),
                "sm_max_mhz": max(r[1] for r in self.rows), "reasons": reasons,
                "samples": len(self.rows), "gpu": getattr(self, "ident", None)}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_reference(threads: int, heads: int, T: int, D: int, seed: int = 0):
    """Times the reference forward on the host cores: gdn_reference, the fp32 torch
    chunk loop of the reference (examples/attention/_gdn_full.py:57-97, one (b, h)
    pair and one chunk at a time) as restated in pto_fuser.forwards.gdn, on `heads`
    pairs of length T with the benchmark's input distributions. Returns (seconds,
    sample description)."""
    import torch
    from pto_fuser.forwards.gdn import gdn_reference
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(seed)
    nc, C = T // 64, 64
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(1, heads, nc, C, D, generator=gen), dim=-1)
    k = nrm(torch.randn(1, heads, nc, C, D, generator=gen), dim=-1)
    v = torch.randn(1, heads, nc, C, D, generator=gen)
    beta = torch.sigmoid(torch.randn(1, heads, nc, C, generator=gen))
    g = torch.nn.functional.logsigmoid(torch.randn(1, heads, nc, C, generator=gen) + 2.0)
    t0 = time.perf_counter()
    gdn_reference(q, k, v, beta, g, D ** -0.5, return_final_state=True)
    dt = time.perf_counter() - t0
    return dt, (f"{heads} of the (b,h) pairs x T={T}, D={D}: the reference's fp32 torch "
                f"gdn_reference chunk loop on {threads} host threads")


def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return
    B, H, T, D = CFG["B"], CFG["H"], CFG["T"], CFG["D"]
    threads = os.cpu_count() or 1
    heads = 8
    for _ in range(args.warmup):
        cpu_reference(threads, 1, 1024, D)
    times = []
    desc = ""
    for s in range(args.steps):
        dt, desc = cpu_reference(threads, heads, T, D, seed=s)
        times.append(dt)
    tsec = sum(times) / len(times)
    # one step = `heads` of the B*H pairs; scale to the whole config-2 workload
    tok_s = (B * T) * heads / (B * H) / tsec
    out = {"impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tokens/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": tsec * 1e3, "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": "cfg2: GDN chunk forward B4 H32 T16384 D128 C64 (CPU sample "
                                  "of the 128 (b,h) pairs, scaled to the whole batch)",
                      "sample_pairs": heads, "T": T, "D": D},
           "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "port",
                            "sample": desc},
           "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def _nvml_handle(nv, dev):
    """The NVML handle of the CUDA device `dev`, found by UUID (else PCI bus id):
    NVML numbers GPUs in PCI order and ignores CUDA_VISIBLE_DEVICES, so the CUDA
    ordinal may name another GPU."""
    import torch
    props = torch.cuda.get_device_properties(dev)
    uuid = str(getattr(props, "uuid", "") or "")
    if uuid:
        u = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        try:
            return nv.nvmlDeviceGetHandleByUUID(u), u
        except Exception:
            pass
    bus = "%08X:%02X:%02X.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
    return nv.nvmlDeviceGetHandleByPciBusId(bus), bus


def run_ours(args):
    import torch
    import torch.distributed as dist
    world, rank, local = _dist()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    from pto_fuser import GDNChunkForward, make_gdn_inputs
    from pto_fuser.segment import GDNLocalSplit, plan_local_split
    from pto_fuser.shard import shard_pairs

    B, H, T, D = CFG["B"], CFG["H"], CFG["T"], CFG["D"]
    # strong scaling: the job's B*H pairs split into contiguous blocks, one per rank
    p0, p1 = shard_pairs(B * H, world, rank)
    P = p1 - p0
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    # The forward is one CTA per pair walking its chunks in order, so a shard with
    # fewer pairs than SMs leaves SMs idle: such a rank splits every pair into a head
    # segment (from the true initial state) and tail segments that run as A and B
    # chains on the free SMs, composed by seg_scan and fixed up by seg_fix
    # (segment.plan_local_split; None = the plain forward).
    plan = plan_local_split(P, T, sms, D=D)
    segs = 1 if plan is None else 1 + plan[1]
    inp = make_gdn_inputs(1, P, T, D, dtype=torch.bfloat16, device=dev, mu=2.0,
                          seed=1234 + rank)
    o = torch.empty(1, P, T, D, device=dev, dtype=torch.bfloat16)
    S = torch.empty(1, P, D, D, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    if plan is None:
        runner = GDNChunkForward(1, P, T, D, D, in_dtype=torch.bfloat16, device=dev)

        def forward(q, k, v, beta, g, o_, S_):
            runner(q, k, v, beta, g, o=o_, final_state=S_)
        launches = 2   # coefficient pre-pass + fused forward
        how = "plain fused forward, one CTA per (b,h) pair"
    else:
        L0, ns, Ls = plan
        runner = GDNLocalSplit(P, T, D, L0, ns, Ls, device=dev)

        def forward(q, k, v, beta, g, o_, S_):
            _, Sx = runner(q[0], k[0], v[0], beta[0], g[0], None, o=o_[0])
            S_.view(P, D, D).copy_(Sx)
        # head, tail B and tail A runs (coefficient pre-pass + forward each), seg_scan,
        # seg_fix (the final-state copy is a torch copy)
        launches = 8
        how = (f"head/tail split inside the GPU: per pair a {L0}-token head and {ns} "
               f"tail segments of {Ls} tokens; {P} head chains + {2 * P * ns} tail chains")

    def step():
        forward(inp["q"], inp["k"], inp["v"], inp["beta"], inp["g"], o, S)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    runner.check_status()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---- device-timed, inputs resident (per-launch events give the kernel average) ----
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(dev) as clk:
        barrier()
        evs[0].record(stream)
        for i in range(args.steps):
            step()
            evs[i + 1].record(stream)
        barrier()
    runner.check_status()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    ms = evs[0].elapsed_time(evs[-1])
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    tokens = B * T * args.steps          # the whole job's tokens (all ranks together)
    value = tokens / (ms_max / 1e3)

    # ---- end to end through the public API: pinned host in, host out ----
    # Every step uploads its own inputs from pinned host memory and downloads its own
    # result (o and the final state). The two PCIe directions and the kernels are
    # independent engines, so steps are pipelined over three streams with
    # double-buffered device operands: upload(i) || forward(i-1) || download(i-2).
    names = ("q", "k", "v", "beta", "g")
    host = {n: inp[n].cpu().pin_memory() for n in names}
    dev_in = [{n: torch.empty_like(inp[n]) for n in names} for _ in range(2)]
    dev_o = [o, torch.empty_like(o)]
    dev_S = [S, torch.empty_like(S)]
    o_h = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for _ in range(2)]
    S_h = [torch.empty(S.shape, dtype=S.dtype, pin_memory=True) for _ in range(2)]
    h2d = sum(host[n].numel() * host[n].element_size() for n in names)
    d2h = o_h[0].numel() * o_h[0].element_size() + S_h[0].numel() * S_h[0].element_size()
    e2e_steps = max(2, min(args.steps, 6))
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def e2e_run(n_steps):
        ev_in = [torch.cuda.Event() for _ in range(n_steps)]
        ev_fw = [torch.cuda.Event() for _ in range(n_steps)]
        ev_out = [torch.cuda.Event() for _ in range(n_steps)]
        for i in range(n_steps):
            j = i & 1
            with torch.cuda.stream(up):            # buffer j last read by forward(i-2)
                if i >= 2:
                    up.wait_event(ev_fw[i - 2])
                for n in names:
                    dev_in[j][n].copy_(host[n], non_blocking=True)
                ev_in[i].record(up)
            stream.wait_event(ev_in[i])            # forward(i) on the compute stream
            if i >= 2:
                stream.wait_event(ev_out[i - 2])   # its outputs' last download is done
            d = dev_in[j]
            forward(d["q"], d["k"], d["v"], d["beta"], d["g"], dev_o[j], dev_S[j])
            ev_fw[i].record(stream)
            with torch.cuda.stream(down):
                down.wait_event(ev_fw[i])
                o_h[j].copy_(dev_o[j], non_blocking=True)
                S_h[j].copy_(dev_S[j], non_blocking=True)
                ev_out[i].record(down)
        stream.wait_event(ev_out[n_steps - 1])

    e2e_run(2)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up.wait_event(e0)
    e2e_run(e2e_steps)
    e1.record(stream)
    barrier()
    t2 = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_value = B * T * e2e_steps / (float(t2.item()) / 1e3)
    runner.check_status()

    # ---- secondary: weak scaling (every rank its own whole config-2 batch) ----
    weak = None
    if world > 1:
        full = make_gdn_inputs(B, H, T, D, dtype=torch.bfloat16, device=dev, mu=2.0,
                               seed=99 + rank)
        wr = GDNChunkForward(B, H, T, D, D, in_dtype=torch.bfloat16, device=dev)
        wo = torch.empty(B, H, T, D, device=dev, dtype=torch.bfloat16)
        wS = torch.empty(B, H, D, D, device=dev)
        wstep = lambda: wr(full["q"], full["k"], full["v"], full["beta"], full["g"], o=wo,
                           final_state=wS)
        for _ in range(3):
            wstep()
        n_w = max(3, min(args.steps, 10))
        barrier()
        w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0.record(stream)
        for _ in range(n_w):
            wstep()
        w1.record(stream)
        barrier()
        wr.check_status()
        tw = torch.tensor([w0.elapsed_time(w1)], device=dev)
        dist.all_reduce(tw, op=dist.ReduceOp.MAX)
        weak = {"value": B * T * world * n_w / (float(tw.item()) / 1e3), "unit": "tokens/s",
                "ms_per_step": float(tw.item()) / n_w, "steps": n_w,
                "workload": "every rank its own config-2 batch (128 pairs per GPU)"}
        del full, wo, wS
        wr.close()

    # ---- roofline of one GPU's share (HBM bound, algorithmic bytes) ----
    peak, peak_kind = _peaks()
    kern_ms = sum(per) / len(per)
    algo = _algo_bytes(1, P, T, D)
    achieved = algo / (kern_ms / 1e3) / 1e9

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            threads = os.cpu_count() or 1
            nh = 48
            dt, desc = cpu_reference(threads, nh, T, D)
            cpu = {"value": (B * T) * nh / (B * H) / dt, "unit": "tokens/s", "cores": threads,
                   "kind": "port", "sample": desc}
        wl = ("cfg2: GDN chunk forward B4 H32 T16384 Dk=Dv=128 C64 bf16, the 128 (b,h) "
              f"pairs sharded over {world} GPU(s)" if not args.shape else
              f"custom shape B{B} H{H} T{T} D{D} (profiling case)")
        out = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
               "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
               "dtype": "bf16", "data": "synthetic",
               "config": {"workload": wl, "B": B, "H": H, "T": T, "D": D, "C": CFG["C"],
                          "pairs_per_gpu": P, "segments_per_pair": segs, "plan": how,
                          "global_batch": B, "parallelism": f"(b,h) shards x{world}",
                          "l2": f"inputs+outputs {algo / 1e9:.2f} GB per GPU vs 126 MB L2"
                                + (" (no flush needed)" if algo > 126e6 * 4 else
                                   " (smaller than 4x L2: not a bandwidth figure)")},
               "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                       "d2h_bytes_per_step": d2h},
               "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                            "frac": achieved / peak,
                            "traffic": (FWD_DRAM_BYTES_PER_HEAD_TOKEN * P * T
                                        if plan is None and not args.shape else None),
                            "peak_kind": peak_kind,
                            "kernel": ("gdn_coef_kernel + gdn_fwd_tc_kernel (one forward call)"
                                       if plan is None else "whole split step"),
                            "algo_bytes_per_launch": algo, "avg_launch_ms": kern_ms,
                            "tflops": _algo_flops(1, P, T, D) / (kern_ms / 1e3) / 1e12},
               "cpu_baseline": cpu,
               "gpu_launches": launches * args.steps,
               "clocks": clk.summary()}
        if weak is not None:
            out["weak_value"] = weak
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# DRAM bytes (read + write) of one forward per head-token, from an ncu capture of the
# fused kernel and its coefficient pre-pass on an L2-exceeding small case of config 2
# (B4 H32 T2048 D128: 210.4 MB read + 45.7 MB written for 262,144 head-tokens; the
# traffic grows in proportion to the tokens, so it scales to the full launch by the
# head-tokens processed). The algorithmic figure is 1,034 B per head-token.
FWD_DRAM_BYTES_PER_HEAD_TOKEN = (208.8e6 + 1.58e6 + 45.7e6) / (4 * 32 * 2048)


def run_configs(args):
    """One JSON line per BASELINE configuration on one GPU: device time of the op
    through its C ABI (CUDA events, inputs resident, 3 warm-up calls), with the
    algorithmic HBM bytes of the configuration and its roofline fraction. These are
    supporting numbers; the headline line is the default mode (config 2)."""
    import torch
    from pto_fuser import GDNChunkForward, native as nv
    peaks = _peaks()
    hbm = peaks[0]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device="cuda").manual_seed(0)
    nrm = torch.nn.functional.normalize

    def inputs(B, H, T, D, dt, mu=2.0, gated=True):
        q = nrm(torch.randn(B, H, T, D, device=dev, generator=gen), dim=-1).to(dt)
        k = nrm(torch.randn(B, H, T, D, device=dev, generator=gen), dim=-1).to(dt)
        v = torch.randn(B, H, T, D, device=dev, generator=gen).to(dt)
        beta = torch.sigmoid(torch.randn(B, H, T, device=dev, generator=gen)).to(dt)
        g = torch.nn.functional.logsigmoid(torch.randn(B, H, T, device=dev, generator=gen) + mu)
        return q, k, v, beta, (g if gated else torch.zeros_like(g))

    def timed(fn, n):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    def line(name, desc, ms, tokens, algo, dtype):
        print(json.dumps({"config": name, "workload": desc, "ms": ms,
                          "tokens_per_s": tokens / (ms / 1e3), "dtype": dtype,
                          "algo_bytes": algo, "achieved_gbs": algo / (ms / 1e3) / 1e9,
                          "roofline_frac_hbm": algo / (ms / 1e3) / 1e9 / hbm,
                          "peak_gbs": hbm}), flush=True)

    def want(name):
        return not args.only or name in args.only

    def fwd(name, desc, B, H, T, D, dt, mu=2.0, gate="raw", s0_std=None):
        if not want(name):
            return
        q, k, v, beta, g = inputs(B, H, T, D, dt, mu, gate != "none")
        S0 = (torch.randn(B, H, D, D, device=dev, generator=gen) * s0_std) if s0_std else None
        r = GDNChunkForward(B, H, T, D, D, in_dtype=dt, gate=gate)
        o = torch.empty_like(v)
        S = torch.empty(B, H, D, D, device=dev)
        ms = timed(lambda: r(q, k, v, beta, g, S0, o=o, final_state=S), args.steps)
        r.check_status()
        e = 2 if dt != torch.float32 else 4
        per_tok = 3 * D * e + e + (4 if gate != "none" else 0) + D * e
        algo = B * H * T * per_tok + B * H * D * D * 4 * (2 if S0 is not None else 1)
        line(name, desc, ms, B * T, algo, str(dt).split(".")[-1])
        r.close()

    fwd("cfg0", "GDN forward fp32 B1 H4 T512 D128 (SIMT fp32 path)", 1, 4, 512, 128, torch.float32)
    if want("cfg1"):   # kkt + inverse alone
        B, H, T, D = 8, 32, 8192, 128
        _, k, _, beta, g = inputs(B, H, T, D, torch.bfloat16)
        out = torch.empty(B, H, T // 64, 64, 64, device=dev)
        ws = nv.lib().ptof_ws_setup()
        ms = timed(lambda: nv.check(nv.lib().ptof_kkt_inv_exec(
            ws, k.data_ptr(), beta.data_ptr(), g.data_ptr(), out.data_ptr(), B, H, T, D,
            nv.BF16, nv.BF16, nv.GATE_RAW, nv.LAYOUT_BHTD, nv.stream_handle())), args.steps)
        nv.check(nv.lib().ptof_check_status(ws, nv.stream_handle()))
        nv.lib().ptof_ws_teardown(ws)
        M = B * H * (T // 64)
        line("cfg1", "kkt + tri-inv B8 H32 T8192 D128 bf16 -> fp32 T", ms, B * T,
             M * (64 * D * 2 + 64 * 2 + 64 * 4 + 64 * 64 * 4), "bf16")
        del k, beta, g, out
    fwd("cfg2", "GDN forward bf16 B4 H32 T16384 D128", 4, 32, 16384, 128, torch.bfloat16)
    fwd("cfg3", "DeltaNet (g = 0) bf16 B16 H16 T4096 D64", 16, 16, 4096, 64, torch.bfloat16,
        gate="none")
    fwd("cfg4", "long-context GDN bf16 B1 H64 T131072 D128, S0 ~ N(0,0.02^2), mu 3", 1, 64,
        131072, 128, torch.bfloat16, mu=3.0, s0_std=0.02)

    if want("cfg4-split"):
        # config 4 through the head/tail split inside the GPU (segment.GDNLocalSplit): 64
        # pairs leave 84 SMs idle in the serial forward; the plan is the measured best of
        # a sweep (a 80,896-token head, 7 tail segments of 7,168 tokens)
        from pto_fuser.segment import GDNLocalSplit
        B, H, T, D = 1, 64, 131072, 128
        q, k, v, beta, g = inputs(B, H, T, D, torch.bfloat16, 3.0, True)
        S0 = torch.randn(H, D, D, device=dev, generator=gen) * 0.02
        sp = GDNLocalSplit(H, T, D, 80896, 7, 7168, device=dev)
        o = torch.empty(H, T, D, device=dev, dtype=torch.bfloat16)
        ms = timed(lambda: sp(q[0], k[0], v[0], beta[0], g[0], S0, o=o), args.steps)
        sp.check_status()
        line("cfg4-split", "long-context GDN B1 H64 T131072 D128, S0, head/tail split in one GPU",
             ms, B * T, B * H * T * 1030 + B * H * D * D * 4 * 2, "bfloat16")
        sp.close()
        del q, k, v, beta, g, o

    if want("kda"):
        # KDA (per-dimension gate; the reference's next family): the fused tensor-core
        # forward at config 3's shape, g = -U(0,1) * 0.05 per token and dimension
        from pto_fuser import KDAChunkForward
        B, H, T, D = 16, 16, 4096, 64
        q = nrm(torch.randn(B, H, T, D, device=dev, generator=gen), dim=-1).bfloat16()
        k = nrm(torch.randn(B, H, T, D, device=dev, generator=gen), dim=-1).bfloat16()
        v = torch.randn(B, H, T, D, device=dev, generator=gen).bfloat16()
        beta = torch.sigmoid(torch.randn(B, H, T, device=dev, generator=gen)).bfloat16()
        g = -torch.rand(B, H, T, D, device=dev, generator=gen) * 0.05
        r = KDAChunkForward(B, H, T, D)
        o = torch.empty_like(v)
        S = torch.empty(B, H, D, D, device=dev)
        ms = timed(lambda: r(q, k, v, beta, g, o=o, final_state=S), args.steps)
        r.check_status()
        # algorithmic bytes: q, k, v, o bf16, beta bf16, g fp32 per (token, dimension),
        # plus the final state (the operand pre-pass's own traffic is not algorithmic)
        algo = B * H * T * (4 * D * 2 + 2 + 4 * D) + B * H * D * D * 4
        line("kda", "KDA forward bf16 B16 H16 T4096 D64 (fused tcgen05, operand pre-pass)", ms,
             B * T, algo, "bfloat16")
        r.close()


def run_long(args):
    """Config 4 (one long sequence, few heads) with the token axis split over the
    ranks: the chunk-segment scan (pto_fuser.segment), strong scaling. Each rank holds
    its token range of all 64 heads (inputs drawn on its device, S0 identical on every
    rank); the timed step is the whole segment-parallel forward including the NCCL
    all-gather of the segment maps. N = 1 with one segment is the serial forward."""
    import torch
    import torch.distributed as dist
    world, rank, local = _dist()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    from pto_fuser import GDNChunkForward
    from pto_fuser.segment import GDNSegmentScan, split_tokens
    B, H, T, D = 1, 64, args.long_tokens or 131072, 128
    P = B * H
    Tl = split_tokens(T, world)[rank]
    segs = args.segments if args.segments else 1
    gen = torch.Generator(device=dev).manual_seed(4321 + rank)
    nrm = torch.nn.functional.normalize
    bf = torch.bfloat16
    q = nrm(torch.randn(P, Tl, D, device=dev, generator=gen), dim=-1).to(bf)
    k = nrm(torch.randn(P, Tl, D, device=dev, generator=gen), dim=-1).to(bf)
    v = torch.randn(P, Tl, D, device=dev, generator=gen).to(bf)
    beta = torch.sigmoid(torch.randn(P, Tl, device=dev, generator=gen)).to(bf)
    g = torch.nn.functional.logsigmoid(torch.randn(P, Tl, device=dev, generator=gen) + 3.0)
    S0 = torch.randn(P, D, D, device=dev,
                     generator=torch.Generator(device=dev).manual_seed(99)) * 0.02
    o = torch.empty(P, Tl, D, device=dev, dtype=bf)
    if world == 1 and segs == 1:
        run = GDNChunkForward(B, H, Tl, D, D, device=dev)
        S = torch.empty(B, H, D, D, device=dev)
        step = lambda: run(q[None], k[None], v[None], beta[None], g[None], S0[None],
                           o=o[None], final_state=S)
        launches = 2
        check = [run]
        how = "serial chunk scan (one CTA per head)"
    else:
        run = GDNSegmentScan(P, Tl, D, segments=segs,
                             group=dist.group.WORLD if world > 1 else None, device=dev)
        step = lambda: run(q, k, v, beta, g, S0, o=o)
        launches = 2 + 2 + (2 if world > 1 else 0) + (1 if rank > 0 else 0) + 1 + 1
        check = [run]
        how = f"chunk-segment scan: {world} rank(s) x {segs} sub-segments, NCCL all-gather"
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    for r in check:
        r.check_status()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        barrier()
    for r in check:
        r.check_status()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    hbm = _peaks()[0]
    algo = B * H * T * 1030 + B * H * D * D * 4 * 2
    if rank == 0:
        print(json.dumps({
            "metric": "GDN chunk-forward tokens/s, long context (config 4), whole box",
            "value": B * T / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"cfg4: GDN forward B1 H64 T{T} D128 bf16, S0 ~ N(0,0.02^2), "
                                   "g = logsigmoid(N(3,1))", "parallelism": how,
                       "tokens_per_rank": Tl,
                       "l2": f"{algo / 1e9:.2f} GB of operands vs 126 MB L2 (no flush needed)"},
            "roofline": {"bound": "hbm", "algo_bytes": algo,
                         "achieved": algo / (ms / 1e3) / 1e9, "peak": hbm * world,
                         "unit": "GB/s", "frac": algo / (ms / 1e3) / 1e9 / (hbm * world),
                         "peak_kind": "measured, per GPU x n_gpus"},
            "gpu_launches": launches * args.steps, "clocks": clk.summary()}), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--configs", action="store_true",
                    help="one supporting JSON line per BASELINE configuration (0-4), 1 GPU")
    ap.add_argument("--only", nargs="+", metavar="NAME",
                    help="with --configs: only these lines (cfg0 cfg1 cfg2 cfg3 cfg4 cfg4-split "
                         "kda), e.g. for a launch list of one configuration")
    ap.add_argument("--shape", type=int, nargs=4, metavar=("B", "H", "T", "D"),
                    help="per-GPU problem other than config 2 (small cases for profiling; "
                         "not a bench line of the headline metric)")
    ap.add_argument("--long-context", action="store_true",
                    help="config 4 (B1 H64 T131072) with the token axis split over the ranks "
                         "(chunk-segment scan, strong scaling)")
    ap.add_argument("--long-tokens", type=int, default=0,
                    help="sequence length for --long-context other than config 4's 131072 "
                         "(small cases for profiling; not a bench line of config 4)")
    ap.add_argument("--segments", type=int, default=0,
                    help="sub-segments per rank for --long-context (default 1; on one GPU 1 is "
                         "the serial forward)")
    args = ap.parse_args()
    if args.shape:
        CFG.update(B=args.shape[0], H=args.shape[1], T=args.shape[2], D=args.shape[3])
    if args.configs:
        run_configs(args)
    elif args.long_context:
        run_long(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
