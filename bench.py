"""Benchmark of the Anima DiT attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--L 4096] [--shard heads|replicas] [--workload attn|dit|schedules|qkv]

One step = one fused attention call of one DiT block over one synthetic batch: per-head
q/k RMSNorm + 3D RoPE + bf16 cast (prologue kernel) and the tcgen05 flash attention
(attention kernel), B=2 (CFG pair) x 16 heads x L tokens x D=128, inputs resident in HBM.
The default L=4096 is the 4096-token point of the sequence-length sweep (1024x1024 image),
the point the target is quoted on; the other configurations are reported in the same JSON
line as sections of their own.

Headline line (rank 0 prints one JSON line):
  value         attention TFLOP/s of the whole job (4*B*H*L^2*D per step / step time).
  e2e           the same metric through the reference-facing host C ABI
                (anima_rt_run_attention) with page-locked host buffers, copies inside the
                timed region; e2e_pageable the same with ordinary (pageable) host arrays,
                as the reference's numpy callers pass them.
  roofline      the attention kernel alone (CUDA events on its stream) against the measured
                dense bf16 peak (MEASURED_PEAKS.json); prologue_roofline against HBM.
  cpu_baseline  the reference's anima_rt CPU path (oracle/_ref, compiled from the reference
                sources; the C restatement if that is absent), run BEFORE any GPU work by the
                same function and step counts as --impl reference: all host cores and one
                core, plus the prologue alone (two anima_rt_run_rmsnorm calls, the numpy RoPE
                and the transposes of the reference's NumpyAttention.forward).
  cross_attention  config 3: q RMSNorm + masked cross-attention, Lq=4096, Lk=512, valid
                lengths U{32..512} from the seed, masked FLOP count, tensor and AI-bound
                rooflines.
  sweep         config 5: fused prologue + attention at L in {256, 1024, 4096, 9216, 16384}.
  library_anchor  torch's cuDNN SDPA on the same bf16 operands (a library reference point).
  dit_step      config 4: one 28-block Euler+CFG DiT step replayed as a CUDA graph, ms at N
                GPUs in the head-parallel layout (and, for N > 1, the token-split layout),
                with CUDA-event shares of GEMMs, attention, fused passes and collectives in an
                eager step.

Other workloads (one JSON object each): schedules (the attention kernel's three schedules on
given shapes) and qkv (anima_qkv_projection, the q/k/v projection GEMM with the prologue in its
epilogue, against a cuBLAS GEMM followed by the prologue kernel, at the DiT's shapes).

Multi-GPU (torchrun, one process per GPU): "heads" (default) splits the 16 heads over the
ranks (strong scaling; N=1 is the full problem); "replicas" runs the whole workload on every
rank (independent CFG batches, weak scaling).  Timing is the max over ranks.
"""
from __future__ import annotations

import argparse
import ctypes as ct
import json
import math
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(REPO, "anima-on-android_b200")
for _p in (PKG_ROOT, REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "attn TFLOP/s per B200 (% dense BF16 peak); DiT step ms at 1/2/4/8 GPUs"
UNIT = "TFLOP/s"
B, H, D = 2, 16, 128
SWEEP = (256, 1024, 4096, 9216, 16384)


def attn_flops(b, h, lq, lk, d=D):
    return 4.0 * b * h * lq * lk * d


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"tflops": p["bf16_tflops"], "tflops_sustained": p["bf16_tflops_sustained"],
                "hbm_gbs": p["hbm_gbs"], "source": "measured"}
    return {"tflops": 1590.0, "tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def load_traffic(L):
    """dram read+write bytes per launch of each kernel, from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    if not os.path.exists(path):
        return {}
    with open(path) as f:
        t = json.load(f)
    return t.get(str(L), {})


# ---------------------------------------------------------------- clocks (NVML)
class ClockSampler:
    """NVML sampler of SM clock, power and throttle reasons on a background thread.

    Samples carry host timestamps; summary(t0, t1) reports the samples taken inside the
    timed region [t0, t1] (or the whole sampling window when the region was too short
    for three samples, which is then stated)."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting"}

    def __init__(self, index):
        self.samples = []  # (t, sm_mhz, power_w, reasons_mask)
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False
        self._stop = threading.Event()

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                t = time.perf_counter()
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((t, mhz, pw, r))
            except Exception:
                pass
            time.sleep(0.001)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self, t0=None, t1=None):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        inside = [s for s in self.samples if t0 is not None and t0 <= s[0] <= t1]
        window = "timed region"
        if len(inside) < 3:
            inside, window = self.samples, "warm-up + timed region (timed region too short)"
        reasons = set()
        for s in inside:
            for bit, name in self.REASONS.items():
                if s[3] & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(inside), "window": window,
                "power_w_median": round(statistics.median(s[2] for s in inside), 1)}


# ---------------------------------------------------------------- inputs
def make_inputs(L, heads, seed):
    import numpy as np
    rng = np.random.default_rng(seed)
    side = int(round(math.sqrt(L)))
    assert side * side == L, "L must be a square latent grid"
    q, k, v = (rng.standard_normal((B, L, heads, D), dtype=np.float32) for _ in range(3))
    qw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    return q, k, v, qw, kw, side


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


# ---------------------------------------------------------------- reference CPU path
def cpu_reference(L, steps, warmup, seed=0, threads=None):
    """anima_rt's CPU path on the host cores, a bounded sample per step: every thread runs
    the reference sequence (rmsnorm q,k -> rope q,k -> flash SDPA) for one (b, h) head over
    a block of query rows against all L keys.  Query rows and heads are independent, so
    TFLOP/s over the sample equals TFLOP/s of the whole workload.  threads=None uses every
    core this process may run on; 1 gives the reference's own single-core design."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    from oracle import oracle as O

    kind = "reference" if O.have_reference() else "port"
    be = O.backend(kind)
    if kind == "reference":
        be.lib.anima_rt_init()
    cores = threads or len(os.sched_getaffinity(0))
    rows = 256 if L >= 4096 else min(L, 512)
    rng = np.random.default_rng(seed)
    side = int(round(math.sqrt(L)))
    freqs = O.rope_freqs_3d(1, side, side)
    qw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    work = []
    for t in range(cores):
        q = rng.standard_normal((rows, D), dtype=np.float32)
        k = rng.standard_normal((L, D), dtype=np.float32)
        v = rng.standard_normal((L, D), dtype=np.float32)
        q0 = int(rng.integers(0, L - rows + 1))
        work.append((q, k, v, q0, np.zeros((rows, D), np.float32), np.zeros_like(q),
                     np.zeros_like(k), np.zeros_like(q), np.zeros_like(k)))

    def one(wi):
        q, k, v, q0, out, qn, kn, qr, kr = wi
        be.rmsnorm(q.ctypes.data, qw.ctypes.data, qn.ctypes.data, rows, D, 1e-6)
        be.rmsnorm(k.ctypes.data, kw.ctypes.data, kn.ctypes.data, L, D, 1e-6)
        be.rope(qn.ctypes.data, freqs[q0:q0 + rows].ctypes.data, qr.ctypes.data, 1, rows, D)
        be.rope(kn.ctypes.data, freqs.ctypes.data, kr.ctypes.data, 1, L, D)
        be.sdpa_flash(qr.ctypes.data, kr.ctypes.data, v.ctypes.data, out.ctypes.data, 1, rows, L,
                      D, 1.0 / math.sqrt(D), False)

    times = []
    with ThreadPoolExecutor(cores) as ex:
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            list(ex.map(one, work))
            if i >= warmup:
                times.append(time.perf_counter() - t0)
    step_s = statistics.median(times)
    value = attn_flops(1, cores, rows, L) / step_s / 1e12
    sample = (f"{cores} thread(s) x one (b,h) head each: {rows} query rows x {L} keys "
              f"(rmsnorm+rope+flash SDPA), {attn_flops(1, 1, rows, L) / 1e9:.2f} GFLOP per thread, "
              f"median of {steps} steps after {warmup} warm-up; per-row work identical, so "
              f"TFLOP/s is that of the full B={B} H={H} L={L} step")
    return {"value": value, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample,
            "ms_per_step": step_s * 1e3, "cpu_model": _cpu_model()}


def cpu_prologue(L, steps, warmup, seed=0):
    """The reference's prologue on the host, full size: two anima_rt_run_rmsnorm calls over
    the [B*L*H, 128] q and k rows, the numpy RoPE of NumpyAttention.forward
    (anima_rt/scripts/numpy_dit.py:285-291) and the transposes to [B, H, L, D] that
    NumpyRT.run_sdpa makes contiguous.  Reported as the same algorithmic bytes per second
    as the GPU prologue (read q, k, v fp32, write three 16-bit operands)."""
    import numpy as np
    from oracle import oracle as O

    kind = "reference" if O.have_reference() else "port"
    be = O.backend(kind)
    if kind == "reference":
        be.lib.anima_rt_init()
    q, k, v, qw, kw, side = make_inputs(L, H, seed)
    freqs = O.rope_freqs_3d(1, side, side)
    M = B * L * H

    def step():
        qn, kn = np.empty_like(q), np.empty_like(k)
        be.rmsnorm(q.ctypes.data, qw.ctypes.data, qn.ctypes.data, M, D, 1e-6)
        be.rmsnorm(k.ctypes.data, kw.ctypes.data, kn.ctypes.data, M, D, 1e-6)
        qr, kr = O.numpy_rope(qn, freqs), O.numpy_rope(kn, freqs)
        return [np.ascontiguousarray(t.transpose(0, 2, 1, 3)) for t in (qr, kr, v)]

    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        step()
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    s = statistics.median(times)
    nbytes = 3 * B * L * H * D * 4 + 3 * B * L * H * D * 2
    return {"value": round(nbytes / s / 1e9, 2), "unit": "GB/s", "ms_per_step": round(s * 1e3, 2),
            "cores": 1, "kind": kind,
            "sample": f"full B={B} H={H} L={L}: rmsnorm q,k (anima_rt) + numpy RoPE q,k + "
                      f"transposes; {nbytes / 1e6:.0f} MB of algorithmic bytes per step"}


def cpu_baselines(L, steps, warmup):
    """Every CPU figure of the line, measured before any GPU work of the process."""
    allc = cpu_reference(L, steps, warmup)
    one = cpu_reference(L, max(2, min(steps, 5)), 1, threads=1)
    pro = cpu_prologue(L, max(2, min(steps, 3)), 1)
    return {"value": round(allc["value"], 5), "unit": UNIT, "cores": allc["cores"],
            "kind": allc["kind"], "sample": allc["sample"], "cpu_model": allc["cpu_model"],
            "ms_per_step": round(allc["ms_per_step"], 2),
            "cores_all": {"value": round(allc["value"], 5), "cores": allc["cores"]},
            "cores_1": {"value": round(one["value"], 6), "cores": 1,
                        "ms_per_step": round(one["ms_per_step"], 2)},
            "prologue": pro}


# ---------------------------------------------------------------- helpers (GPU)
def _barrier(dist):
    import torch
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(vals, dist, dev):
    import torch
    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


_FLUSH = {}


def _flush_l2(dev):
    """Write 256 MiB (twice the 126 MB L2) so the next call starts with a cold L2."""
    import torch
    buf = _FLUSH.get(str(dev))
    if buf is None:
        buf = _FLUSH[str(dev)] = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    buf.zero_()


L2_BYTES = 126e6  # B200 L2; calls whose inputs are smaller flush it between timed calls


def _head_start(steps):
    """A GPU-side delay queued before a timed loop (about 0.5 ms per step, at most 20 ms), so
    that the host enqueues every timed call before the GPU reaches the first one and no
    host-side launch time (Python wrappers, eight ranks sharing the host's cores) falls
    inside a call's events."""
    import torch
    torch.cuda._sleep(int(min(20.0, 0.5 * steps) * 1.0e6))  # ~1e6 cycles per ms at 1-2 GHz


def _time_events(fn, steps, warmup, dist, dev, flush=True):
    """Device time per call of fn: CUDA events around each call on the current stream; with
    flush (inputs smaller than L2) a 256 MiB write before every call, outside the events;
    mean over calls, max over ranks."""
    import torch
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    _barrier(dist)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    _head_start(steps)
    for e0, e1 in evs:
        if flush:
            _flush_l2(dev)
        e0.record(stream)
        fn()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / steps
    _barrier(dist)
    return _max_over_ranks([ms], dist, dev)[0]


# ---------------------------------------------------------------- headline (config 5 @ L)
def run_ours(args, rank, world, local_rank, dist):
    import numpy as np
    import torch
    import anima_attn
    from anima_attn import _lib as L

    dev = torch.device("cuda", local_rank)
    L_ = args.L
    heads = H if args.shard == "replicas" else H // world
    q, k, v, qw, kw, side = make_inputs(L_, heads, seed=args.seed + rank)
    freqs = anima_attn.rope_freqs_3d(1, side, side, device=dev)
    dq, dk, dv = (torch.from_numpy(a).to(dev) for a in (q, k, v))
    dqw, dkw = torch.from_numpy(qw).to(dev), torch.from_numpy(kw).to(dev)
    ws = tuple(torch.empty((B * heads, L_, D), device=dev, dtype=torch.bfloat16) for _ in range(3))
    out = torch.empty((B, L_, heads, D), device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream()

    def step(evs=None):
        if evs is not None:
            evs[0].record(stream)
        qh, kh, vh = anima_attn.prologue(dq, dk, dv, dqw, dkw, freqs, out=ws)
        if evs is not None:
            evs[1].record(stream)
        anima_attn.attention_core(qh, kh, vh, B, heads, out=out, schedule=args.schedule)
        if evs is not None:
            evs[2].record(stream)

    in_bytes = 3 * B * L_ * heads * D * 4
    flush = in_bytes < L2_BYTES
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    clocks = ClockSampler(local_rank)
    with clocks:
        for _ in range(args.warmup):
            step()
        _barrier(dist)
        t_begin = time.perf_counter()
        _head_start(args.steps)
        for i in range(args.steps):
            if flush:
                _flush_l2(dev)  # outside the step's events: the step starts with a cold L2
            step(evs[i])
        torch.cuda.synchronize()
        t_end = time.perf_counter()
        _barrier(dist)
    if anima_attn.status() != 0:
        raise SystemExit("device status word reports a kernel timeout")
    total_ms = sum(e[0].elapsed_time(e[2]) for e in evs)
    pro_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    att_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    total_ms, pro_ms, att_ms = _max_over_ranks([total_ms, pro_ms, att_ms], dist, dev)
    ms_step = total_ms / args.steps
    flops_rank = attn_flops(B, heads, L_, L_)
    value = flops_rank * world / (ms_step * 1e-3) / 1e12

    # ---- e2e through the host C ABI: page-locked buffers, then ordinary numpy arrays
    e2e = e2e_pageable = None
    if not args.no_e2e:
        pq, pk, pv = (torch.from_numpy(a).pin_memory() for a in (q, k, v))
        pqw, pkw = torch.from_numpy(qw).pin_memory(), torch.from_numpy(kw).pin_memory()
        pf = freqs.cpu().pin_memory()
        pout = torch.empty((B, L_, heads, D), dtype=torch.float32).pin_memory()
        nf, nout = freqs.cpu().numpy(), np.zeros((B, L_, heads, D), np.float32)
        assert L.lib.anima_rt_init()
        flags = L.FLAG_QNORM | L.FLAG_KNORM | L.FLAG_ROPE

        def timed(ptrs, optr):
            def host_step():
                ok = L.lib.anima_rt_run_attention(*ptrs, None, optr, B, L_, L_, heads, D,
                                                  ct.c_float(1e-6), ct.c_float(1 / math.sqrt(D)),
                                                  flags)
                if not ok:
                    raise SystemExit("anima_rt_run_attention failed: " + L.last_error())
            for _ in range(max(1, min(args.warmup, 3))):
                host_step()
            n = max(3, min(args.steps, 20))
            _barrier(dist)
            t0 = time.perf_counter()
            for _ in range(n):
                host_step()
            el = _max_over_ranks([time.perf_counter() - t0], dist, dev)[0]
            return el / n, n

        h2d = 3 * q.nbytes + nf.nbytes + 2 * D * 4
        s, n = timed((pq.data_ptr(), pk.data_ptr(), pv.data_ptr(), pqw.data_ptr(),
                      pkw.data_ptr(), pf.data_ptr()), pout.data_ptr())
        e2e = {"value": flops_rank * world / s / 1e12, "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": pout.numel() * 4, "ms_per_step": s * 1e3, "steps": n,
               "path": "anima_rt_run_attention (C ABI, page-locked host buffers, wall clock)"}
        host_ptrs = (q.ctypes.data, k.ctypes.data, v.ctypes.data, qw.ctypes.data,
                     kw.ctypes.data, nf.ctypes.data)
        s, n = timed(host_ptrs, nout.ctypes.data)
        # the same call with the library's page-locked staging ring turned off: the CUDA
        # driver's own pageable copies
        os.environ["ANIMA_RT_STAGE"] = "0"
        try:
            s_drv, _ = timed(host_ptrs, nout.ctypes.data)
        finally:
            os.environ.pop("ANIMA_RT_STAGE", None)
        e2e_pageable = {"value": flops_rank * world / s / 1e12, "unit": UNIT,
                        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": nout.nbytes,
                        "ms_per_step": s * 1e3, "steps": n,
                        "driver_copies": {"value": flops_rank * world / s_drv / 1e12,
                                          "ms_per_step": s_drv * 1e3},
                        "path": "anima_rt_run_attention (C ABI, pageable numpy arrays, as the "
                                "reference's callers pass them, copied through the library's "
                                "page-locked staging ring; wall clock)"}

    peaks = load_peaks()
    achieved = flops_rank / (att_ms * 1e-3) / 1e12
    sched_flags = {"auto": 0, "unit": L.FLAG_UNIT, "whole": L.FLAG_WHOLE, "split": L.FLAG_SPLIT}
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    sched_run = {0: "unit", 1: "whole", 2: "cut"}.get(
        L.lib.anima_attn_schedule(B, heads, L_, L_, sched_flags[args.schedule], sms), "error")
    traffic = load_traffic(L_).get("attn_fwd")
    pro_bytes = (3 * B * L_ * heads * D * 4) + (3 * B * L_ * heads * D * 2)
    return {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak" if args.shard == "replicas" else "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v, N(1,0.1) norm weights)",
        "config": {"workload": f"fused q/k RMSNorm + 3D RoPE + flash attention (prologue + tcgen05 "
                               f"attention), B={B} H={H} L={L_} D={D}, BASELINE config 5 @ L={L_}",
                   "global_batch": B * (world if args.shard == "replicas" else 1), "seq_len": L_,
                   "heads_per_gpu": heads, "parallelism": f"{args.shard}{world}",
                   "l2": (f"inputs {in_bytes / 2**20:.0f} MiB fp32 < 126 MB L2: L2 flushed "
                          "(256 MiB write) before every timed step, outside its events" if flush
                          else f"inputs {in_bytes / 2**20:.0f} MiB fp32 > 126 MB L2"),
                   "attn_ms": round(att_ms, 4), "prologue_ms": round(pro_ms, 4),
                   "schedule": args.schedule, "schedule_run": sched_run,
                   "prologue_gbs": round(pro_bytes / (pro_ms * 1e-3) / 1e9, 1),
                   "pct_of_dense_bf16_peak": round(100 * value / world / peaks["tflops"], 2)},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["tflops"],
                     "unit": "TFLOP/s", "frac": round(achieved / peaks["tflops"], 4),
                     "traffic": traffic, "kernel": "attn_fwd_kernel",
                     "peak_source": f"{peaks['source']} (bf16_tflops burst)"},
        "prologue_roofline": {"bound": "hbm", "achieved": round(pro_bytes / (pro_ms * 1e-3) / 1e9, 1),
                              "peak": peaks["hbm_gbs"], "unit": "GB/s",
                              "frac": round(pro_bytes / (pro_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                              "traffic": load_traffic(L_).get("prologue")},
        "e2e": e2e,
        "e2e_pageable": e2e_pageable,
        "gpu_launches": 2 * args.steps,
        "clocks": clocks.summary(t_begin, t_end),
    }


# ---------------------------------------------------------------- config 3
def run_cross(args, rank, world, local_rank, dist):
    """Masked cross-attention of config 3: q [2, 4096, 16, 128] ~N(0,1) with q RMSNorm
    (w ~N(1, 0.1)), context [2, 512, 1024] ~N(0,1) projected to K/V by bf16 weights [2048,
    1024] ~N(0, 0.02) (timed separately), key-padding mask with valid_b ~ U{32..512}.  The
    step is the prologue (q norm, 16-bit operands) and the masked attention."""
    import numpy as np
    import torch
    import anima_attn

    dev = torch.device("cuda", local_rank)
    Lq, Lk, C = 4096, 512, 1024
    heads = H if args.shard == "replicas" else H // world
    rng = np.random.default_rng(args.seed + 3 + rank)
    q = torch.from_numpy(rng.standard_normal((B, Lq, heads, D), dtype=np.float32)).to(dev)
    ctx = torch.from_numpy(rng.standard_normal((B, Lk, C), dtype=np.float32)).to(dev)
    wkv = torch.from_numpy((0.02 * rng.standard_normal((2 * heads * D, C))).astype(np.float32))
    wkv = wkv.to(dev).to(torch.bfloat16)
    qw = torch.from_numpy((1 + 0.1 * rng.standard_normal(D)).astype(np.float32)).to(dev)
    valid = rng.integers(32, 513, size=B).astype(np.int32)
    dvalid = torch.from_numpy(valid).to(dev)
    out = torch.empty((B, Lq, heads, D), device=dev)

    def project():  # bf16 operands, fp32 accumulation and output (the prologue's input type)
        return torch.mm(ctx.reshape(B * Lk, C).to(torch.bfloat16), wkv.t(),
                        out_dtype=torch.float32).view(B, Lk, 2, heads, D)

    kv = project()
    k, v = kv[:, :, 0], kv[:, :, 1]
    bufs = (torch.empty((B * heads, Lq, D), device=dev, dtype=torch.bfloat16),
            torch.empty((B * heads, Lk, D), device=dev, dtype=torch.bfloat16),
            torch.empty((B * heads, Lk, D), device=dev, dtype=torch.bfloat16))
    ops = {}

    def pro():
        ops["qkv"] = anima_attn.prologue(q, k, v, qw, None, None, norm_q=True, norm_k=False, out=bufs)

    def att():
        qh, kh, vh = ops["qkv"]
        anima_attn.attention_core(qh, kh, vh, B, heads, kv_valid_len=dvalid, out=out)

    pro()
    proj_ms = _time_events(project, args.steps, args.warmup, dist, dev)
    pro_ms = _time_events(pro, args.steps, args.warmup, dist, dev)
    att_ms = _time_events(att, args.steps, args.warmup, dist, dev)
    if anima_attn.status() != 0:
        raise SystemExit("device status word reports a kernel timeout")
    peaks = load_peaks()
    masked = 4.0 * heads * D * Lq * float(valid.sum())
    unmasked = attn_flops(B, heads, Lq, Lk)
    # bytes the attention kernel must move: Q and the valid K/V rows (bf16), O fp32
    att_bytes = B * heads * (Lq * D * 2 + 2 * float(valid.mean()) * D * 2 + Lq * D * 4)
    ai = masked / att_bytes
    bound = min(peaks["tflops"], ai * peaks["hbm_gbs"] / 1e3)
    achieved = masked / (att_ms * 1e-3) / 1e12
    pro_bytes = B * heads * (Lq * D * 4 + Lq * D * 2 + 2 * Lk * D * (4 + 2))
    return {"workload": f"config 3: q RMSNorm + masked cross-attention B={B} H={heads} "
                        f"Lq={Lq} Lk={Lk}, valid lengths {valid.tolist()}",
            "attn_ms": round(att_ms, 4), "prologue_ms": round(pro_ms, 4),
            "kv_projection_ms": round(proj_ms, 4),
            "tflops_masked": round(achieved * world, 1),
            "tflops_unmasked_equivalent": round(unmasked / (att_ms * 1e-3) / 1e12 * world, 1),
            "flop_masked": masked * world, "flop_unmasked": unmasked * world,
            "step_tflops_masked": round(masked * world / ((att_ms + pro_ms) * 1e-3) / 1e12, 1),
            "roofline": {"tensor_frac": round(achieved / peaks["tflops"], 4),
                         "arithmetic_intensity": round(ai, 1),
                         "ai_bound_tflops": round(bound, 1),
                         "ai_bound_frac": round(achieved / bound, 4)},
            "prologue_gbs": round(pro_bytes / (pro_ms * 1e-3) / 1e9, 1)}


# ---------------------------------------------------------------- config 5 sweep
def run_sweep(args, rank, world, local_rank, dist):
    import torch
    import anima_attn

    dev = torch.device("cuda", local_rank)
    peaks = load_peaks()
    heads = H if args.shard == "replicas" else H // world
    res = {}
    for Ls in SWEEP:
        side = int(round(math.sqrt(Ls)))
        g = torch.Generator(device=dev).manual_seed(args.seed + Ls + rank)
        q, k, v = (torch.randn((B, Ls, heads, D), device=dev, generator=g) for _ in range(3))
        qw = 1 + 0.1 * torch.randn(D, device=dev, generator=g)
        kw = 1 + 0.1 * torch.randn(D, device=dev, generator=g)
        freqs = anima_attn.rope_freqs_3d(1, side, side, device=dev)
        bufs = tuple(torch.empty((B * heads, Ls, D), device=dev, dtype=torch.bfloat16)
                     for _ in range(3))
        out = torch.empty((B, Ls, heads, D), device=dev)

        def step():
            qh, kh, vh = anima_attn.prologue(q, k, v, qw, kw, freqs, out=bufs)
            anima_attn.attention_core(qh, kh, vh, B, heads, out=out)

        n = args.steps if Ls < 16384 else max(3, args.steps // 4)
        ms = _time_events(step, n, args.warmup, dist, dev,
                          flush=3 * B * Ls * heads * D * 4 < L2_BYTES)
        fl = attn_flops(B, heads, Ls, Ls) * world
        res[str(Ls)] = {"ms": round(ms, 4), "tflops": round(fl / (ms * 1e-3) / 1e12, 1),
                        "pct_of_dense_bf16_peak": round(100 * fl / world / (ms * 1e-3) / 1e12 /
                                                        peaks["tflops"], 2)}
        del q, k, v, bufs, out
    if anima_attn.status() != 0:
        raise SystemExit("device status word reports a kernel timeout")
    return res


def run_anchor(args, rank, world, local_rank, dist):
    """torch's cuDNN SDPA on bf16 [B, H, L, D] operands of the headline shape and of the
    longest sweep point: a library reference point for the attention kernel alone."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    dev = torch.device("cuda", local_rank)
    heads = H if args.shard == "replicas" else H // world
    res = {}
    for Ls in (args.L, 16384):
        q, k, v = (torch.randn((B, heads, Ls, D), device=dev, dtype=torch.bfloat16) for _ in range(3))
        try:
            with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
                ms = _time_events(lambda: F.scaled_dot_product_attention(q, k, v),
                                  args.steps if Ls < 16384 else 5, args.warmup, dist, dev)
            res[f"cudnn_sdpa_L{Ls}"] = {"ms": round(ms, 4), "tflops": round(
                attn_flops(B, heads, Ls, Ls) * world / (ms * 1e-3) / 1e12, 1)}
        except Exception as ex:  # noqa: BLE001 -- an anchor that cannot run is reported as such
            res[f"cudnn_sdpa_L{Ls}"] = f"unavailable: {str(ex)[:120]}"
        del q, k, v
    return res


# ---------------------------------------------------------------- DiT step (config 4)
def dit_flops(blocks=28, L=4096, B=2, ctx=512, hidden=2048, mlp=8192, ctx_dim=1024):
    """Matmul FLOP of one CFG-batched forward (GEMMs + attention), as counted for the
    config: per block self q/k/v/o, cross q/o, cross k/v, MLP, and both attentions."""
    g = lambda m, n, k: 2.0 * m * n * k
    per = (4 * g(B * L, hidden, hidden) + 2 * g(B * L, hidden, hidden) +
           2 * g(B * ctx, hidden, ctx_dim) + g(B * L, mlp, hidden) + g(B * L, hidden, mlp) +
           attn_flops(B, 16, L, L) + attn_flops(B, 16, L, ctx))
    return blocks * per


def sampler_run(model, x, cc, cu, args, dist, dev, steps):
    """A whole sampling run (EulerSampler.sample over the z_image schedule) with the
    cross-attention K/V of every block prepared once per run: the precompute, and the
    steps replayed from one captured graph, each timed with CUDA events (max over ranks)."""
    import torch
    from anima_attn.sampling import EulerCFGSampler, z_image_sigmas

    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    s = EulerCFGSampler(model, cc, cu, 5.0, x.shape, graph=bool(args.graph))
    sig = z_image_sigmas(steps)
    s.sample(x, sig)  # warm
    _barrier(dist)
    e[0].record()
    s.refresh_context(cc, cu)  # the per-run precompute: K/V of every block's cross-attention
    e[1].record()
    s.sample(x, sig)
    e[2].record()
    torch.cuda.synchronize()
    pre, run = _max_over_ranks([e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2])], dist, dev)
    del s
    return {"steps": steps, "schedule": "z_image (shift 3)", "context_precompute_ms": round(pre, 3),
            "ms_per_step": round(run / steps, 3), "run_ms": round(pre + run, 3),
            "cuda_graph": bool(args.graph)}


def dit_step_ms(args, rank, world, local_rank, dist, shard, profile=True, sampler_steps=0,
                fused_qkv=True, peer_gather=True, peer_a2a=True):
    """One Euler+CFG step of the Anima DiT (config 4): latent 16x128x128 (4096 tokens), 28
    blocks, hidden 2048, 16 heads, CFG pair batched (B=2), sigma 0.5 -> 0, cfg 5; attention
    split by head over the ranks in the given layout.  fused_qkv: q/k/v projections through
    anima_qkv_projection (else cuBLAS GEMMs + the attention prologue).  Returns device ms
    per step (graph replay, max over ranks), e2e ms through host tensors, clocks and the
    eager breakdown."""
    import torch
    from anima_attn.dit import AnimaDiT, DiTConfig, StepGraph, make_weights, profile_step

    dev = torch.device("cuda", local_rank)
    cfg = DiTConfig(blocks=args.blocks)
    group = None
    if world > 1:
        import torch.distributed as tdist
        group = tdist.group.WORLD
    if args.weights:
        from anima_attn.checkpoint import load_dit_weights
        weights = load_dit_weights(args.weights, cfg, device=dev)
    else:
        weights = make_weights(cfg, seed=1234, device=dev, rng_device=dev)
    model = AnimaDiT(cfg, weights, rank=rank, world=world, group=group, shard=shard,
                     fused_qkv=fused_qkv, peer_gather=peer_gather, peer_a2a=peer_a2a)
    del weights
    side = args.latent
    g = torch.Generator(device=dev).manual_seed(4321)
    x = torch.randn(1, 16, side, side, device=dev, generator=g)
    cc = torch.randn(1, 512, 1024, device=dev, generator=g)
    cu = torch.randn(1, 512, 1024, device=dev, generator=g)
    with torch.no_grad():
        if profile:  # an eager step first: library start-up stays out of the breakdown
            model.euler_cfg_step(x, 0.5, 0.0, cc, cu, 5.0)
            breakdown = profile_step(model, x, 0.5, 0.0, cc, cu, 5.0)
        else:
            breakdown = None
        if args.graph:
            graph = StepGraph(model, x, 0.5, 0.0, cc, cu, 5.0)
            run_step = lambda xx=None, c1=None, c2=None: graph(xx, c1, c2)
        else:
            graph = None
            run_step = lambda xx=None, c1=None, c2=None: model.euler_cfg_step(
                x if xx is None else xx, 0.5, 0.0, cc if c1 is None else c1,
                cu if c2 is None else c2, 5.0)
        clocks = ClockSampler(local_rank)
        with clocks:
            for _ in range(args.warmup):
                run_step()
            _barrier(dist)
            stream = torch.cuda.current_stream()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t_begin = time.perf_counter()
            e0.record(stream)
            for _ in range(args.dit_steps):
                run_step()
            e1.record(stream)
            torch.cuda.synchronize()
            t_end = time.perf_counter()
            _barrier(dist)
        ms = e0.elapsed_time(e1) / args.dit_steps
        # end to end: host latent + contexts in, host latent out, every step
        hx, hcc, hcu = (t.cpu().pin_memory() for t in (x, cc, cu))
        hout = torch.empty_like(hx).pin_memory()

        def host_step():
            dx, dcc, dcu = (t.to(dev, non_blocking=True) for t in (hx, hcc, hcu))
            hout.copy_(run_step(dx, dcc, dcu), non_blocking=True)
            torch.cuda.synchronize()

        host_step()
        _barrier(dist)
        t0 = time.perf_counter()
        n_e2e = max(2, min(args.dit_steps, 5))
        for _ in range(n_e2e):
            host_step()
        e2e_ms = (time.perf_counter() - t0) / n_e2e * 1e3
        del graph, run_step  # a graph holding NCCL calls goes before the process group
        sampler = None
        if sampler_steps:
            sampler = sampler_run(model, x, cc, cu, args, dist, dev, sampler_steps)
    ms, e2e_ms = _max_over_ranks([ms, e2e_ms], dist, dev)
    Lt = (side // 2) ** 2
    fl = dit_flops(args.blocks, Lt)
    res = {"ms": round(ms, 3), "tflops_per_gpu": round(fl / world / (ms * 1e-3) / 1e12, 1),
           "e2e_ms": round(e2e_ms, 3),
           "e2e_bytes": {"h2d_per_step": (hx.numel() + hcc.numel() + hcu.numel()) * 4,
                         "d2h_per_step": hout.numel() * 4},
           "clocks": clocks.summary(t_begin, t_end), "breakdown_eager": breakdown,
           "layout": shard if world > 1 else "one GPU", "sampler": sampler,
           "qkv_projection": ("anima_qkv_projection (GEMM + norm/RoPE epilogue)" if model.fused_qkv
                              else "cuBLAS GEMM + attention prologue"),
           "head_gather": (None if world == 1 or shard != "heads" else
                           "attention epilogue stores to every rank over NVLink + 1-element "
                           "all-reduce" if model.peer_gather else "NCCL all_gather_into_tensor"),
           "all_to_all": (None if world == 1 or shard != "tokens" else
                          "projection and attention epilogues store to the owning ranks over "
                          "NVLink + 1-element all-reduces" if model.peer_a2a else
                          "NCCL all_to_all_single x2 per attention")}
    torch.cuda.synchronize()
    model.close()
    del model
    torch.cuda.empty_cache()
    return res


def run_dit_section(args, rank, world, local_rank, dist):
    shards = ["heads"] if world == 1 else ["heads", "tokens"]
    side = args.latent
    Lt = (side // 2) ** 2
    out = {"workload": f"Anima DiT Euler+CFG step, {args.blocks} blocks, latent 16x{side}x{side} "
                       f"({Lt} tokens), context 512x1024, CFG pair, sigma 0.5 -> 0, cfg 5",
           "dtype": "fp16 GEMM/attention operands, fp32 activations",
           "cuda_graph": bool(args.graph), "steps": args.dit_steps, "n_gpus": world,
           "model_tflop_per_step": round(dit_flops(args.blocks, Lt) / 1e12, 2),
           "data": ("synthetic (seeded latent and context, N(0,0.02) bf16-valued weights)"
                    if not args.weights else
                    f"synthetic latent and context; weights from {os.path.basename(args.weights)}")}
    for i, sh in enumerate(shards):
        out[sh] = dit_step_ms(args, rank, world, local_rank, dist, sh,
                              sampler_steps=args.sampler_steps if i == 0 else 0)
    if world == 1:  # the same step with the projections as cuBLAS GEMMs + the prologue
        out["heads_cublas_qkv"] = dit_step_ms(args, rank, world, local_rank, dist, "heads",
                                              fused_qkv=False)
    else:  # both layouts with NCCL collectives instead of the epilogues' peer stores
        out["heads_nccl_gather"] = dit_step_ms(args, rank, world, local_rank, dist, "heads",
                                               profile=False, peer_gather=False)
        out["tokens_nccl_a2a"] = dit_step_ms(args, rank, world, local_rank, dist, "tokens",
                                             profile=False, peer_a2a=False)
    out["ms"] = out["heads"]["ms"]
    return out


# ---------------------------------------------------------------- schedules
def run_schedules(args):
    """The attention kernel's three schedules on given shapes (B=2, H=--sched-heads, bf16
    operands, fp32 output): ANIMA_FLAG_UNIT (one CTA per 256-row unit), ANIMA_FLAG_WHOLE (persistent grid,
    whole units), ANIMA_FLAG_SPLIT (persistent grid, last round cut into key-tile slices) and
    the library's own choice, interleaved over --rounds rounds so clock drift hits all alike;
    median TFLOP/s of each, every launch timed by its own events after an L2 flush.  The schedules' outputs are checked against each other first.
    --kv64 times the 64-key-tile kernel instead of the default."""
    import torch
    from anima_attn import _lib as L

    torch.cuda.set_device(0)
    H = args.sched_heads  # heads per GPU (16 / N under the N-GPU head split)
    kf = L.FLAG_KV64 if args.kv64 else 0
    flags = {"unit": L.FLAG_UNIT, "whole": L.FLAG_WHOLE, "split": L.FLAG_SPLIT, "auto": 0}
    st = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    out_all = {}
    for shape in args.shapes.split(","):
        Sq, Skv = (int(x) for x in shape.split(":"))
        q = torch.randn(B * H, Sq, D, device="cuda", dtype=torch.bfloat16)
        k, v = (torch.randn(B * H, Skv, D, device="cuda", dtype=torch.bfloat16) for _ in range(2))
        out = torch.empty(B, Sq, H, D, device="cuda")
        ws = torch.zeros(max(1, int(L.lib.anima_attn_workspace_size(B, H, Sq, Skv, L.FLAG_SPLIT | kf))),
                         dtype=torch.uint8, device="cuda")

        def attn_args(f):
            a = L.AttnArgs()
            a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
            a.op_dtype, a.out, a.out_dtype = L.DTYPE_BF16, out.data_ptr(), L.DTYPE_F32
            a.out_stride[:] = [out.stride(0), out.stride(2), out.stride(1)]
            a.B, a.H, a.S_q, a.S_kv, a.D = B, H, Sq, Skv, D
            a.scale, a.flags = 1 / math.sqrt(D), flags[f] | kf
            a.kv_valid_len = None
            a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
            return a

        fl = attn_flops(B, H, Sq, Skv)
        n = max(5, min(200, int(2e12 / fl)))
        res = {f: [] for f in flags}
        ref = None
        for r in range(args.rounds):
            for f in flags:
                a = attn_args(f)
                for _ in range(2):
                    L.check(L.lib.anima_attn_fwd(ct.byref(a), st), "anima_attn_fwd")
                torch.cuda.synchronize()
                if r == 0:
                    if ref is None:
                        ref = out.clone()
                    elif (out - ref).abs().max().item() > 2e-2:
                        raise SystemExit(f"schedule {f} disagrees at {Sq}x{Skv}")
                evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                       for _ in range(n)]
                for e0, e1 in evs:
                    _flush_l2("cuda")  # cold L2 for every launch, outside its events
                    e0.record()
                    L.lib.anima_attn_fwd(ct.byref(a), st)
                    e1.record()
                torch.cuda.synchronize()
                ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / n
                res[f].append(fl / (ms * 1e-3) / 1e12)
        sched = {0: "unit", 1: "whole", 2: "cut"}.get(L.lib.anima_attn_schedule(B, H, Sq, Skv, kf, 0))
        out_all[shape] = {**{f: round(statistics.median(t), 1) for f, t in res.items()},
                          "auto_runs": sched}
    return {"workload": f"attention schedules, B=2 H={H} bf16 -> fp32, TFLOP/s (median of rounds)",
            "kernel": "64-key tiles" if args.kv64 else "128-key tiles", "shapes": out_all}


# ---------------------------------------------------------------- qkv projection
def run_qkv(args):
    """anima_qkv_projection (the projection GEMM with q/k RMSNorm, RoPE and the head-major
    16-bit store in its epilogue) against the path it replaces: a cuBLAS GEMM writing
    [B, L, n, H, 128] followed by the attention prologue; and the cuBLAS GEMM alone, the
    tensor-core anchor.  DiT shapes: B=2 (CFG pair), L=--L tokens, K=2048, fp16; --qkv-shapes
    lists H:n (heads per GPU, tensors: 3 = q/k/v of self-attention, 1 = the cross-attention
    query).  Median of --steps timed launches, each after a 256 MiB write that flushes L2."""
    import torch
    import anima_attn
    from anima_attn import ops

    torch.cuda.set_device(0)
    dev, dt, Bq, K = "cuda", torch.float16, 2, 2048
    L = args.L
    side = int(math.isqrt(L))
    if side * side != L:
        raise SystemExit("qkv: --L must be a square token grid")
    peak = load_peaks()["tflops"]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(args.seed)
    freqs = anima_attn.rope_freqs_3d(1, side, side, device=dev)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    out = {}
    for spec in args.qkv_shapes.split(","):
        Hh, n = (int(v) for v in spec.split(":"))
        x = torch.randn(Bq, L, K, device=dev, generator=g).to(dt)
        w = (0.02 * torch.randn(n * Hh * 128, K, device=dev, generator=g)).to(dt)
        qw = 1 + 0.1 * torch.randn(128, device=dev, generator=g)
        kw = 1 + 0.1 * torch.randn(128, device=dev, generator=g)
        rope = freqs if n == 3 else None

        def fused():
            return ops.qkv_projection(x, w, Hh, n, 0, qw, kw, rope, 1e-6, True, n == 3)

        def unfused():
            c = torch.mm(x.view(Bq * L, K), w.t()).view(Bq, L, n, Hh, 128)
            if n == 3:
                return ops.prologue(c[:, :, 0], c[:, :, 1], c[:, :, 2], qw, kw, rope, 1e-6,
                                    True, True, dt)
            return ops.prologue(c[:, :, 0], None, None, qw, None, None, 1e-6, True, False, dt)

        a, b = fused(), unfused()
        diff = max(float((u.float() - v.float()).abs().max()) for u, v in zip(a, b)
                   if u is not None)
        tf, tu = timed(fused), timed(unfused)
        tg = timed(lambda: torch.mm(x.view(Bq * L, K), w.t()))
        fl = 2.0 * Bq * L * K * n * Hh * 128
        tflops = lambda ms: round(fl / (ms * 1e-3) / 1e12, 1)
        out[spec] = {"fused_ms": round(tf, 4), "cublas_plus_prologue_ms": round(tu, 4),
                     "cublas_gemm_ms": round(tg, 4), "fused_tflops": tflops(tf),
                     "fused_frac_of_measured_peak": round(fl / (tf * 1e-3) / 1e12 / peak, 3),
                     "cublas_gemm_tflops": tflops(tg), "speedup_vs_unfused": round(tu / tf, 3),
                     "max_abs_diff_vs_unfused": round(diff, 4)}
    # The MLP's first layer + GELU (B*L x 8192 x 2048): anima_gemm_gelu against the cuBLAS
    # GEMM followed by the library's GELU pass.
    x = torch.randn(Bq * L, K, device=dev, generator=g).to(dt)
    w = (torch.randn(4 * K, K, device=dev, generator=g) / K ** 0.5).to(dt)
    fused = lambda: ops.gemm_gelu(x, w)
    unfused = lambda: ops.gelu_(torch.mm(x, w.t()))
    diff = float((fused().float() - unfused().float()).abs().max())
    tf, tu = timed(fused), timed(unfused)
    tg = timed(lambda: torch.mm(x, w.t()))
    fl = 2.0 * Bq * L * K * 4 * K
    out["mlp1_gelu"] = {"fused_ms": round(tf, 4), "cublas_plus_gelu_ms": round(tu, 4),
                        "cublas_gemm_ms": round(tg, 4),
                        "fused_tflops": round(fl / (tf * 1e-3) / 1e12, 1),
                        "fused_frac_of_measured_peak": round(fl / (tf * 1e-3) / 1e12 / peak, 3),
                        "speedup_vs_unfused": round(tu / tf, 3),
                        "max_abs_diff_vs_unfused": round(diff, 4)}
    if anima_attn.status() != 0:
        raise SystemExit("device-side timeout recorded")
    return {"workload": f"q/k/v projection + prologue, and MLP layer 1 + GELU, B={Bq} L={L} "
                        f"K={K} fp16 (DiT shapes)",
            "peak_bf16_tflops_measured": peak, "shapes": out}


# ---------------------------------------------------------------- main
def reference_line(args, world):
    r = cpu_reference(args.L, args.steps, args.warmup)
    one = cpu_reference(args.L, max(2, min(args.steps, 5)), 1, threads=1)
    pro = cpu_prologue(args.L, max(2, min(args.steps, 3)), 1)
    return {"metric": METRIC, "value": round(r["value"], 5), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": f"anima_rt CPU rmsnorm+rope+flash SDPA sample of B={B} H={H} "
                                   f"L={args.L} D={D}", "seq_len": args.L},
            "cpu_baseline": {"value": round(r["value"], 5), "unit": UNIT, "cores": r["cores"],
                             "kind": r["kind"], "sample": r["sample"], "cpu_model": r["cpu_model"],
                             "cores_1": {"value": round(one["value"], 6), "cores": 1},
                             "prologue": pro},
            "e2e": {"value": round(r["value"], 5), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--L", type=int, default=4096)
    ap.add_argument("--shard", choices=["heads", "replicas"], default="heads",
                    help="N GPUs: heads = the 16 heads split over the ranks (strong scaling); "
                         "replicas = the whole workload on every rank (weak scaling)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--workload", choices=["attn", "dit", "schedules", "qkv"], default="attn",
                    help="attn: the headline line with every section; dit: only the DiT step; "
                         "schedules: the attention kernel's schedules on --shapes; qkv: the "
                         "fused projection against cuBLAS + prologue on --qkv-shapes")
    ap.add_argument("--qkv-shapes", default="16:3,4:3,2:3,16:1",
                    help="qkv: H:n[,H:n...] (heads per GPU, tensors projected)")
    ap.add_argument("--shapes", default="4096:4096", help="schedules: SQ:SKV[,SQ:SKV...]")
    ap.add_argument("--rounds", type=int, default=3, help="schedules: interleaved rounds")
    ap.add_argument("--kv64", action="store_true", help="schedules: the 64-key-tile kernel")
    ap.add_argument("--sched-heads", type=int, default=16,
                    help="schedules: heads per GPU (16 / N under the N-GPU head split)")
    ap.add_argument("--blocks", type=int, default=28, help="DiT blocks")
    ap.add_argument("--latent", type=int, default=128, help="DiT latent side")
    ap.add_argument("--dit-steps", type=int, default=10, help="timed DiT steps")
    ap.add_argument("--sampler-steps", type=int, default=10,
                    help="DiT: steps of the timed sampling run (0: none)")
    ap.add_argument("--graph", type=int, choices=[0, 1], default=1,
                    help="DiT: replay the step as one captured CUDA graph (1) or issue it op by "
                         "op from Python (0)")
    ap.add_argument("--weights", default=None,
                    help="DiT: safetensors checkpoint of the model (default: seeded weights)")
    ap.add_argument("--schedule", choices=["auto", "unit", "whole", "split"], default="auto",
                    help="attention schedule for calls of more than one wave of 256-row units")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="headline only: skip the cross-attention, sweep, anchor and DiT sections")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(reference_line(args, world)))
        return

    if args.workload == "schedules":
        if rank == 0:
            print(json.dumps(run_schedules(args)))
        return
    if args.workload == "qkv":
        if rank == 0:
            print(json.dumps(run_qkv(args)))
        return
    if args.shard == "heads" and H % world:
        raise SystemExit("heads must divide over ranks")
    # CPU figures first, before any GPU work in this process (rank 0, one GPU only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "attn":
        cpu = cpu_baselines(args.L, args.steps, args.warmup)

    import torch
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "dit":
            d = run_dit_section(args, rank, world, local_rank, dist)
            res = {"metric": METRIC, "value": d["ms"], "unit": "ms", "n_gpus": world,
                   "steps": args.dit_steps, "warmup": args.warmup, "ms_per_step": d["ms"],
                   "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
                   "dtype": d["dtype"], "data": d["data"],
                   "config": {"workload": d["workload"], "global_batch": 2, "seq_len": 4096,
                              "parallelism": f"heads{world}"},
                   "e2e": {"value": d["heads"]["e2e_ms"], "unit": "ms",
                           "h2d_bytes_per_step": d["heads"]["e2e_bytes"]["h2d_per_step"],
                           "d2h_bytes_per_step": d["heads"]["e2e_bytes"]["d2h_per_step"]},
                   "gpu_launches": args.dit_steps * (args.blocks * 8 + 1),
                   "clocks": d["heads"]["clocks"], "dit_step": d}
        else:
            res = run_ours(args, rank, world, local_rank, dist)
            if not args.no_extras:
                res["cross_attention"] = run_cross(args, rank, world, local_rank, dist)
                res["sweep"] = run_sweep(args, rank, world, local_rank, dist)
                res["library_anchor"] = run_anchor(args, rank, world, local_rank, dist)
                res["dit_step"] = run_dit_section(args, rank, world, local_rank, dist)
            if cpu is not None:
                res["cpu_baseline"] = cpu
        if rank == 0:
            print(json.dumps(res))
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
