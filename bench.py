"""Benchmark of the Anima DiT attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--L 4096] [--shard replicas|heads]

One step = one fused attention call of one DiT block over one synthetic batch:
per-head q/k RMSNorm + 3D RoPE + bf16 cast (prologue kernel) and the tcgen05 flash
attention (attention kernel), B=2 (CFG pair) x 16 heads x L tokens x D=128, inputs
resident in HBM.  The default L=4096 is the 4096-token point of the sequence-length sweep
(1024x1024 image); other configs are parity tests, not bench lines.

metric  : attention TFLOP/s (4*B*H*L^2*D per step / step time), whole job.
e2e     : the same metric through the reference-facing C ABI (anima_rt_run_attention)
          with page-locked HOST buffers, host->device and device->host copies inside
          the timed region (wall clock; the call is synchronous).
roofline: the attention kernel's achieved TFLOP/s (CUDA events around its launches)
          over the measured dense bf16 peak in MEASURED_PEAKS.json.
cpu_baseline: the reference's anima_rt CPU path (oracle/_ref, compiled from the
          reference sources; our C restatement if that is absent) on the host cores,
          on a bounded sample of the same workload.

Multi-GPU (torchrun): "replicas" (default) runs the whole workload on every rank
(independent CFG batches, weak scaling, no collective on the data path); "heads"
splits the 16 heads across ranks (strong scaling).  Timing is the max over ranks.
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


# ---------------------------------------------------------------- reference arm
def cpu_reference(L, steps, warmup, seed=0, emit=True):
    """anima_rt's CPU path on the host cores, bounded sample per step: every thread runs
    the reference sequence (rmsnorm q,k -> rope q,k -> flash SDPA) for one (b, h) head
    over a block of query rows against all L keys.  Query rows and heads are
    independent, so TFLOP/s over the sample equals TFLOP/s of the whole workload."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    from oracle import oracle as O

    kind = "reference" if O.have_reference() else "port"
    be = O.backend(kind)
    if kind == "reference":
        be.lib.anima_rt_init()
    cores = len(os.sched_getaffinity(0))
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
    step_s = sum(times) / len(times)
    flops = attn_flops(1, cores, rows, L)
    value = flops / step_s / 1e12
    sample = (f"{cores} threads x one (b,h) head each: {rows} query rows x {L} keys "
              f"(rmsnorm+rope+flash SDPA), {attn_flops(1, 1, rows, L) / 1e9:.2f} GFLOP per thread; "
              f"per-row work identical, so TFLOP/s is that of the full B=2 H=16 L={L} step")
    return {"value": value, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample,
            "ms_per_step": step_s * 1e3, "cpu_model": _cpu_model()}


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


# ---------------------------------------------------------------- DiT step (config 4)
def dit_flops(blocks=28, L=4096, B=2, ctx=512, hidden=2048, mlp=8192, ctx_dim=1024):
    """Matmul FLOP of one CFG-batched forward (GEMMs + attention), as counted for the
    config: per block self q/k/v/o, cross q/o, cross k/v, MLP, and both attentions."""
    g = lambda m, n, k: 2.0 * m * n * k
    per = (4 * g(B * L, hidden, hidden) + 2 * g(B * L, hidden, hidden) +
           2 * g(B * ctx, hidden, ctx_dim) + g(B * L, mlp, hidden) + g(B * L, hidden, mlp) +
           attn_flops(B, 16, L, L) + attn_flops(B, 16, L, ctx))
    return blocks * per


def run_dit(args, rank, world, local_rank):
    """One Euler+CFG step of the Anima DiT (the full-step configuration): latent 16x128x128 (4096
    tokens), 28 blocks, hidden 2048, 16 heads, CFG pair batched (B=2), sigma 0.5 -> 0,
    cfg 5; heads split over the ranks, one NCCL all-gather per attention."""
    import torch
    from anima_attn.dit import AnimaDiT, DiTConfig, make_weights

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = DiTConfig(blocks=args.blocks)
    group = None
    if world > 1:
        import torch.distributed as dist
        group = dist.group.WORLD
    if args.weights:
        from anima_attn.checkpoint import load_dit_weights
        weights = load_dit_weights(args.weights, cfg, device=dev)
    else:
        weights = make_weights(cfg, seed=1234, device=dev, rng_device=dev)
    model = AnimaDiT(cfg, weights, rank=rank, world=world, group=group, shard=args.dit_shard)
    del weights
    side = args.latent
    g = torch.Generator(device=dev).manual_seed(4321)
    x = torch.randn(1, 16, side, side, device=dev, generator=g)
    cc = torch.randn(1, 512, 1024, device=dev, generator=g)
    cu = torch.randn(1, 512, 1024, device=dev, generator=g)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    with torch.no_grad():
        if args.graph:
            from anima_attn.dit import StepGraph
            graph = StepGraph(model, x, 0.5, 0.0, cc, cu, 5.0)
            run_step = lambda xx=None, c1=None, c2=None: graph(xx, c1, c2)
        else:
            graph = None
            run_step = lambda xx=None, c1=None, c2=None: model.euler_cfg_step(
                x if xx is None else xx, 0.5, 0.0, cc if c1 is None else c1, cu if c2 is None else c2, 5.0)
        clocks = ClockSampler(local_rank)
        with clocks:
            for _ in range(args.warmup):
                run_step()
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t_begin = time.perf_counter()
            e0.record(stream)
            for _ in range(args.steps):
                run_step()
            e1.record(stream)
            torch.cuda.synchronize()
            t_end = time.perf_counter()
            barrier()
        ms = e0.elapsed_time(e1) / args.steps
        # end to end: host latent + contexts in, host latent out, every step
        hx, hcc, hcu = (t.cpu().pin_memory() for t in (x, cc, cu))
        hout = torch.empty_like(hx).pin_memory()

        def host_step():
            dx, dcc, dcu = (t.to(dev, non_blocking=True) for t in (hx, hcc, hcu))
            hout.copy_(run_step(dx, dcc, dcu), non_blocking=True)
            torch.cuda.synchronize()

        host_step()
        barrier()
        t0 = time.perf_counter()
        n_e2e = max(2, min(args.steps, 5))
        for _ in range(n_e2e):
            host_step()
        e2e_ms = (time.perf_counter() - t0) / n_e2e * 1e3
        del graph, run_step  # a graph holding NCCL calls goes before the process group
    t = torch.tensor([ms, e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = t.tolist()
    L = (side // 2) ** 2
    fl = dit_flops(args.blocks, L)
    return {
        "metric": METRIC, "value": round(ms, 3), "unit": "ms", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp16 GEMM/attention operands, fp32 activations",
        "data": ("synthetic (seeded latent and context, N(0,0.02) bf16-valued weights)"
                 if not args.weights else
                 f"synthetic latent and context; weights from {os.path.basename(args.weights)}"),
        "config": {"workload": f"Anima DiT Euler+CFG step, {args.blocks} blocks, latent "
                               f"16x{side}x{side} ({L} tokens), context 512x1024, CFG pair",
                   "global_batch": 2, "seq_len": L,
                   "parallelism": (f"heads{world}" if world == 1 or args.dit_shard == "heads"
                                   else f"heads{world} (attention) + tokens{world} (rest), all-to-all"),
                   "heads_per_gpu": 16 // world, "tflops_per_gpu": round(fl / world / (ms * 1e-3) / 1e12, 1),
                   "l2": "weights (4 GB fp16) exceed L2 every step",
                   "cuda_graph": bool(args.graph),
                   "model_tflop_per_step": round(fl / 1e12, 2)},
        "e2e": {"value": round(e2e_ms, 3), "unit": "ms", "h2d_bytes_per_step": (hx.numel() + hcc.numel() + hcu.numel()) * 4,
                "d2h_bytes_per_step": hout.numel() * 4},
        # library kernels per step: per block 2 prologues, 2 attentions, 3 LayerNorm passes
        # (fused with the preceding residual update except the step's first), 1 GELU; plus
        # the final layer's fused pass
        "gpu_launches": args.steps * (args.blocks * 8 + 1),
        "clocks": clocks.summary(t_begin, t_end),
    }


# ---------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import anima_attn
    from anima_attn import _lib as L

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    L_ = args.L
    heads = H if args.shard == "replicas" else H // world
    if args.shard == "heads" and H % world:
        raise SystemExit("heads must divide over ranks")
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
        anima_attn.attention_core(qh, kh, vh, B, heads, out=out,
                                  schedule=args.schedule)
        if evs is not None:
            evs[2].record(stream)

    dist = None
    if world > 1:
        import torch.distributed as dist

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    clocks = ClockSampler(local_rank)
    with clocks:
        for _ in range(args.warmup):
            step()
        barrier()
        t_begin = time.perf_counter()
        for i in range(args.steps):
            step(evs[i])
        torch.cuda.synchronize()
        t_end = time.perf_counter()
        barrier()
    if anima_attn.status() != 0:
        raise SystemExit("device status word reports a kernel timeout")
    total_ms = evs[0][0].elapsed_time(evs[-1][2])
    pro_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    att_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    t = torch.tensor([total_ms, pro_ms, att_ms], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, pro_ms, att_ms = t.tolist()
    ms_step = total_ms / args.steps
    flops_rank = attn_flops(B, heads, L_, L_)
    value = flops_rank * world / (ms_step * 1e-3) / 1e12

    # ---- e2e through the host C ABI, pinned buffers, copies inside the region
    e2e = None
    if not args.no_e2e:
        pq, pk, pv = (torch.from_numpy(a).pin_memory() for a in (q, k, v))
        pqw, pkw = torch.from_numpy(qw).pin_memory(), torch.from_numpy(kw).pin_memory()
        pf = freqs.cpu().pin_memory()
        pout = torch.empty((B, L_, heads, D), dtype=torch.float32).pin_memory()
        assert L.lib.anima_rt_init()
        flags = L.FLAG_QNORM | L.FLAG_KNORM | L.FLAG_ROPE

        def host_step():
            ok = L.lib.anima_rt_run_attention(pq.data_ptr(), pk.data_ptr(), pv.data_ptr(),
                                              pqw.data_ptr(), pkw.data_ptr(), pf.data_ptr(), None,
                                              pout.data_ptr(), B, L_, L_, heads, D,
                                              ct.c_float(1e-6), ct.c_float(1 / math.sqrt(D)),
                                              flags)
            if not ok:
                raise SystemExit("anima_rt_run_attention failed: " + L.last_error())

        for _ in range(max(1, min(args.warmup, 3))):
            host_step()
        e2e_steps = max(3, min(args.steps, 20))
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            host_step()
        el = time.perf_counter() - t0
        te = torch.tensor([el], device=dev, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        el = te.item()
        h2d = 3 * pq.numel() * 4 + pf.numel() * 4 + 2 * D * 4
        e2e = {"value": flops_rank * world * e2e_steps / el / 1e12, "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": pout.numel() * 4,
               "ms_per_step": el / e2e_steps * 1e3, "steps": e2e_steps,
               "path": "anima_rt_run_attention (C ABI, page-locked host buffers, wall clock)"}

    peaks = load_peaks()
    achieved = flops_rank / (att_ms * 1e-3) / 1e12
    # The schedule that ran (the library's planner, given the workspace attention_core passes).
    sched_flags = {"auto": 0, "unit": L.FLAG_UNIT, "whole": L.FLAG_WHOLE, "split": L.FLAG_SPLIT}
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    sched_run = {0: "unit", 1: "whole", 2: "cut"}.get(
        L.lib.anima_attn_schedule(B, heads, L_, L_, sched_flags[args.schedule], sms), "error")
    traffic = load_traffic(L_).get("attn_fwd")
    pro_bytes = (3 * B * L_ * heads * D * 4) + (3 * B * L_ * heads * D * 2)
    res = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak" if args.shard == "replicas" else "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) q/k/v, N(1,0.1) norm weights)",
        "config": {"workload": f"fused q/k RMSNorm + 3D RoPE + flash attention (prologue + tcgen05 "
                               f"attention), B={B} H={heads} L={L_} D={D}, BASELINE config 5 @ L={L_}",
                   "global_batch": B * (world if args.shard == "replicas" else 1), "seq_len": L_,
                   "heads_per_gpu": heads,
                   "parallelism": f"{args.shard}{world}",
                   "l2": f"inputs {3 * B * L_ * heads * D * 4 / 2**20:.0f} MiB fp32 > 126 MB L2",
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
        "gpu_launches": 2 * args.steps,
        "clocks": clocks.summary(t_begin, t_end),
    }
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--L", type=int, default=4096)
    ap.add_argument("--shard", choices=["replicas", "heads"], default="replicas")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--workload", choices=["attn", "dit"], default="attn",
                    help="attn: fused attention op (headline); dit: one full DiT step (config 4)")
    ap.add_argument("--blocks", type=int, default=28, help="DiT blocks (dit workload)")
    ap.add_argument("--latent", type=int, default=128, help="latent side (dit workload)")
    ap.add_argument("--graph", type=int, choices=[0, 1], default=1,
                    help="dit workload: replay the step as one captured CUDA graph (1) or issue "
                         "it op by op from Python (0)")
    ap.add_argument("--weights", default=None,
                    help="dit workload: safetensors checkpoint of the model (default: seeded weights)")
    ap.add_argument("--dit-shard", choices=["tokens", "heads"], default="tokens",
                    help="dit workload on N GPUs: heads = all-gather of head outputs before a "
                         "replicated o-proj; tokens = rows split over ranks, all-to-all around "
                         "the head-parallel attention")
    ap.add_argument("--schedule", choices=["auto", "unit", "whole", "split"], default="auto",
                    help="attention schedule for calls of more than one wave of 256-row units: "
                         "auto: the library's choice; unit: one CTA per unit; whole: persistent "
                         "grid of whole units; split: persistent grid, last round cut into "
                         "key-tile slices")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        r = cpu_reference(args.L, args.steps, args.warmup)
        line = {"metric": METRIC, "value": round(r["value"], 5), "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 2),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "impl": "reference",
                "config": {"workload": f"anima_rt CPU rmsnorm+rope+flash SDPA sample of B={B} H={H} "
                                       f"L={args.L} D={D}", "seq_len": args.L},
                "cpu_baseline": {"value": round(r["value"], 5), "unit": UNIT, "cores": r["cores"],
                                 "kind": r["kind"], "sample": r["sample"], "cpu_model": r["cpu_model"]},
                "e2e": {"value": round(r["value"], 5), "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    if args.workload == "dit":
        res = run_dit(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(res))
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return
    res = run_ours(args, rank, world, local_rank)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_reference(args.L, steps=2, warmup=1)
            res["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
            res["cpu_baseline"]["value"] = round(cb["value"], 5)
        print(json.dumps(res))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
