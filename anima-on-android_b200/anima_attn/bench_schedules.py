"""Times the attention kernel's three schedules on given shapes (needs a B200).

    python -m anima_attn.bench_schedules [--rounds R] [--kv64] SQ:SKV [SQ:SKV ...]

For each shape (B=2, H=16, bf16 operands, fp32 output) it runs the call with
ANIMA_FLAG_UNIT (one CTA per 256-row unit), ANIMA_FLAG_WHOLE (persistent grid, whole
units), ANIMA_FLAG_SPLIT (persistent grid, last round cut into key-tile slices) and no
override (the library's choice), interleaved over R rounds so that clock drift hits all
alike, and prints the median TFLOP/s of each.  The outputs of the schedules are checked
against each other first.  Use it to see which schedule a shape gets and what the others
would give.  --kv64 times the 64-key-tile kernel (ANIMA_FLAG_KV64) instead of the default.
"""
from __future__ import annotations

import argparse
import ctypes as ct
import math
import statistics

import torch

from . import _lib as L


def time_shape(Sq: int, Skv: int, rounds: int, B: int = 2, H: int = 16,
               kernel_flags: int = 0) -> dict:
    q = torch.randn(B * H, Sq, 128, device="cuda", dtype=torch.bfloat16)
    k, v = (torch.randn(B * H, Skv, 128, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    out = torch.empty(B, Sq, H, 128, device="cuda")
    ws = torch.zeros(max(1, int(L.lib.anima_attn_workspace_size(B, H, Sq, Skv,
                                                                L.FLAG_SPLIT | kernel_flags))),
                     dtype=torch.uint8, device="cuda")
    st = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    flags = {"unit": L.FLAG_UNIT, "whole": L.FLAG_WHOLE, "split": L.FLAG_SPLIT, "auto": 0}

    def args(f):
        a = L.AttnArgs()
        a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
        a.op_dtype = 1
        a.out, a.out_dtype = out.data_ptr(), 0
        a.out_stride[:] = [out.stride(0), out.stride(2), out.stride(1)]
        a.B, a.H, a.S_q, a.S_kv, a.D = B, H, Sq, Skv, 128
        a.scale = 1 / math.sqrt(128)
        a.flags = flags[f] | kernel_flags
        a.kv_valid_len = None
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        return a

    fl = 4 * B * H * Sq * Skv * 128
    n = max(5, int(2e12 / fl))
    res = {f: [] for f in flags}
    ref = None
    for r in range(rounds):
        for f in flags:
            a = args(f)
            for _ in range(2):
                L.check(L.lib.anima_attn_fwd(ct.byref(a), st), "anima_attn_fwd")
            torch.cuda.synchronize()
            if r == 0:
                if ref is None:
                    ref = out.clone()
                elif (out - ref).abs().max().item() > 2e-2:
                    raise RuntimeError(f"schedule {f} disagrees at {Sq}x{Skv}")
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(n):
                L.lib.anima_attn_fwd(ct.byref(a), st)
            e1.record()
            torch.cuda.synchronize()
            res[f].append(fl / (e0.elapsed_time(e1) / n * 1e-3) / 1e12)
    return {f: statistics.median(v_) for f, v_ in res.items()}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--rounds", type=int, default=3)
    ap.add_argument("--kv64", action="store_true", help="the 64-key-tile kernel")
    ap.add_argument("shapes", nargs="+", help="SQ:SKV")
    a = ap.parse_args(argv)
    torch.cuda.set_device(0)
    for s in a.shapes:
        Sq, Skv = (int(x) for x in s.split(":"))
        med = time_shape(Sq, Skv, a.rounds, kernel_flags=L.FLAG_KV64 if a.kv64 else 0)
        print(f"{Sq:6d}x{Skv:<6d} " + "  ".join(f"{f} {t:7.1f}" for f, t in med.items()), flush=True)


if __name__ == "__main__":
    main()
