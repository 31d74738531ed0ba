"""anima_attn_fwd_noalloc: the attention entry for callers that cannot allocate.

Some hosts cannot let a library allocate device memory: a host that owns the whole
device budget through its own allocator, or a C plugin handed only device pointers and
sizes.  For them the library keeps the split schedule's scratch in a static device
array, so this entry needs no workspace argument and calls no allocator.  This test
calls it through the C ABI, twice in a row (the second call reuses the array the first
one left behind), and checks each result against the regular entry anima_attn_fwd with
a caller workspace, within the attention tolerance used by every parity test.

This file sorts last on purpose, so a run that stops at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import ctypes as ct
import math
import os

import numpy as np
import pytest

from conftest import ATTN_MAX_ABS, ATTN_REL_L2, max_abs, rel_l2

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _args(L, q, k, v, out, B, H, Sq, Skv, workspace=None, flags=0):
    a = L.AttnArgs()
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    a.op_dtype = L.DTYPE_BF16
    a.out = out.data_ptr()
    a.out_dtype = L.DTYPE_F32
    a.out_stride[:] = [out.stride(0), out.stride(2), out.stride(1)]  # [B, S, H, D]
    a.B, a.H, a.S_q, a.S_kv, a.D = B, H, Sq, Skv, 128
    a.scale = 1.0 / math.sqrt(128)
    a.flags = flags
    a.kv_valid_len = None
    a.workspace = None if workspace is None else workspace.data_ptr()
    a.workspace_bytes = 0 if workspace is None else workspace.numel()
    return a


# With ANIMA_FLAG_SPLIT, (4096, 4096) and (1300, 700) run the cut schedule (they use the
# scratch); (512, 384) fits in one wave and runs one CTA per unit, using none.
@pytest.mark.parametrize("Sq,Skv,sched", [(4096, 4096, "cut"), (1300, 700, "cut"),
                                          (512, 384, "unit")])
def test_noalloc_entry_matches_workspace_entry_twice(Sq, Skv, sched):
    from anima_attn import _lib as L
    torch.cuda.set_device(0)
    B, H = 2, 16
    want = {"cut": L.SCHED_CUT, "unit": L.SCHED_UNIT}[sched]
    assert L.lib.anima_attn_schedule(B, H, Sq, Skv, L.FLAG_SPLIT, 0) == want
    g = torch.Generator(device="cuda").manual_seed(Sq + Skv)
    q = torch.randn(B * H, Sq, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B * H, Skv, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B * H, Skv, 128, device="cuda", generator=g).to(torch.bfloat16)
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)

    flags = L.FLAG_SPLIT
    need = int(L.lib.anima_attn_workspace_size(B, H, Sq, Skv, flags))
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    ref = torch.empty(B, Sq, H, 128, device="cuda")
    a = _args(L, q, k, v, ref, B, H, Sq, Skv, ws if need else None, flags)
    assert L.lib.anima_attn_fwd(ct.byref(a), stream) == L.OK, L.last_error()

    outs = []
    for _ in range(2):
        out = torch.full((B, Sq, H, 128), float("nan"), device="cuda")
        a = _args(L, q, k, v, out, B, H, Sq, Skv, flags=flags)
        assert L.lib.anima_attn_fwd_noalloc(ct.byref(a), stream) == L.OK, L.last_error()
        outs.append(out)
    torch.cuda.synchronize()
    assert L.lib.anima_attn_status(stream, 1) == 0
    r = ref.cpu().numpy()
    for out in outs:
        o = out.cpu().numpy()
        assert np.isfinite(o).all()
        assert rel_l2(o, r) <= ATTN_REL_L2 and max_abs(o, r) <= ATTN_MAX_ABS


# A fresh process that loads the library, sets up its device state through a
# device-pointer entry, and then measures the device's free memory around two calls of
# the no-allocation entry on the cut schedule.  CUDA_MODULE_LOADING=EAGER loads every
# kernel module of the library (and so reserves the static scratch) when the library's
# runtime first initialises, i.e. before the first measurement; from then on any device
# allocation by the entry -- its own cudaMalloc, or a local-memory reservation grown by a
# kernel launch -- would lower the free memory.  No torch in that process: its buffers
# come from the CUDA runtime directly, allocated before the first measurement.
_FRESH = r"""
import ctypes as ct, json, math, os, sys
import numpy as np
sys.path[:0] = [os.environ["PKG_ROOT"]]
from anima_attn import _lib as L
rt = ct.CDLL(os.environ["CUDART"])
rt.cudaMemGetInfo.argtypes = [ct.POINTER(ct.c_size_t)] * 2
rt.cudaMalloc.argtypes = [ct.POINTER(ct.c_void_p), ct.c_size_t]
rt.cudaMemcpy.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_size_t, ct.c_int]
rt.cudaMemset.argtypes = [ct.c_void_p, ct.c_int, ct.c_size_t]
assert rt.cudaSetDevice(0) == 0
B, H, S, D = 2, 16, 4096, 128
def dmalloc(n):
    p = ct.c_void_p()
    assert rt.cudaMalloc(ct.byref(p), n) == 0
    return p.value
rng = np.random.default_rng(5)
ops = []
for _ in range(3):
    a = rng.standard_normal((B * H, S, D), dtype=np.float32)
    bits = (a.view(np.uint32) >> 16).astype(np.uint16)  # bf16 by truncation
    p = dmalloc(bits.nbytes)
    assert rt.cudaMemcpy(p, bits.ctypes.data, bits.nbytes, 1) == 0
    ops.append(p)
nout = B * S * H * D * 4
outs = [dmalloc(nout) for _ in range(3)]
need = int(L.lib.anima_attn_workspace_size(B, H, S, S, L.FLAG_SPLIT))
ws = dmalloc(need)
assert rt.cudaMemset(ws, 0, need) == 0
def args(out, workspace):
    a = L.AttnArgs()
    a.q, a.k, a.v = ops
    a.op_dtype = L.DTYPE_BF16
    a.out, a.out_dtype = out, L.DTYPE_F32
    a.out_stride[:] = [S * H * D, D, H * D]
    a.B, a.H, a.S_q, a.S_kv, a.D = B, H, S, S, D
    a.scale, a.flags = 1 / math.sqrt(D), L.FLAG_SPLIT
    a.kv_valid_len = None
    a.workspace, a.workspace_bytes = workspace, (need if workspace else 0)
    return a
sm, cc = ct.c_int(), ct.c_int()
assert L.lib.anima_attn_device_info(ct.byref(sm), ct.byref(cc)) == 0
assert L.lib.anima_attn_schedule(B, H, S, S, L.FLAG_SPLIT, 0) == L.SCHED_CUT
def free():
    assert rt.cudaDeviceSynchronize() == 0
    f, t = ct.c_size_t(), ct.c_size_t()
    assert rt.cudaMemGetInfo(ct.byref(f), ct.byref(t)) == 0
    return f.value
f0 = free()
for out in outs[:2]:
    assert L.lib.anima_attn_fwd_noalloc(ct.byref(args(out, None)), None) == 0, L.last_error()
f1 = free()
assert L.lib.anima_attn_fwd(ct.byref(args(outs[2], ws)), None) == 0
assert L.lib.anima_attn_status(None, 1) == 0
res = []
for out in outs:
    h = np.empty(nout // 4, np.float32)
    assert rt.cudaMemcpy(h.ctypes.data, out, nout, 2) == 0
    res.append(h)
print(json.dumps({"free_before": f0, "free_after": f1,
                  "max_diff": [float(np.abs(r - res[2]).max()) for r in res[:2]],
                  "finite": bool(all(np.isfinite(r).all() for r in res))}))
"""


def _cudart():
    import glob
    cands = glob.glob("/usr/local/cuda/lib64/libcudart.so.12*")
    try:
        import nvidia.cuda_runtime as cr
        cands += glob.glob(os.path.join(os.path.dirname(cr.__file__), "lib", "libcudart.so.12*"))
    except ImportError:
        pass
    if not cands:
        pytest.skip("no libcudart.so.12 found")
    return sorted(cands)[0]


def test_noalloc_entry_allocates_nothing_in_a_fresh_process():
    import json
    import subprocess
    import sys
    from conftest import PKG_ROOT
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER", PKG_ROOT=PKG_ROOT, CUDART=_cudart(),
               CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "0"))
    r = subprocess.run([sys.executable, "-c", _FRESH], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["finite"]
    # Same kernel and schedule with the scratch elsewhere.  The cut schedule's merge takes
    # the slices in the order their CTAs finish, so results agree to fp32 rounding.
    assert max(res["max_diff"]) <= 1e-6, res
    assert res["free_after"] == res["free_before"], res
