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


# With ANIMA_FLAG_SPLIT, (4096, 4096) and (1300, 700) run the split schedule (they use the
# scratch); (512, 384) fits in one wave and uses none.
@pytest.mark.parametrize("Sq,Skv", [(4096, 4096), (1300, 700), (512, 384)])
def test_noalloc_entry_matches_workspace_entry_twice(Sq, Skv):
    from anima_attn import _lib as L
    torch.cuda.set_device(0)
    B, H = 2, 16
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
