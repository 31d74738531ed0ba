"""Host entries with ordinary (pageable) numpy arrays: the page-locked staging ring.

The reference's callers hand the anima_rt entries pageable numpy arrays.  Above 1 MiB
the library copies those through its own page-locked ring (host threads gather rows into
a slot while the copy engine moves the previous ones; device->host pieces are scattered
back), instead of the driver's single-threaded bounce buffer.  The kernels are the same
either way, so a staged output must equal the driver-copied one (ANIMA_RT_STAGE=0) and a
repeated call to fp32 rounding (bit for bit, except that a call on the cut schedule merges
its key slices in the order their CTAs finish, which moves the last bit between any two
calls).  With page-locked arrays the last chunk is split into fewer heads, whose schedule
may differ, so that result is compared at the attention parity bar.  A row copied to the
wrong place would differ by O(1).  The ragged case is also checked against the oracle.
"""
import ctypes as ct
import os

import numpy as np
import pytest

from conftest import ATTN_MAX_ABS, ATTN_REL_L2, max_abs, rel_l2

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def O():
    from oracle import oracle
    from anima_attn import _lib as L
    torch.cuda.set_device(0)
    assert L.lib.anima_rt_init()
    oracle.build(ref=False)
    return oracle


def _pinned(a):
    t = torch.empty(a.shape, dtype=torch.float32, pin_memory=True)
    p = t.numpy()
    p[...] = a
    return t, p


class _stage_off:
    def __enter__(self):
        self.old = os.environ.get("ANIMA_RT_STAGE")
        os.environ["ANIMA_RT_STAGE"] = "0"

    def __exit__(self, *exc):
        if self.old is None:
            os.environ.pop("ANIMA_RT_STAGE", None)
        else:
            os.environ["ANIMA_RT_STAGE"] = self.old


def _attention(L, q, k, v, qw, kw, freqs, valid, B, Sq, Skv, H, flags):
    out = np.full((B, Sq, H, 128), np.nan, dtype=np.float32)
    ptr = lambda a: None if a is None else a.ctypes.data
    ok = L.lib.anima_rt_run_attention(ptr(q), ptr(k), ptr(v), ptr(qw), ptr(kw), ptr(freqs),
                                      ptr(valid), out.ctypes.data, B, Sq, Skv, H, 128,
                                      ct.c_float(1e-6), ct.c_float(128 ** -0.5), ct.c_uint(flags))
    assert ok, L.last_error()
    return out


@pytest.mark.parametrize("B,H,Sq,Skv,masked,rope", [
    (2, 16, 4096, 4096, False, True),   # the bench shape: 64 MiB arrays, pitch 2x the chunk row
    (3, 6, 1000, 700, True, False),     # ragged rows per piece, short last chunk, key padding
    (1, 1, 3000, 2000, False, False),   # one head: contiguous rows, pieces of whole slots
])
def test_staged_attention_is_bit_identical_to_page_locked(O, B, H, Sq, Skv, masked, rope):
    from anima_attn import _lib as L
    rng = np.random.default_rng(B * 7 + H + Sq)
    q = rng.standard_normal((B, Sq, H, 128), dtype=np.float32)
    k = rng.standard_normal((B, Skv, H, 128), dtype=np.float32)
    v = rng.standard_normal((B, Skv, H, 128), dtype=np.float32)
    qw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    freqs = O.rope_freqs_3d(1, 64, 64) if rope else None
    valid = rng.integers(1, Skv + 1, size=B).astype(np.int32) if masked else None
    flags = L.FLAG_QNORM | L.FLAG_KNORM | (L.FLAG_ROPE if rope else 0)

    staged = _attention(L, q, k, v, qw, kw, freqs, valid, B, Sq, Skv, H, flags)
    again = _attention(L, q, k, v, qw, kw, freqs, valid, B, Sq, Skv, H, flags)  # ring reused
    with _stage_off():
        driver = _attention(L, q, k, v, qw, kw, freqs, valid, B, Sq, Skv, H, flags)
    keep = [_pinned(a) for a in (q, k, v)]
    tout, pout = _pinned(np.full((B, Sq, H, 128), np.nan, np.float32))
    ptr = lambda a: None if a is None else a.ctypes.data
    ok = L.lib.anima_rt_run_attention(keep[0][1].ctypes.data, keep[1][1].ctypes.data,
                                      keep[2][1].ctypes.data, qw.ctypes.data, kw.ctypes.data,
                                      ptr(freqs), ptr(valid), pout.ctypes.data, B, Sq, Skv, H,
                                      128, ct.c_float(1e-6), ct.c_float(128 ** -0.5),
                                      ct.c_uint(flags))
    assert ok, L.last_error()
    assert np.isfinite(staged).all() and np.isfinite(pout).all()
    for other in (again, driver):  # same chunks and schedules: fp32 rounding at most
        assert max_abs(staged, other) <= 1e-6
    # With a page-locked output the library splits the last chunk into fewer heads, which
    # may run another schedule (the one-wave cut rounds P to 16 bits against each slice's
    # own running max): two bf16 roundings of the same heads, which differ by up to the
    # size of the bf16 error itself, so the bar is the attention parity bar -- far below
    # a misplaced row's O(1).
    assert rel_l2(staged, pout) <= ATTN_REL_L2 and max_abs(staged, pout) <= ATTN_MAX_ABS
    if not rope:  # small enough for the oracle
        rq, rk, rv = O.prologue(q, k, v, qw, kw)
        n = min(8, os.cpu_count() or 1)
        ref = (O.sdpa_varlen(rq, rk, rv, valid, threads=n) if masked
               else O.sdpa(rq, rk, rv, threads=n))
        got = staged.transpose(0, 2, 1, 3)
        assert rel_l2(got, ref) <= ATTN_REL_L2 and max_abs(got, ref) <= ATTN_MAX_ABS


def test_staged_single_kernel_entry_with_tail(O):
    """anima_rt_run_rmsnorm on a 5 MB pageable array that is no multiple of the 256 KiB
    staging row: staged body plus a direct tail, both directions."""
    from anima_attn import _lib as L
    rng = np.random.default_rng(11)
    M, d = 10007, 128
    x = rng.standard_normal((M, d), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)

    def run(xa):
        out = np.full((M, d), np.nan, np.float32)
        assert L.lib.anima_rt_run_rmsnorm(xa.ctypes.data, w.ctypes.data, out.ctypes.data, M, d,
                                          ct.c_float(1e-6)), L.last_error()
        return out

    staged = run(x)
    with _stage_off():
        driver = run(x)
    tx, px = _pinned(x)
    pinned = run(px)
    ref = x / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + 1e-6) * w
    assert np.array_equal(staged, driver) and np.array_equal(staged, pinned)
    assert max_abs(staged, ref) <= 1e-5
