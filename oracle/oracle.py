"""CPU oracle for the Anima DiT attention hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this
module, and only as the checker (or as the timed CPU baseline).  The product path
(``anima_attn``) never imports it and has no CPU fallback.

Two CPU implementations are exposed through one interface:

* ``port``      -- ``oracle/liboracle.so``, our C restatement (anima_oracle.c) of
                   anima_rt's flash attention / RMSNorm / RoPE and of
                   VideoRopePosition3DEmb; always buildable with gcc.
* ``reference`` -- ``oracle/_ref/libanima_rt_ref.so``, the reference's own anima_rt
                   sources compiled by ``make -C oracle ref`` (present when the
                   reference tree was available at build time).

Compositions follow the reference callers:
  prologue   anima_rt/scripts/numpy_dit.py:285-291 (q/k RMSNorm via
             anima_rt_run_rmsnorm, RoPE for self-attention, transpose to [B,H,S,D])
  sdpa       scripts/phone_pipeline_nd.py:61-68 (NumpyRT.run_sdpa ->
             anima_rt_run_sdpa_flash with scale 1/sqrt(D), is_causal False)
"""
from __future__ import annotations

import ctypes as ct
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libanima_rt_ref.so")


def reference_tree():
    """The reference checkout: $ANIMA_REFERENCE_TREE, else a sibling checkout named
    ``reference`` next to this repository; None when neither holds anima_rt/."""
    cands = [os.environ.get("ANIMA_REFERENCE_TREE"),
             os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")]
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "anima_rt")):
            return c
    return None


REF_TREE = reference_tree()

_P = ct.c_void_p


def build(ref: bool = True) -> None:
    """Compile liboracle.so and, when the reference tree exists, the reference lib."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    if ref and REF_TREE is not None:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={REF_TREE}"], check=True)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class _Port:
    kind = "port"

    def __init__(self, path: str = PORT_SO):
        if not os.path.exists(path):
            build(ref=False)
        lib = ct.CDLL(path)
        lib.oracle_flash_attention.argtypes = [_P] * 4 + [ct.c_int] * 4 + [ct.c_float, ct.c_int]
        lib.oracle_flash_attention.restype = ct.c_int
        lib.oracle_flash_attention_varlen.argtypes = ([_P] * 4 + [ct.c_int] * 4 +
                                                      [ct.c_float, _P, ct.c_int, ct.c_int])
        lib.oracle_flash_attention_varlen.restype = ct.c_int
        lib.oracle_rmsnorm.argtypes = [_P, _P, _P, ct.c_int64, ct.c_int64, ct.c_float]
        lib.oracle_rmsnorm.restype = None
        lib.oracle_rope.argtypes = [_P, _P, _P, ct.c_int, ct.c_int, ct.c_int]
        lib.oracle_rope.restype = None
        lib.oracle_rope_freqs_3d.argtypes = [_P] + [ct.c_int] * 4 + [ct.c_double] * 4
        lib.oracle_rope_freqs_3d.restype = ct.c_int
        self.lib = lib

    def sdpa_flash(self, q, k, v, out, bh, sq, skv, d, scale, causal):
        rc = self.lib.oracle_flash_attention(q, k, v, out, bh, sq, skv, d, scale, int(causal))
        return rc == 0

    def rmsnorm(self, x, w, out, m, d, eps):
        self.lib.oracle_rmsnorm(x, w, out, m, d, eps)
        return True

    def rope(self, t, f, out, n, s, d):
        self.lib.oracle_rope(t, f, out, n, s, d)
        return True


class _Reference:
    """The reference's anima_rt C ABI (anima_rt/src/anima_rt.cpp:13-171) via ctypes,
    with the argtypes of anima_rt/scripts/anima_rt_ops.py:11-34."""
    kind = "reference"

    def __init__(self, path: str = REF_SO):
        lib = ct.CDLL(path)
        lib.anima_rt_init.restype = ct.c_bool
        lib.anima_rt_run_sdpa_flash.argtypes = [_P] * 4 + [ct.c_int] * 4 + [ct.c_float, ct.c_bool]
        lib.anima_rt_run_sdpa_flash.restype = ct.c_bool
        lib.anima_rt_run_rmsnorm.argtypes = [_P, _P, _P, ct.c_int, ct.c_int, ct.c_float]
        lib.anima_rt_run_rmsnorm.restype = ct.c_bool
        lib.anima_rt_run_rope.argtypes = [_P, _P, _P, ct.c_int, ct.c_int, ct.c_int]
        lib.anima_rt_run_rope.restype = ct.c_bool
        if not lib.anima_rt_init():
            raise RuntimeError("reference anima_rt_init failed")
        self.lib = lib

    def sdpa_flash(self, q, k, v, out, bh, sq, skv, d, scale, causal):
        return bool(self.lib.anima_rt_run_sdpa_flash(q, k, v, out, bh, sq, skv, d, scale,
                                                     bool(causal)))

    def rmsnorm(self, x, w, out, m, d, eps):
        return bool(self.lib.anima_rt_run_rmsnorm(x, w, out, m, d, eps))

    def rope(self, t, f, out, n, s, d):
        return bool(self.lib.anima_rt_run_rope(t, f, out, n, s, d))


_cache: dict = {}


def have_reference() -> bool:
    return os.path.exists(REF_SO)


def backend(kind: str = "port"):
    """``port`` (our C restatement) or ``reference`` (the compiled reference)."""
    if kind not in _cache:
        _cache[kind] = _Port() if kind == "port" else _Reference()
    return _cache[kind]


def _slices(n: int, parts: int):
    parts = max(1, min(parts, n))
    step = -(-n // parts)
    return [(i, min(n, i + step)) for i in range(0, n, step)]


def sdpa(q, k, v, scale=None, causal=False, threads=1, kind="port"):
    """Reference flash SDPA on [BH, S, D] (or [B, H, S, D]) fp32 arrays.

    Mirrors NumpyRT.run_sdpa (scripts/phone_pipeline_nd.py:61-68): contiguous fp32,
    scale 1/sqrt(D).  ``threads`` > 1 splits the BH heads into contiguous slices, one
    ctypes call per slice (ctypes releases the GIL); per-head work is independent so
    results are identical to one call.
    """
    shape = q.shape
    d = shape[-1]
    sq, skv = q.shape[-2], k.shape[-2]
    q3, k3, v3 = (_f32(t.reshape(-1, t.shape[-2], d)) for t in (q, k, v))
    bh = q3.shape[0]
    out = np.zeros((bh, sq, d), dtype=np.float32)
    scale = float(1.0 / np.sqrt(d)) if scale is None else float(scale)
    be = backend(kind)

    def run(sl):
        a, b = sl
        ok = be.sdpa_flash(q3[a:b].ctypes.data, k3[a:b].ctypes.data, v3[a:b].ctypes.data,
                           out[a:b].ctypes.data, b - a, sq, skv, d, scale, causal)
        if not ok:
            raise RuntimeError("oracle sdpa failed")

    sl = _slices(bh, threads)
    if len(sl) == 1:
        run(sl[0])
    else:
        with ThreadPoolExecutor(len(sl)) as ex:
            list(ex.map(run, sl))
    return out.reshape(*shape[:-2], sq, d)


def sdpa_varlen(q, k, v, valid, scale=None, threads=1):
    """Key-padding-masked SDPA on [B, H, S, D]: sample b attends to keys [0, valid[b])."""
    B, H, sq, d = q.shape
    skv = k.shape[2]
    q3, k3, v3 = (_f32(t) for t in (q, k, v))
    out = np.zeros((B, H, sq, d), dtype=np.float32)
    vl = np.ascontiguousarray(valid, dtype=np.int32)
    scale = float(1.0 / np.sqrt(d)) if scale is None else float(scale)
    lib = backend("port").lib

    def run(sl):
        rc = lib.oracle_flash_attention_varlen(q3.ctypes.data, k3.ctypes.data, v3.ctypes.data,
                                               out.ctypes.data, H, sq, skv, d, scale,
                                               vl.ctypes.data, sl[0], sl[1])
        if rc:
            raise RuntimeError("oracle varlen sdpa failed")

    sl = _slices(B * H, threads)
    with ThreadPoolExecutor(len(sl)) as ex:
        list(ex.map(run, sl))
    return out


def rmsnorm(x, w, eps=1e-6, kind="port"):
    """anima_rt_run_rmsnorm over the last axis (phone_pipeline_nd.py:53-58)."""
    xs = _f32(x)
    d = xs.shape[-1]
    m = xs.size // d
    out = np.zeros_like(xs)
    wp = None if w is None else _f32(w)
    backend(kind).rmsnorm(xs.ctypes.data, None if wp is None else wp.ctypes.data,
                          out.ctypes.data, m, d, float(eps))
    return out


def rope(t, freqs, kind="port"):
    """anima_rt_run_rope on t [N, S, D] or [B, S, H, D] (anima_rt_ops.py:127-143)."""
    t = _f32(t)
    if t.ndim == 4:
        B, S, H, D = t.shape
        flat = np.ascontiguousarray(t.transpose(0, 2, 1, 3)).reshape(B * H, S, D)
    else:
        flat = t
        B = None
    N, S, D = flat.shape
    f = _f32(freqs)
    out = np.zeros_like(flat)
    backend(kind).rope(flat.ctypes.data, f.ctypes.data, out.ctypes.data, N, S, D)
    if B is not None:
        return np.ascontiguousarray(out.reshape(B, H, S, D).transpose(0, 2, 1, 3))
    return out


def rope_freqs_3d(T, H, W, head_dim=128, h_ratio=4.0, w_ratio=4.0, t_ratio=1.0,
                  theta=10000.0):
    """VideoRopePosition3DEmb table [(T*H*W), head_dim/2, 2, 2] fp32."""
    out = np.zeros((T * H * W, head_dim // 2, 2, 2), dtype=np.float32)
    rc = backend("port").lib.oracle_rope_freqs_3d(out.ctypes.data, T, H, W, head_dim,
                                                  h_ratio, w_ratio, t_ratio, theta)
    if rc:
        raise ValueError("bad head_dim for 3D RoPE")
    return out


def prologue(q, k, v, q_w, k_w, freqs=None, eps=1e-6, kind="port"):
    """Per-head q/k RMSNorm then optional RoPE, returning [B, H, S, D] fp32.

    q [B, Sq, H, D], k/v [B, Skv, H, D] pre-norm projections; ``k_w`` None skips the
    k norm (config 3 normalises q only).  Follows numpy_dit.py:285-291.
    """
    qn = rmsnorm(q, q_w, eps, kind)
    kn = rmsnorm(k, k_w, eps, kind) if k_w is not None else _f32(k)
    if freqs is not None:
        qn = rope(qn, freqs, kind)
        kn = rope(kn, freqs, kind)
    tr = lambda t: np.ascontiguousarray(_f32(t).transpose(0, 2, 1, 3))
    return tr(qn), tr(kn), tr(v)


def numpy_rope(t, freqs):
    """The reference's live-path RoPE, numpy broadcasting on [B, S, H, D] fp32
    (anima_rt/scripts/numpy_dit.py:33-37, the numpy twin of predict2.apply_rotary_pos_emb):
    with freqs [S, D/2, 2, 2] = [[cos, -sin], [sin, cos]] per pair p and x = (t[p], t[p+D/2]),
    out[p] = cos x0 - sin x1, out[p+D/2] = sin x0 + cos x1, computed as the reference does
    (elementwise products of broadcast arrays, fp32), so its cost is the reference's cost.
    Used as the timed CPU baseline of the prologue and as a checker."""
    t = np.asarray(t, dtype=np.float32)
    B, S, H, D = t.shape
    half = D // 2
    f = np.asarray(freqs, dtype=np.float32).reshape(S, 1, half, 2, 2)
    x = np.moveaxis(t.reshape(B, S, H, 2, half), -2, -1)[..., None, :]  # [B,S,H,half,1,2]
    y = f[..., 0] * x[..., 0] + f[..., 1] * x[..., 1]                   # [B,S,H,half,2]
    return np.moveaxis(y, -1, -2).reshape(B, S, H, D)
