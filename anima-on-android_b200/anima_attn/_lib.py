"""ctypes binding of libanima_attn.so (include/anima_rt.h, include/anima_attn.h).

The shared library is built in-tree by ``build.py`` next to this file.  There is no
fallback: if the library is missing or does not load, importing the package raises.
"""
from __future__ import annotations

import ctypes as ct
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# ANIMA_ATTN_LIB points at another build of the same library (e.g. a tuning variant).
LIB_PATH = os.environ.get("ANIMA_ATTN_LIB", os.path.join(HERE, "libanima_attn.so"))

# status codes and flags (anima_attn.h)
OK, ERR_ARG, ERR_SHAPE, ERR_CUDA, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_NOMEM = 0, -1, -2, -3, -4, -5, -6
DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
FLAG_QNORM, FLAG_KNORM, FLAG_ROPE, FLAG_MASK, FLAG_CAUSAL, FLAG_PAIR = 0x1, 0x2, 0x4, 0x8, 0x10, 0x20
FLAG_SPLIT, FLAG_UNIT, FLAG_WHOLE, FLAG_KV64 = 0x40, 0x80, 0x100, 0x200
SCHED_UNIT, SCHED_WHOLE, SCHED_CUT = 0, 1, 2
IPC_HANDLE_BYTES = 64  # ANIMA_IPC_HANDLE_BYTES

ERR_NAMES = {OK: "ok", ERR_ARG: "bad argument", ERR_SHAPE: "unsupported shape",
             ERR_CUDA: "CUDA error", ERR_TIMEOUT: "device-side wait timed out",
             ERR_UNSUPPORTED: "unsupported device", ERR_NOMEM: "out of device memory"}

_P = ct.c_void_p
_I64x3 = ct.c_int64 * 3


class PrologueArgs(ct.Structure):
    _fields_ = [("q", _P), ("k", _P), ("v", _P), ("in_dtype", ct.c_int),
                ("q_stride", _I64x3), ("k_stride", _I64x3), ("v_stride", _I64x3),
                ("B", ct.c_int), ("H", ct.c_int), ("S_q", ct.c_int), ("S_kv", ct.c_int),
                ("D", ct.c_int), ("q_norm_w", _P), ("k_norm_w", _P), ("eps", ct.c_float),
                ("rope_freqs", _P), ("flags", ct.c_uint), ("q_out", _P), ("k_out", _P),
                ("v_out", _P), ("op_dtype", ct.c_int)]


class AttnArgs(ct.Structure):
    _fields_ = [("q", _P), ("k", _P), ("v", _P), ("op_dtype", ct.c_int), ("out", _P),
                ("out_dtype", ct.c_int), ("out_stride", _I64x3), ("B", ct.c_int),
                ("H", ct.c_int), ("S_q", ct.c_int), ("S_kv", ct.c_int), ("D", ct.c_int),
                ("scale", ct.c_float), ("flags", ct.c_uint), ("kv_valid_len", _P),
                ("workspace", _P), ("workspace_bytes", ct.c_uint64)]


class QkvProjArgs(ct.Structure):
    _fields_ = [("x", _P), ("w", _P), ("dtype", ct.c_int), ("B", ct.c_int), ("L", ct.c_int),
                ("H", ct.c_int), ("K", ct.c_int), ("n_tensors", ct.c_int),
                ("first_tensor", ct.c_int), ("q_norm_w", _P), ("k_norm_w", _P),
                ("eps", ct.c_float), ("rope_freqs", _P), ("flags", ct.c_uint), ("q_out", _P),
                ("k_out", _P), ("v_out", _P)]


# Every symbol the headers declare, with its ctypes signature.
SIGNATURES = {
    # include/anima_rt.h -- argtypes as the reference binds them (anima_rt_ops.py:11-34)
    "anima_rt_init": ([], ct.c_bool),
    "anima_rt_destroy": ([], None),
    "anima_rt_run_sdpa_flash": ([_P] * 4 + [ct.c_int] * 4 + [ct.c_float, ct.c_bool], ct.c_bool),
    "anima_rt_run_sdpa": ([_P] * 4 + [ct.c_int] * 4 + [ct.c_float, ct.c_bool], ct.c_bool),
    "anima_rt_run_rmsnorm": ([_P, _P, _P, ct.c_int, ct.c_int, ct.c_float], ct.c_bool),
    "anima_rt_run_rope": ([_P, _P, _P, ct.c_int, ct.c_int, ct.c_int], ct.c_bool),
    "anima_rt_run_gelu": ([_P, _P, ct.c_int], ct.c_bool),
    "anima_rt_run_silu": ([_P, _P, ct.c_int], ct.c_bool),
    "anima_rt_run_layernorm": ([_P, _P, ct.c_int, ct.c_int, ct.c_float], ct.c_bool),
    "anima_rt_run_softmax": ([_P, _P, ct.c_int, ct.c_int], ct.c_bool),
    "anima_rt_run_gemm_fp32": ([_P, _P, _P, ct.c_int, ct.c_int, ct.c_int], ct.c_bool),
    "anima_rt_run_gemm_bf16": ([_P, _P, _P, ct.c_int, ct.c_int, ct.c_int], ct.c_bool),
    "anima_rt_run_attention": ([_P] * 8 + [ct.c_int] * 5 + [ct.c_float, ct.c_float, ct.c_uint],
                               ct.c_bool),
    "anima_rt_last_error": ([], ct.c_char_p),
    # include/anima_attn.h
    "anima_attn_prologue": ([ct.POINTER(PrologueArgs), _P], ct.c_int),
    "anima_attn_fwd": ([ct.POINTER(AttnArgs), _P], ct.c_int),
    "anima_attn_fwd_noalloc": ([ct.POINTER(AttnArgs), _P], ct.c_int),
    "anima_attn_fwd_gather": ([ct.POINTER(AttnArgs), ct.POINTER(_P), ct.c_int, _P], ct.c_int),
    "anima_gemm_gelu": ([_P, _P, _P] + [ct.c_int] * 4 + [_P], ct.c_int),
    "anima_qkv_projection_scatter": ([ct.POINTER(QkvProjArgs), ct.c_int, ct.c_int, ct.POINTER(_P),
                                      ct.c_int, _P], ct.c_int),
    "anima_attn_fwd_scatter_rows": ([ct.POINTER(AttnArgs), ct.POINTER(_P), ct.c_int, ct.c_int,
                                     ct.c_int64, ct.c_int, _P], ct.c_int),
    "anima_ipc_export": ([_P, _P, ct.POINTER(ct.c_uint64)], ct.c_int),
    "anima_ipc_open": ([_P, ct.c_uint64, ct.POINTER(_P)], ct.c_int),
    "anima_ipc_close": ([_P, ct.c_uint64], ct.c_int),
    "anima_attn_workspace_size": ([ct.c_int] * 4 + [ct.c_uint], ct.c_uint64),
    "anima_attn_schedule": ([ct.c_int] * 4 + [ct.c_uint, ct.c_int], ct.c_int),
    "anima_attn_status": ([_P, ct.c_int], ct.c_int),
    "anima_attn_selftest_timeout": ([ct.c_uint, _P], ct.c_int),
    "anima_qkv_projection": ([ct.POINTER(QkvProjArgs), _P], ct.c_int),
    "anima_attn_rope": ([_P, ct.POINTER(ct.c_int64), _P, _P, ct.POINTER(ct.c_int64), ct.c_int,
                         ct.c_int, ct.c_int, ct.c_int, _P], ct.c_int),
    "anima_dit_ln_modulate": ([_P, _P, _P, ct.c_int64, _P, ct.c_int, ct.c_int64, ct.c_int, ct.c_int,
                               ct.c_float, _P], ct.c_int),
    "anima_dit_gate_residual": ([_P, _P, ct.c_int64, _P, ct.c_int64, ct.c_int, ct.c_int, _P], ct.c_int),
    "anima_dit_gate_residual_ln_modulate": ([_P, _P, ct.c_int64, _P, ct.c_int, _P, _P, ct.c_int64, _P,
                                             ct.c_int, ct.c_int64, ct.c_int, ct.c_int, ct.c_float, _P],
                                            ct.c_int),
    "anima_dit_gelu": ([_P, _P, ct.c_int, ct.c_int64, _P], ct.c_int),
    "anima_attn_device_info": ([ct.POINTER(ct.c_int), ct.POINTER(ct.c_int)], ct.c_int),
    "anima_attn_version": ([], ct.c_char_p),
}


def load(path: str = LIB_PATH) -> ct.CDLL:
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build the CUDA library first "
            "(python -c 'import __graft_entry__ as g; g.build()' from the repository root)")
    lib = ct.CDLL(path)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


lib = load()


class AnimaError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != OK:
        raise AnimaError(f"{what} failed: {ERR_NAMES.get(rc, rc)}")


def last_error() -> str:
    s = lib.anima_rt_last_error()
    return s.decode() if s else ""
