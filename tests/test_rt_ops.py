"""The reference runtime's whole host ABI, as its own Python binding uses it.

anima_rt/scripts/anima_rt_ops.py:10-34 loads libanima_rt with ctypes and sets argtypes on
eleven anima_rt_* symbols before anything else; a library missing any of them fails that
module at import.  The CPU test here runs that file unmodified except for its hard-coded
library path (line 10) against libanima_attn.so and checks every argtypes line bound to
a symbol with the signature this library declares.  The GPU tests run the six entries
beyond the attention path (GELU, SiLU, LayerNorm, softmax and the two GEMMs) through
those signatures and compare them with PyTorch fp32/fp64 CPU results and, where it was
built, with the compiled reference library itself.
"""
import ctypes as ct
import os
import re

import numpy as np
import pytest

from conftest import has_gpu, max_abs, rel_l2

from anima_attn import _lib as L
from oracle import oracle as O

BOUND_BY_REFERENCE = ["anima_rt_init", "anima_rt_run_gelu", "anima_rt_run_silu",
                      "anima_rt_run_layernorm", "anima_rt_run_rmsnorm", "anima_rt_run_softmax",
                      "anima_rt_run_gemm_fp32", "anima_rt_run_gemm_bf16", "anima_rt_run_sdpa",
                      "anima_rt_run_sdpa_flash", "anima_rt_run_rope"]


def test_reference_binding_loads_this_library():
    tree = O.reference_tree()
    if tree is None:
        pytest.skip("reference checkout not available (set ANIMA_REFERENCE_TREE)")
    path = os.path.join(tree, "anima_rt", "scripts", "anima_rt_ops.py")
    src = open(path).read()
    lines = src.splitlines(True)
    assert "CDLL(" in lines[9], "line 10 of anima_rt_ops.py is its library path"
    lines[9] = f"_lib = _ct.CDLL({L.LIB_PATH!r})\n"
    ns = {"__name__": "anima_rt_ops_under_test"}
    try:
        exec(compile("".join(lines), path, "exec"), ns)
    except AssertionError:
        # `assert _lib.anima_rt_init()` follows the argtypes lines; without a CUDA device
        # init returns false, which is this library's documented behaviour.
        assert not has_gpu()
    lib = ns["_lib"]
    bound = sorted(set(re.findall(r"_lib\.(anima_rt_\w+)\.(?:argtypes|restype)", src)))
    assert bound == sorted(BOUND_BY_REFERENCE), bound
    for name in bound:
        fn = getattr(lib, name)
        args, res = L.SIGNATURES[name]
        if re.search(rf"_lib\.{name}\.argtypes", src):
            assert tuple(fn.argtypes) == tuple(args), name
        assert fn.restype == res, name


def test_compat_entries_fail_before_init_and_on_bad_arguments():
    """As in the reference, activation/norm/softmax entries need anima_rt_init; argument
    errors return false with a message instead of aborting.  (No GPU work is done.)"""
    x = np.zeros(8, np.float32)
    if not has_gpu():
        for name in ("anima_rt_run_gelu", "anima_rt_run_silu"):
            assert getattr(L.lib, name)(x.ctypes.data, x.ctypes.data, 8) is False
            assert "anima_rt_init" in L.last_error()
        assert L.lib.anima_rt_run_layernorm(x.ctypes.data, x.ctypes.data, 2, 4, ct.c_float(1e-6)) is False
        assert L.lib.anima_rt_run_softmax(x.ctypes.data, x.ctypes.data, 2, 4) is False
    assert L.lib.anima_rt_run_gemm_fp32(None, x.ctypes.data, x.ctypes.data, 2, 2, 2) is False
    assert "bad arguments" in L.last_error()
    assert L.lib.anima_rt_run_gemm_bf16(x.ctypes.data, x.ctypes.data, x.ctypes.data, -1, 2, 2) is False


# ---------------------------------------------------------------- GPU numerics
def _torch():
    import torch
    return torch


def _ref_lib():
    """The compiled reference (oracle/_ref) with the reference binding's signatures, or None."""
    if not O.have_reference():
        return None
    lib = ct.CDLL(O.REF_SO)
    for name in BOUND_BY_REFERENCE:
        fn = getattr(lib, name)
        if name != "anima_rt_init":
            fn.argtypes = L.SIGNATURES[name][0]
        fn.restype = L.SIGNATURES[name][1]
    assert lib.anima_rt_init()
    return lib


@pytest.fixture(scope="module")
def rt():
    import torch
    torch.cuda.set_device(0)
    assert L.lib.anima_rt_init(), L.last_error()
    return L.lib


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 7, 4096, 100003])
def test_gelu_silu_match_torch(rt, n):
    torch = _torch()
    x = (np.random.default_rng(n).standard_normal(n) * 4).astype(np.float32)
    for name, f in (("anima_rt_run_gelu", torch.nn.functional.gelu),
                    ("anima_rt_run_silu", torch.nn.functional.silu)):
        out = np.full(n, np.nan, np.float32)
        assert getattr(rt, name)(x.ctypes.data, out.ctypes.data, n), L.last_error()
        ref = f(torch.from_numpy(x).double()).numpy()
        assert max_abs(out, ref) <= 2e-6 * max(1.0, float(np.abs(ref).max())), name
        ref_lib = _ref_lib()
        if ref_lib is not None:
            r2 = np.zeros(n, np.float32)
            assert getattr(ref_lib, name)(x.ctypes.data, r2.ctypes.data, n)
            assert max_abs(out, r2) <= 2e-6 * max(1.0, float(np.abs(r2).max())), name


@pytest.mark.gpu
@pytest.mark.parametrize("m,d", [(1, 128), (33, 2048), (300, 77), (4, 5000)])
def test_layernorm_softmax_match_torch(rt, m, d):
    torch = _torch()
    rng = np.random.default_rng(m * 7 + d)
    x = (rng.standard_normal((m, d)) * 3 + 0.5).astype(np.float32)
    out = np.full((m, d), np.nan, np.float32)
    assert rt.anima_rt_run_layernorm(x.ctypes.data, out.ctypes.data, m, d, ct.c_float(1e-6)), L.last_error()
    ref = torch.nn.functional.layer_norm(torch.from_numpy(x).double(), (d,), eps=1e-6).numpy()
    assert max_abs(out, ref) <= 2e-5
    out = np.full((m, d), np.nan, np.float32)
    assert rt.anima_rt_run_softmax(x.ctypes.data, out.ctypes.data, m, d), L.last_error()
    ref = torch.softmax(torch.from_numpy(x).double(), -1).numpy()
    assert max_abs(out, ref) <= 1e-6 and rel_l2(out, ref) <= 1e-5
    ref_lib = _ref_lib()
    if ref_lib is not None:
        r2 = np.zeros((m, d), np.float32)
        assert ref_lib.anima_rt_run_softmax(x.ctypes.data, r2.ctypes.data, m, d)
        # the reference sums a row sequentially in fp32: its own error grows with d
        assert rel_l2(out, r2) <= 1e-5 and max_abs(out, r2) <= 5e-6


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (37, 130, 70), (256, 512, 1024), (1000, 48, 3)])
def test_gemm_fp32_and_bf16_match_torch(rt, M, N, K):
    torch = _torch()
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    Bf = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    C = np.full((M, N), np.nan, np.float32)
    assert rt.anima_rt_run_gemm_fp32(A.ctypes.data, Bf.ctypes.data, C.ctypes.data, M, N, K), L.last_error()
    ref = (torch.from_numpy(A).double() @ torch.from_numpy(Bf).double().T).numpy()
    assert rel_l2(C, ref) <= 1e-6
    # bf16 weights as uint16 bit patterns, widened exactly
    Wb = torch.from_numpy(Bf).to(torch.bfloat16)
    W16 = np.ascontiguousarray(Wb.view(torch.int16).numpy().view(np.uint16))
    C2 = np.full((M, N), np.nan, np.float32)
    assert rt.anima_rt_run_gemm_bf16(A.ctypes.data, W16.ctypes.data, C2.ctypes.data, M, N, K), L.last_error()
    ref2 = (torch.from_numpy(A).double() @ Wb.double().T).numpy()
    assert rel_l2(C2, ref2) <= 1e-6
    ref_lib = _ref_lib()
    if ref_lib is not None and M * N * K <= 2 ** 22:
        r3 = np.zeros((M, N), np.float32)
        assert ref_lib.anima_rt_run_gemm_bf16(A.ctypes.data, W16.ctypes.data, r3.ctypes.data, M, N, K)
        assert rel_l2(C2, r3) <= 1e-6
