"""The C-ABI boundary without a GPU: the library loads, exports every declared symbol,
its struct layouts match the headers, and host-side validation fails cleanly."""
import ctypes as ct
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import REPO, has_gpu

import anima_attn
from anima_attn import _lib as L

HEADERS = [os.path.join(REPO, "include", h) for h in ("anima_rt.h", "anima_attn.h")]


def declared_functions():
    names = []
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(anima_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_every_declared_symbol_is_exported_and_bound():
    names = declared_functions()
    assert "anima_rt_run_sdpa_flash" in names and "anima_attn_fwd" in names
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    assert set(names) == set(L.SIGNATURES), set(names) ^ set(L.SIGNATURES)
    for n in names:
        assert getattr(L.lib, n) is not None


def test_reference_signatures_unchanged():
    """The drop-in symbols keep the reference's ctypes argtypes (anima_rt_ops.py:11-34)."""
    P = ct.c_void_p
    assert L.SIGNATURES["anima_rt_run_sdpa_flash"][0] == [P] * 4 + [ct.c_int] * 4 + [ct.c_float, ct.c_bool]
    assert L.SIGNATURES["anima_rt_run_rmsnorm"][0] == [P, P, P, ct.c_int, ct.c_int, ct.c_float]
    assert L.SIGNATURES["anima_rt_run_rope"][0] == [P, P, P, ct.c_int, ct.c_int, ct.c_int]


def _c_layout(struct, fields, tmp_path):
    src = tmp_path / "layout.c"
    body = "\n".join(f'printf("{f} %zu\\n", offsetof({struct}, {f}));' for f in fields)
    src.write_text(f"""#include <stdio.h>
#include <stddef.h>
#include "anima_attn.h"
int main(void) {{ printf("size %zu\\n", sizeof({struct})); {body} return 0; }}""")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    return {k: int(v) for k, v in (line.split() for line in out.strip().splitlines())}


@pytest.mark.parametrize("cls,cname", [(L.PrologueArgs, "AnimaPrologueArgs"), (L.AttnArgs, "AnimaAttnArgs"),
                                       (L.QkvProjArgs, "AnimaQkvProjArgs")])
def test_struct_layout_matches_header(cls, cname, tmp_path):
    fields = [f for f, _ in cls._fields_]
    c = _c_layout(cname, fields, tmp_path)
    assert c["size"] == ct.sizeof(cls)
    for f in fields:
        assert c[f] == getattr(cls, f).offset, f


def test_sdpa_flash_rejects_unsupported_head_size_without_aborting():
    q = np.zeros((1, 4, 64), np.float32)
    ok = L.lib.anima_rt_run_sdpa_flash(q.ctypes.data, q.ctypes.data, q.ctypes.data, q.ctypes.data,
                                       1, 4, 4, 64, ct.c_float(0.125), ct.c_bool(False))
    assert ok is False
    assert "head size" in L.last_error()


def test_null_and_empty_arguments_fail_cleanly():
    assert L.lib.anima_rt_run_sdpa_flash(None, None, None, None, 1, 4, 4, 128,
                                         ct.c_float(0.1), ct.c_bool(False)) is False
    assert "null" in L.last_error()
    q = np.zeros((1, 4, 128), np.float32)
    assert L.lib.anima_rt_run_sdpa_flash(q.ctypes.data, q.ctypes.data, q.ctypes.data,
                                         q.ctypes.data, 0, 4, 4, 128, ct.c_float(0.1),
                                         ct.c_bool(False)) is False
    assert L.lib.anima_attn_fwd(None, None) == L.ERR_ARG
    assert L.lib.anima_attn_prologue(None, None) == L.ERR_ARG


@pytest.mark.skipif(has_gpu(), reason="checks behaviour without a device")
def test_init_without_device_returns_false():
    assert L.lib.anima_rt_init() is False
    assert L.lib.anima_attn_device_info(None, None) == L.ERR_CUDA


def test_rmsnorm_before_init_returns_false_like_reference():
    """anima_rt.cpp:45-50: run_rmsnorm returns false while g_backend is null."""
    L.lib.anima_rt_destroy()
    x = np.ones((2, 128), np.float32)
    assert L.lib.anima_rt_run_rmsnorm(x.ctypes.data, None, x.ctypes.data, 2, 128,
                                      ct.c_float(1e-6)) is False


def test_version_string():
    assert "sm_100a" in anima_attn.version()


# (S_q, S_kv, flags) -> schedule anima_attn_fwd runs on a 148-SM B200 with B=2, H=16: the
# choices measured fastest and listed with the planner (csrc/attn_fwd.cu, plan_split).
SCHEDULES = [
    (2048, 2048, 0, "whole"), (2560, 2560, 0, "cut"), (3072, 3072, 0, "cut"),
    (4096, 4096, 0, "cut"), (5120, 5120, 0, "cut"), (6144, 6144, 0, "cut"),
    (8192, 8192, 0, "unit"), (16384, 16384, 0, "unit"), (4096, 512, 0, "whole"),
    (4096, 1024, 0, "whole"), (4096, 2048, 0, "cut"),
    (1024, 1024, 0, "unit"),                                 # 128 units: one wave
    (4096, 4096, L.FLAG_MASK, "unit"), (4096, 4096, L.FLAG_CAUSAL, "unit"),
    (4096, 4096, L.FLAG_UNIT, "unit"), (4096, 4096, L.FLAG_WHOLE, "whole"),
    (2048, 2048, L.FLAG_SPLIT, "cut"), (8192, 8192, L.FLAG_SPLIT, "cut"),
    (4096, 4096, L.FLAG_PAIR, "unit"), (4096, 4096, L.FLAG_KV64, "cut"),
    (4096, 512, L.FLAG_KV64, "whole"),
    (4096, 512, L.FLAG_MASK, "whole"), (4096, 2048, L.FLAG_MASK, "whole"),  # cross-attention
    (4096, 512, L.FLAG_MASK | L.FLAG_SPLIT, "whole"),  # masked calls are never cut
    (4096, 4096, L.FLAG_MASK | L.FLAG_WHOLE, "whole"), (1024, 512, L.FLAG_MASK, "unit"),
    (4096, 512, L.FLAG_MASK | L.FLAG_KV64, "unit"),
]
SCHED_CODE = {"unit": 0, "whole": 1, "cut": 2}


@pytest.mark.parametrize("Sq,Skv,flags,want", SCHEDULES)
def test_schedule_choice(Sq, Skv, flags, want):
    """The schedule query runs the launcher's own planner on the host (no GPU needed when
    the SM count is given)."""
    assert L.lib.anima_attn_schedule(2, 16, Sq, Skv, flags, 148) == SCHED_CODE[want]


@pytest.mark.parametrize("H,want", [(16, "cut"), (8, "whole"), (4, "unit"), (2, "cut"), (1, "cut")])
def test_schedule_choice_by_heads_per_gpu(H, want):
    """B=2, L=4096 split over 1/2/4/8 GPUs by head: 512, 256, 128, 64 units on 148 SMs.  One
    wave that would leave most SMs idle (2 heads: 64 units; 1 head: 32) is cut over all SMs;
    ANIMA_FLAG_UNIT and ANIMA_FLAG_WHOLE keep one CTA per unit there."""
    assert L.lib.anima_attn_schedule(2, H, 4096, 4096, 0, 148) == SCHED_CODE[want]
    if H <= 4:
        assert L.lib.anima_attn_schedule(2, H, 4096, 4096, L.FLAG_UNIT, 148) == SCHED_CODE["unit"]
        assert L.lib.anima_attn_schedule(2, H, 4096, 4096, L.FLAG_WHOLE, 148) == SCHED_CODE["unit"]


def test_schedule_query_rejects_bad_shapes():
    assert L.lib.anima_attn_schedule(0, 16, 4096, 4096, 0, 148) < 0
    assert L.lib.anima_attn_schedule(2, 16, 4096, -1, 0, 148) < 0
