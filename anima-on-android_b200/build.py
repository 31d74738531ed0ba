"""Build libanima_attn.so in-tree with nvcc for sm_100a (no GPU needed).

    python anima-on-android_b200/build.py [--verbose]

The library lands next to the Python package (anima_attn/libanima_attn.so), so it
travels with a snapshot of the repository; nothing is installed into site-packages.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "anima_attn", "libanima_attn.so")
SOURCES = ["attn_fwd.cu", "attn_fwd64.cu", "attn_fwd2.cu", "prologue.cu", "dit_ops.cu", "selftest.cu",
           "rt_ops.cu", "qkv_gemm.cu", "abi.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def needs_rebuild() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps += [os.path.join(REPO, "include", f) for f in os.listdir(os.path.join(REPO, "include"))]
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_rebuild():
        return OUT
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           f"-I{os.path.join(REPO, 'include')}", "-o", OUT + ".tmp",
           *[os.path.join(CSRC, s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose, a.force))
    sys.exit(0)
