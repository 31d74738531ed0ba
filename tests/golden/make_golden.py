"""Generate the golden fixtures in this directory from the reference itself.

Run where the reference checkout is available ($ANIMA_REFERENCE_TREE, or a sibling
checkout named ``reference`` next to this repository):

    python tests/golden/make_golden.py

It compiles the reference's anima_rt sources (``make -C oracle ref``), loads the
resulting library through the reference's own ctypes signatures, imports the
reference's Python modules (src/position_embedding.py, src/predict2.py), and writes
small .npz fixtures.  The GPU box has no reference tree; the tests there read only
these files.  Every array here is an output of reference code on seeded inputs:

  sdpa_square.npz   anima_rt_run_sdpa_flash, BH=1, S=256, D=128
  sdpa_ragged.npz   anima_rt_run_sdpa_flash, BH=2, Sq=130, Skv=77 (not tile multiples)
  sdpa_causal.npz   anima_rt_run_sdpa_flash, is_causal=True, BH=1, Sq=Skv=160
  sdpa_cross.npz    anima_rt_run_sdpa_flash, BH=1, Sq=256, Skv=512 (cross shape)
  rmsnorm.npz       anima_rt_run_rmsnorm M=64 D=128 (with and without weight)
  rope.npz          VideoRopePosition3DEmb 16x16 table, predict2.apply_rotary_pos_emb
                    and anima_rt_run_rope on t [1,256,1,128]
  prologue_sdpa.npz numpy_dit.py:285-292 composition (rmsnorm q,k -> rope -> sdpa)
                    on an 8x8 grid, B=1, H=2
  verify_flash.json the reference's own known-answer check
                    (scripts/archive/_verify_flash.py: torch.manual_seed(42) randn
                    [2,16,256,128], anima_rt flash vs torch F.sdpa) reduced to
                    checksums of the reference output and its max error vs torch
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle as O  # noqa: E402

REF = O.reference_tree()
if REF is None:
    raise SystemExit("no reference checkout: set ANIMA_REFERENCE_TREE")


def _ref_python():
    sys.path.insert(0, os.path.join(REF, "src"))
    import position_embedding  # noqa: F401
    import predict2
    return position_embedding, predict2


def main():
    import torch

    O.build(ref=True)
    if not O.have_reference():
        raise SystemExit("reference library not built; is the reference tree present?")
    pe, p2 = _ref_python()
    rng = np.random.default_rng(20261201)
    g = lambda *s: rng.standard_normal(s, dtype=np.float32)

    def sdpa_case(name, bh, sq, skv, causal=False):
        q, k, v = g(bh, sq, 128), g(bh, skv, 128), g(bh, skv, 128)
        out = O.sdpa(q, k, v, causal=causal, kind="reference")
        np.savez_compressed(os.path.join(HERE, name), q=q, k=k, v=v, out=out,
                            causal=np.int32(causal))

    sdpa_case("sdpa_square.npz", 1, 256, 256)
    sdpa_case("sdpa_ragged.npz", 2, 130, 77)
    sdpa_case("sdpa_causal.npz", 1, 160, 160, causal=True)
    sdpa_case("sdpa_cross.npz", 1, 256, 512)

    x, w = g(64, 128), (1.0 + 0.1 * g(128)).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "rmsnorm.npz"), x=x, w=w,
                        out_w=O.rmsnorm(x, w, 1e-6, kind="reference"),
                        out_nw=O.rmsnorm(x, None, 1e-6, kind="reference"))

    emb = pe.VideoRopePosition3DEmb(head_dim=128, len_h=16, len_w=16, len_t=1,
                                    h_extrapolation_ratio=4.0, w_extrapolation_ratio=4.0,
                                    t_extrapolation_ratio=1.0, enable_fps_modulation=False)
    freqs = emb.generate_embeddings(torch.Size([1, 1, 16, 16, 2048])).numpy()
    t = g(1, 256, 1, 128)
    rot_torch = p2.apply_rotary_pos_emb(torch.from_numpy(t),
                                        torch.from_numpy(freqs)[None, :, None]).numpy()
    rot_c = O.rope(t, freqs, kind="reference")
    np.savez_compressed(os.path.join(HERE, "rope.npz"), freqs=freqs, t=t,
                        out_predict2=rot_torch, out_anima_rt=rot_c)

    emb8 = pe.VideoRopePosition3DEmb(head_dim=128, len_h=8, len_w=8, len_t=1,
                                     h_extrapolation_ratio=4.0, w_extrapolation_ratio=4.0,
                                     t_extrapolation_ratio=1.0, enable_fps_modulation=False)
    f8 = emb8.generate_embeddings(torch.Size([1, 1, 8, 8, 2048])).numpy()
    q, k, v = g(1, 64, 2, 128), g(1, 64, 2, 128), g(1, 64, 2, 128)
    qw, kw = (1 + 0.1 * g(128)).astype(np.float32), (1 + 0.1 * g(128)).astype(np.float32)
    qh, kh, vh = O.prologue(q, k, v, qw, kw, f8, kind="reference")
    out = O.sdpa(qh, kh, vh, kind="reference")
    np.savez_compressed(os.path.join(HERE, "prologue_sdpa.npz"), q=q, k=k, v=v, q_w=qw,
                        k_w=kw, freqs=f8, q_ready=qh, k_ready=kh, out=out)

    # The reference's known-answer script, reduced to checksums.
    torch.manual_seed(42)
    B, H, S, D = 2, 16, 256, 128
    tq, tk, tv = (torch.randn(B, H, S, D) for _ in range(3))
    ref = O.sdpa(tq.numpy(), tk.numpy(), tv.numpy(), kind="reference", threads=8)
    pt = torch.nn.functional.scaled_dot_product_attention(tq, tk, tv).numpy()
    summary = {
        "source": "scripts/archive/_verify_flash.py:10-38 (torch.manual_seed(42), "
                  "randn B=2 H=16 S=256 D=128, anima_rt_run_sdpa_flash vs F.sdpa)",
        "shape": [B, H, S, D],
        "ref_sum": float(ref.astype(np.float64).sum()),
        "ref_abs_sum": float(np.abs(ref).astype(np.float64).sum()),
        "ref_l2": float(np.sqrt((ref.astype(np.float64) ** 2).sum())),
        "ref_first8": [float(x) for x in ref.reshape(-1)[:8]],
        "max_err_vs_torch_sdpa": float(np.abs(ref - pt).max()),
        "published_max_err": 4.77e-7,
    }
    with open(os.path.join(HERE, "verify_flash.json"), "w") as f:
        json.dump(summary, f, indent=1)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
