"""Golden latents for one full Euler+CFG DiT step, from the reference model.

    python tests/golden/make_golden_dit.py [small|full]

Runs the reference's own src/predict2.py MiniTrainDIT (fp32, CPU, torch SDPA) with the
Anima 2B configuration of anima_rt/scripts/phone_pipeline_anima_rt.py:192-200, weights
from anima_attn.dit.make_weights (seeded, bf16-rounded, loaded by their reference
names), and one EulerSampler step (anima_rt/scripts/sampling.py:121-138): CFG pair
[uncond, cond], cfg 5.0, sigma 0.5 -> 0.0.  Inputs are seeded; the fixture stores the
seeds, the inputs' shapes and the reference outputs.

  dit_small.npz  2 blocks, latent 16 x 32 x 32 (256 tokens), context 2 x 512 x 1024
  dit_full.npz   28 blocks, latent 16 x 128 x 128 (4096 tokens, 1024 x 1024 image)
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "anima-on-android_b200"))
sys.path.insert(0, REPO)
from oracle.oracle import reference_tree  # noqa: E402

REF = reference_tree()
if REF is None:
    raise SystemExit("no reference checkout: set ANIMA_REFERENCE_TREE")

CASES = {"small": dict(blocks=2, side=32), "full": dict(blocks=28, side=128)}
WEIGHT_SEED, INPUT_SEED = 1234, 4321
SIGMA, SIGMA_NEXT, CFG = 0.5, 0.0, 5.0


def inputs(side: int):
    rng = np.random.default_rng(INPUT_SEED)
    x = rng.standard_normal((1, 16, side, side), dtype=np.float32)
    ctx_cond = rng.standard_normal((1, 512, 1024), dtype=np.float32)
    ctx_uncond = rng.standard_normal((1, 512, 1024), dtype=np.float32)
    return x, ctx_cond, ctx_uncond


class _Ops:
    import torch.nn as nn
    Linear = nn.Linear
    LayerNorm = nn.LayerNorm
    RMSNorm = nn.RMSNorm


def main(which: str):
    import torch
    from anima_attn.dit import DiTConfig, make_weights
    sys.path.insert(0, os.path.join(REF, "src"))
    import predict2

    case = CASES[which]
    cfg = DiTConfig(blocks=case["blocks"])
    model = predict2.MiniTrainDIT(
        max_img_h=240, max_img_w=240, max_frames=128, in_channels=16, out_channels=16,
        patch_spatial=2, patch_temporal=1, concat_padding_mask=True, model_channels=2048,
        num_blocks=cfg.blocks, num_heads=16, mlp_ratio=4.0, crossattn_emb_channels=1024,
        pos_emb_cls="rope3d", pos_emb_learnable=True, pos_emb_interpolation="crop",
        min_fps=1, max_fps=30, use_adaln_lora=True, adaln_lora_dim=256,
        rope_h_extrapolation_ratio=4.0, rope_w_extrapolation_ratio=4.0,
        rope_t_extrapolation_ratio=1.0, extra_per_block_abs_pos_emb=False,
        rope_enable_fps_modulation=False, device="cpu", dtype=torch.float32, operations=_Ops)
    w = make_weights(cfg, seed=WEIGHT_SEED)
    sd = {k: v.float() for k, v in w.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    params = {n for n, _ in model.named_parameters()}
    assert not unexpected, unexpected
    assert params <= set(sd), params - set(sd)
    model.eval()

    x, cc, cu = inputs(case["side"])
    t0 = time.time()
    with torch.no_grad():
        xb = torch.from_numpy(x)[:, :, None].repeat(2, 1, 1, 1, 1)
        ctx = torch.cat([torch.from_numpy(cu), torch.from_numpy(cc)], dim=0)
        sig = torch.full((2,), SIGMA)
        v = model(xb, sig, ctx)
        v_cfg = v[0:1] + CFG * (v[1:2] - v[0:1])
        x_next = torch.from_numpy(x) + v_cfg[:, :, 0] * (SIGMA_NEXT - SIGMA)
    print(f"{which}: reference step in {time.time() - t0:.1f} s")
    extra = {"v": v.numpy().astype(np.float32)} if which == "small" else {}
    np.savez_compressed(os.path.join(HERE, f"dit_{which}.npz"), **extra,
                        x_next=x_next.numpy().astype(np.float32),
                        meta=np.array([cfg.blocks, case["side"], WEIGHT_SEED, INPUT_SEED]),
                        sigma=np.float32(SIGMA), sigma_next=np.float32(SIGMA_NEXT),
                        cfg=np.float32(CFG))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "small")
