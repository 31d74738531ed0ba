"""Golden latent of the reference sampler, for tests of anima_attn.sampling.

Run where the reference checkout is available ($ANIMA_REFERENCE_TREE, or a sibling checkout
named ``reference`` next to this repository):

    python tests/golden/make_golden_sampler.py

It runs the reference's own run_ksampler (anima_rt/scripts/sampling.py:183-209: the z_image
schedule, seeded noise and EulerSampler.sample) around the reference MiniTrainDIT
(src/predict2.py, fp32 on CPU) with the seeded 2-block weights of make_golden_dit.py, a
32x32 latent (256 tokens), 3 steps, CFG 5, and writes sampler_small.npz: the reference's
sigmas and noise and its final latent (the contexts come from np.random.default_rng(99)).
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

BLOCKS, SIDE, STEPS, CFG, SEED, CTX_SEED = 2, 32, 3, 5.0, 6666, 99


def main():
    import torch
    sys.path.insert(0, os.path.join(REF, "src"))
    sys.path.insert(0, os.path.join(REF, "anima_rt", "scripts"))
    sys.path.insert(0, HERE)
    import predict2
    import sampling
    from make_golden_dit import _Ops
    from anima_attn.dit import DiTConfig, make_weights

    cfg = DiTConfig(blocks=BLOCKS)
    model = predict2.MiniTrainDIT(
        max_img_h=240, max_img_w=240, max_frames=128, in_channels=16, out_channels=16,
        patch_spatial=2, patch_temporal=1, concat_padding_mask=True, model_channels=2048,
        num_blocks=BLOCKS, num_heads=16, mlp_ratio=4.0, crossattn_emb_channels=1024,
        pos_emb_cls="rope3d", pos_emb_learnable=True, pos_emb_interpolation="crop",
        min_fps=1, max_fps=30, use_adaln_lora=True, adaln_lora_dim=256,
        rope_h_extrapolation_ratio=4.0, rope_w_extrapolation_ratio=4.0,
        rope_t_extrapolation_ratio=1.0, extra_per_block_abs_pos_emb=False,
        rope_enable_fps_modulation=False, device="cpu", dtype=torch.float32, operations=_Ops)
    model.load_state_dict({k: v.float() for k, v in make_weights(cfg, seed=1234).items()},
                          strict=False)
    model.eval()

    class NumpyModel:  # the model.forward(x_np, sigma_np, ctx_np) interface the sampler calls
        def forward(self, x, sigma, ctx):
            with torch.no_grad():
                return model(torch.from_numpy(x), torch.from_numpy(sigma),
                             torch.from_numpy(ctx)).numpy()

    rng = np.random.default_rng(CTX_SEED)
    cc = rng.standard_normal((1, 512, 1024), dtype=np.float32)
    cu = rng.standard_normal((1, 512, 1024), dtype=np.float32)
    conf = sampling.PipelineConfig(H=SIDE, W=SIDE, steps=STEPS, cfg=CFG, seed=SEED,
                                   sampler="euler", scheduler="z_image")
    t0 = time.time()
    latent = sampling.run_ksampler(NumpyModel(), conf, cc, cu)
    print(f"reference sampler: {STEPS} steps in {time.time() - t0:.1f} s")
    sigmas = sampling.ZImageScheduler().get_sigmas(STEPS, 1.0)
    noise = np.random.default_rng(SEED).standard_normal((1, 16, SIDE, SIDE), dtype=np.float32)
    # the contexts are not stored: np.random.default_rng(CTX_SEED) regenerates them
    np.savez_compressed(os.path.join(HERE, "sampler_small.npz"),
                        sigmas=sigmas, noise=noise, latent=latent.astype(np.float32),
                        meta=np.array([BLOCKS, SIDE, STEPS, SEED, CTX_SEED]), cfg=np.float32(CFG))


if __name__ == "__main__":
    main()
