"""compat.patch_predict2 on the reference's own model (CPU).

The patch replaces the reference's attention call sites in a loaded ``predict2`` module
(src/predict2.py:25-38, 201-214; the same points the reference patches in
anima_rt/scripts/phone_pipeline_anima_rt.py:224-252).  Here it is applied to the reference
MiniTrainDIT itself, with CPU stand-ins for the three operations it installs, so what is
checked is the patch's plumbing -- which call sites it takes over, the layouts and
reshapes it hands on, the RoPE table it extracts for any batch size and frame count -- against
the unpatched reference: the 2-block golden velocity (tests/golden/dit_small.npz) and
on-the-fly runs at T = 2.  The GPU operations behind the default backend are tested on the
GPU (tests/test_attn_gpu.py).  Needs the reference checkout; skipped without it.
"""
import os
import sys

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import golden, rel_l2
from dit_cpu_attention import cpu_attention, rope as cpu_rope
from oracle import oracle as O


def _predict2():
    tree = O.reference_tree()
    if tree is None:
        pytest.skip("reference checkout not available (set ANIMA_REFERENCE_TREE)")
    src = os.path.join(tree, "src")
    if src not in sys.path:
        sys.path.insert(0, src)
    import predict2
    return predict2


class _Ops:
    Linear = torch.nn.Linear
    LayerNorm = torch.nn.LayerNorm
    RMSNorm = torch.nn.RMSNorm


def _model(p2, blocks=2):
    from anima_attn.dit import DiTConfig, make_weights
    cfg = DiTConfig(blocks=blocks)
    m = p2.MiniTrainDIT(
        max_img_h=240, max_img_w=240, max_frames=128, in_channels=16, out_channels=16,
        patch_spatial=2, patch_temporal=1, concat_padding_mask=True, model_channels=2048,
        num_blocks=blocks, num_heads=16, mlp_ratio=4.0, crossattn_emb_channels=1024,
        pos_emb_cls="rope3d", pos_emb_learnable=True, pos_emb_interpolation="crop",
        min_fps=1, max_fps=30, use_adaln_lora=True, adaln_lora_dim=256,
        rope_h_extrapolation_ratio=4.0, rope_w_extrapolation_ratio=4.0,
        rope_t_extrapolation_ratio=1.0, extra_per_block_abs_pos_emb=False,
        rope_enable_fps_modulation=False, device="cpu", dtype=torch.float32, operations=_Ops)
    sd = {k: v.float() for k, v in make_weights(cfg, seed=1234).items()}
    m.load_state_dict(sd, strict=False)
    return m.eval()


class _Counting:
    """CPU backend that counts the calls each patched point makes."""

    def __init__(self):
        self.calls = {"sdpa": 0, "rope": 0, "attention": 0}

    def sdpa(self, q, k, v):
        self.calls["sdpa"] += 1
        return F.scaled_dot_product_attention(q.float(), k.float(), v.float()).to(q.dtype)

    def rope(self, t, freqs):
        self.calls["rope"] += 1
        assert freqs.shape == (t.shape[1], t.shape[-1] // 2, 2, 2)
        return cpu_rope(t.float(), freqs).to(t.dtype)

    def attention(self, *a, **kw):
        self.calls["attention"] += 1
        return cpu_attention(*a, **kw)


def _run(m, x, ctx, sigma):
    with torch.no_grad():
        return m(x, torch.full((x.shape[0],), sigma), ctx)


@pytest.mark.parametrize("fused", [True, False])
def test_patched_reference_model_matches_golden_velocity(fused):
    p2 = _predict2()
    from anima_attn import compat
    g = golden("dit_small.npz")
    rng = np.random.default_rng(4321)  # tests/golden/make_golden_dit.py inputs(32)
    x = rng.standard_normal((1, 16, 32, 32), dtype=np.float32)
    cc = rng.standard_normal((1, 512, 1024), dtype=np.float32)
    cu = rng.standard_normal((1, 512, 1024), dtype=np.float32)
    m = _model(p2)
    be = _Counting()
    orig = compat.patch_predict2(p2, compat.Predict2Backend(be.sdpa, be.rope, be.attention),
                                 fused=fused)
    try:
        xb = torch.from_numpy(x)[:, :, None].repeat(2, 1, 1, 1, 1)
        ctx = torch.cat([torch.from_numpy(cu), torch.from_numpy(cc)], dim=0)
        v = _run(m, xb, ctx, float(g["sigma"]))
    finally:
        compat.unpatch_predict2(p2, orig)
    assert rel_l2(v.numpy(), g["v"]) <= 1e-4
    blocks = 2
    if fused:  # one fused call per attention; the two reference points are not reached
        assert be.calls == {"sdpa": 0, "rope": 0, "attention": 2 * blocks}
    else:      # the reference's patch set: SDPA per attention, RoPE on q and k per self-attn
        assert be.calls == {"sdpa": 2 * blocks, "rope": 2 * blocks, "attention": 0}
    assert p2.Attention.forward is orig["Attention.forward"]


def test_patched_reference_model_several_frames_and_batch():
    """T = 2 latent frames (a 3D RoPE table over t, h, w) and a batch of 3: the patched
    model equals the unpatched one."""
    p2 = _predict2()
    from anima_attn import compat
    g = torch.Generator().manual_seed(7)
    x = torch.randn(3, 16, 2, 8, 8, generator=g)
    ctx = torch.randn(3, 77, 1024, generator=g)
    m = _model(p2, blocks=1)
    ref = _run(m, x, ctx, 0.3)
    be = _Counting()
    orig = compat.patch_predict2(p2, compat.Predict2Backend(be.sdpa, be.rope, be.attention))
    try:
        got = _run(m, x, ctx, 0.3)
    finally:
        compat.unpatch_predict2(p2, orig)
    assert be.calls["attention"] == 2
    assert rel_l2(got.numpy(), ref.numpy()) <= 1e-5


def test_patch_rejects_a_rope_table_of_the_wrong_size():
    from anima_attn import compat
    with pytest.raises(ValueError, match="does not hold one"):
        compat._freqs_per_token(torch.zeros(2, 64, 1, 64, 2, 2), 64, 128)
    assert compat._freqs_per_token(torch.zeros(1, 64, 1, 64, 2, 2), 64, 128).shape == (64, 64, 2, 2)
