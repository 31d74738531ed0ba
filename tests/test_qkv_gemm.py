"""anima_qkv_projection: the projection GEMM with the prologue in its epilogue (GPU).

Against the same math in fp32 on the GPU with torch: C = x W^T, per-head RMSNorm of q and k
(weights [128], eps 1e-6), RoPE pairs (p, 64 + p) on q and k with the reference's table
layout, then the head-major [B*H, L, 128] layout -- i.e. the projection of
src/predict2.py:174-193 / numpy_dit.py:276-291 followed by the prologue, without the 16-bit
rounding of the projection in between.  Bar: rel-L2 <= 2e-3 and max-abs <= 2e-2 per output
(16-bit rounding of the stored operands), over shapes with partial row, column and depth
tiles.
"""
import numpy as np
import pytest

from conftest import max_abs, rel_l2

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _ref(x, w, H, n_tensors, first, qw, kw, freqs, eps, norm_q, norm_k):
    import torch.nn.functional as F
    B, L, K = x.shape
    c = (x.float().reshape(B * L, K) @ w.float().t()).view(B, L, n_tensors, H, 128)
    outs = [None, None, None]
    for i in range(n_tensors):
        t = first + i
        y = c[:, :, i]
        if t < 2 and (norm_q if t == 0 else norm_k):
            y = F.rms_norm(y, (128,), qw if t == 0 else kw, eps)
        if t < 2 and freqs is not None:
            f = freqs.view(L, 64, 4)[None, :, None]
            a, d = y[..., :64], y[..., 64:]
            y = torch.cat([f[..., 0] * a + f[..., 1] * d, f[..., 2] * a + f[..., 3] * d], -1)
        outs[t] = y.permute(0, 2, 1, 3).reshape(B * H, L, 128)
    return outs


CASES = [  # B, L, H, K, n_tensors, first, dtype, rope, norm
    (2, 256, 4, 2048, 3, 0, torch.float16, True, True),     # the DiT's self-attention (H=4 per GPU)
    (1, 96, 3, 200, 3, 0, torch.bfloat16, True, True),      # partial M, N (4.5 tiles) and K tiles
    (2, 128, 16, 1024, 1, 0, torch.float16, False, True),   # q only (cross-attention query)
    (1, 64, 2, 512, 2, 1, torch.float16, False, True),      # k and v (a context's K/V)
    (2, 32, 1, 64, 3, 0, torch.bfloat16, True, False),      # no norm, one head, one k tile
]


@pytest.mark.parametrize("B,L,H,K,n,first,dt,rope,norm", CASES)
def test_fused_projection_matches_fp32_math(B, L, H, K, n, first, dt, rope, norm):
    import anima_attn
    from anima_attn import ops
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + L + H + K)
    x = torch.randn(B, L, K, device="cuda", generator=g).to(dt)
    w = (0.02 * torch.randn(n * H * 128, K, device="cuda", generator=g)).to(dt)
    qw = 1 + 0.1 * torch.randn(128, device="cuda", generator=g)
    kw = 1 + 0.1 * torch.randn(128, device="cuda", generator=g)
    side = int(np.sqrt(L)) if int(np.sqrt(L)) ** 2 == L else None
    freqs = None
    if rope:
        freqs = (anima_attn.rope_freqs_3d(1, side, side, device="cuda") if side else
                 anima_attn.rope_freqs_3d(1, L // 8, 8, device="cuda"))
    got = ops.qkv_projection(x, w, H, n, first, qw, kw, freqs, 1e-6, norm, norm)
    torch.cuda.synchronize()
    assert anima_attn.status() == 0
    ref = _ref(x, w, H, n, first, qw, kw, freqs, 1e-6, norm, norm)
    for t in range(3):
        if ref[t] is None:
            assert got[t] is None
            continue
        a, r = got[t].float().cpu().numpy(), ref[t].float().cpu().numpy()
        assert np.isfinite(a).all()
        assert rel_l2(a, r) <= 2e-3 and max_abs(a, r) <= 2e-2, (t, rel_l2(a, r), max_abs(a, r))


def test_fused_projection_rejects_unsupported_shapes():
    from anima_attn import ops, AnimaError
    torch.cuda.set_device(0)
    x = torch.zeros(1, 48, 64, device="cuda", dtype=torch.float16)  # L not a multiple of 32
    w = torch.zeros(3 * 128, 64, device="cuda", dtype=torch.float16)
    with pytest.raises(AnimaError):
        ops.qkv_projection(x, w, 1)


@pytest.mark.parametrize("M,N,K,dt", [(8192, 8192, 2048, torch.float16), (300, 528, 200, torch.bfloat16),
                                      (33, 16, 8, torch.float16)])
def test_gemm_gelu_matches_fp32_math(M, N, K, dt):
    """anima_gemm_gelu: GELU(x W^T) with the exact GELU on the fp32 accumulator, against the
    same in fp32 torch.  (8192, 8192, 2048) is the DiT MLP's first layer (B=2 x 4096 tokens,
    hidden 2048 -> 8192); the others leave partial row, column and depth tiles."""
    import torch.nn.functional as F
    from anima_attn import ops
    import anima_attn
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).to(dt)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(dt)
    y = ops.gemm_gelu(x, w)
    torch.cuda.synchronize()
    assert anima_attn.status() == 0
    ref = F.gelu(x.float() @ w.float().t())
    a, r = y.float().cpu().numpy(), ref.cpu().numpy()
    assert np.isfinite(a).all()
    tol = 4e-3 if dt == torch.bfloat16 else 2e-3  # 16-bit rounding of the output
    assert rel_l2(a, r) <= tol and max_abs(a, r) <= 3e-2, (rel_l2(a, r), max_abs(a, r))
