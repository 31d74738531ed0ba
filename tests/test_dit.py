"""The DiT step harness (one full Euler+CFG step) against the reference model.

CPU tests: the harness's block arithmetic, patching, timestep/adaLN-LoRA and CFG step,
with a CPU attention injected, against the reference MiniTrainDIT (tests/golden/
dit_small.npz); and the head-parallel path (2 gloo ranks, all-gather before the o-proj)
against the single-rank result.  GPU tests run the same step with the B200 kernels,
small and at full size (28 blocks, 4096 tokens; bar: latent rel-L2 <= 1e-2)."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, rel_l2

LATENT_REL_L2 = 1e-2  # required bar: denoised latent after one full step


def _load(which):
    g = np.load(os.path.join(GOLDEN, f"dit_{which}.npz"))
    blocks, side, wseed, iseed = (int(v) for v in g["meta"])
    rng = np.random.default_rng(iseed)
    x = rng.standard_normal((1, 16, side, side), dtype=np.float32)
    cc = rng.standard_normal((1, 512, 1024), dtype=np.float32)
    cu = rng.standard_normal((1, 512, 1024), dtype=np.float32)
    return g, blocks, wseed, x, cc, cu


def _step(model, g, x, cc, cu, device):
    T = lambda a: torch.from_numpy(a).to(device)
    return model.euler_cfg_step(T(x), float(g["sigma"]), float(g["sigma_next"]), T(cc), T(cu),
                                float(g["cfg"]))


def test_harness_matches_reference_model_cpu():
    from anima_attn.dit import AnimaDiT, DiTConfig, make_weights
    from dit_cpu_attention import cpu_attention
    g, blocks, wseed, x, cc, cu = _load("small")
    cfg = DiTConfig(blocks=blocks)
    model = AnimaDiT(cfg, make_weights(cfg, seed=wseed), attn_fn=cpu_attention)
    with torch.no_grad():
        out = _step(model, g, x, cc, cu, "cpu").numpy()
    assert rel_l2(out, g["x_next"]) <= LATENT_REL_L2


def _rank_main(rank, world, port, q, shard):
    import sys
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from anima_attn.dit import AnimaDiT, DiTConfig, make_weights
        from dit_cpu_attention import cpu_attention
        g, blocks, wseed, x, cc, cu = _load("small")
        cfg = DiTConfig(blocks=blocks)
        model = AnimaDiT(cfg, make_weights(cfg, seed=wseed), rank=rank, world=world,
                         attn_fn=cpu_attention, shard=shard)
        with torch.no_grad():
            out = _step(model, g, x, cc, cu, "cpu").numpy()
        if rank == 0:
            q.put(out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shard", ["tokens", "heads"])
def test_head_parallel_two_ranks_matches_reference_model_cpu(shard):
    """Two gloo ranks, 8 heads each, against the reference model's latent (same bar as one
    rank).  heads: one all_gather_into_tensor per attention before a replicated o-proj;
    tokens: rows split over the ranks, all_to_all_single into and out of the attention."""
    import torch.multiprocessing as mp
    g, blocks, wseed, x, cc, cu = _load("small")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200 + (0 if shard == "tokens" else 7)
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q, shard)) for r in range(2)]
    for p in procs:
        p.start()
    out = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert rel_l2(out, g["x_next"]) <= LATENT_REL_L2


@pytest.mark.gpu
@pytest.mark.parametrize("which", ["small", "full"])
@pytest.mark.parametrize("fused_qkv", [True, False])
def test_dit_step_on_gpu_matches_reference_model(which, fused_qkv):
    """fused_qkv: projections through anima_qkv_projection + the attention core (default),
    or cuBLAS projections + the prologue + the core."""
    from anima_attn.dit import AnimaDiT, DiTConfig, make_weights
    path = os.path.join(GOLDEN, f"dit_{which}.npz")
    if not os.path.exists(path):
        pytest.skip(f"{path} not generated")
    g, blocks, wseed, x, cc, cu = _load(which)
    cfg = DiTConfig(blocks=blocks)
    torch.cuda.set_device(0)
    model = AnimaDiT(cfg, make_weights(cfg, seed=wseed, device="cuda"), fused_qkv=fused_qkv)
    assert model.fused_qkv == fused_qkv
    with torch.no_grad():
        out = _step(model, g, x, cc, cu, "cuda").cpu().numpy()
    assert np.isfinite(out).all()
    r = rel_l2(out, g["x_next"])
    print(f"DiT step {which} fused_qkv={fused_qkv}: latent rel-L2 {r:.3e}")
    assert r <= LATENT_REL_L2


@pytest.mark.gpu
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
def test_ln_modulate_kernel_vs_torch(out_dtype):
    """anima_dit_ln_modulate against fp32 torch LayerNorm * (1 + scale) + shift, with
    scale/shift as chunks of one [B, 1, 3D] tensor (the adaLN layout)."""
    from anima_attn.ops import ln_modulate
    g = torch.Generator(device="cuda").manual_seed(7)
    B, S, D = 2, 777, 2048
    x = torch.randn(B, S, D, device="cuda", generator=g) * 3 + 0.5
    mods = torch.randn(B, 1, 3 * D, device="cuda", generator=g) * 0.2
    sh, sc, _ = mods.chunk(3, dim=-1)
    y = ln_modulate(x, sc, sh, 1e-6, out_dtype=out_dtype)
    ref = torch.nn.functional.layer_norm(x, (D,), eps=1e-6) * (1 + sc) + sh
    tol = 2 ** -8 if out_dtype == torch.float16 else 2 ** -5  # half an ulp of |y| < 4, plus fp32
    err = (y.float() - ref).abs() / ref.abs().clamp_min(1.0)
    assert err.max().item() <= tol


@pytest.mark.gpu
def test_gate_residual_kernel_vs_torch():
    from anima_attn.ops import gate_residual_
    g = torch.Generator(device="cuda").manual_seed(8)
    B, S, D = 2, 1031, 2048
    x = torch.randn(B, S, D, device="cuda", generator=g)
    y = torch.randn(B, S, D, device="cuda", generator=g)
    mods = torch.randn(B, 1, 3 * D, device="cuda", generator=g)
    gate = mods.chunk(3, dim=-1)[2]
    ref = x + gate * y
    out = gate_residual_(x, gate, y)
    assert out.data_ptr() == x.data_ptr()
    torch.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)


@pytest.mark.gpu
def test_step_graph_replay_matches_eager_step():
    """StepGraph (the step captured as one CUDA graph) gives the eager step's latent, also
    after new inputs are copied into its static buffers."""
    from anima_attn.dit import AnimaDiT, DiTConfig, StepGraph, make_weights
    g, blocks, wseed, x, cc, cu = _load("small")
    cfg = DiTConfig(blocks=blocks)
    torch.cuda.set_device(0)
    model = AnimaDiT(cfg, make_weights(cfg, seed=wseed, device="cuda"))
    T = lambda a: torch.from_numpy(a).cuda()
    s, sn, c = float(g["sigma"]), float(g["sigma_next"]), float(g["cfg"])
    with torch.no_grad():
        graph = StepGraph(model, T(x), s, sn, T(cc), T(cu), c)
        for scale in (1.0, 0.5):
            xs = T(x) * scale
            eager = model.euler_cfg_step(xs, s, sn, T(cc), T(cu), c).cpu().numpy()
            replay = graph(xs).cpu().numpy()
            assert rel_l2(replay, eager) <= 1e-6
        assert rel_l2(graph(T(x)).cpu().numpy(), g["x_next"]) <= LATENT_REL_L2


@pytest.mark.gpu
@pytest.mark.parametrize("out_dtype,y_dtype", [(torch.float16, torch.float32),
                                               (torch.bfloat16, torch.float32),
                                               (torch.float16, torch.float16)])
def test_gate_residual_ln_modulate_kernel_vs_torch(out_dtype, y_dtype):
    """anima_dit_gate_residual_ln_modulate: x += gate*y in place, then the modulated
    LayerNorm of the updated x, against fp32 torch (y as the GEMM wrote it)."""
    from anima_attn.ops import gate_residual_ln_modulate_
    g = torch.Generator(device="cuda").manual_seed(9)
    B, S, D = 2, 517, 2048
    x = torch.randn(B, S, D, device="cuda", generator=g) * 2
    y = torch.randn(B, S, D, device="cuda", generator=g).to(y_dtype)
    mods = torch.randn(B, 1, 6 * D, device="cuda", generator=g) * 0.3
    gate, _, _ = mods[:, :, :3 * D].chunk(3, dim=-1)
    sh, sc, _ = mods[:, :, 3 * D:].chunk(3, dim=-1)
    x_ref = x + gate * y
    ref = torch.nn.functional.layer_norm(x_ref, (D,), eps=1e-6) * (1 + sc) + sh
    h = gate_residual_ln_modulate_(x, gate, y, sc, sh, 1e-6, out_dtype=out_dtype)
    torch.testing.assert_close(x, x_ref, rtol=1e-6, atol=1e-5)
    tol = 2 ** -8 if out_dtype == torch.float16 else 2 ** -5
    assert ((h.float() - ref).abs() / ref.abs().clamp_min(1.0)).max().item() <= tol


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gelu_kernel_vs_torch(dtype):
    from anima_attn.ops import gelu_
    g = torch.Generator(device="cuda").manual_seed(10)
    x = (torch.randn(1024, 520, device="cuda", generator=g) * 3).to(dtype)
    ref = torch.nn.functional.gelu(x.float())
    out = gelu_(x.clone())
    ulp = 2 ** -10 if dtype == torch.float16 else 2 ** -7  # one 16-bit ulp, relative
    assert ((out.float() - ref).abs() <= ref.abs() * ulp + 1e-3 * ulp).all()
