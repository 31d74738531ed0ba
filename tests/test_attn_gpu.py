"""Parity of the B200 kernels with the reference (oracle + golden fixtures), on a GPU.

Bar: rel-L2 <= 5e-3 and max-abs <= 2e-2 per attention output against the
reference's fp32 flash SDPA; the RoPE drop-in is bit-exact; the RMSNorm drop-in agrees
to fp32 rounding (its sum is a tree, the reference's is sequential).
"""
import ctypes as ct

import numpy as np
import pytest

from conftest import ATTN_MAX_ABS, ATTN_REL_L2, golden, max_abs, rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def aa():
    import anima_attn
    from anima_attn import _lib as L
    torch.cuda.set_device(0)
    assert L.lib.anima_rt_init()
    return anima_attn


@pytest.fixture(scope="module")
def O():
    from oracle import oracle
    oracle.build(ref=False)
    return oracle


def _ok(got, ref, rel=ATTN_REL_L2, mx=ATTN_MAX_ABS):
    r, m = rel_l2(got, ref), max_abs(got, ref)
    assert np.isfinite(got).all()
    assert r <= rel and m <= mx, f"rel-L2 {r:.3e} max-abs {m:.3e}"
    return r, m


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ------------------------------------------------------------------ drop-in C ABI
@pytest.mark.parametrize("name", ["sdpa_square.npz", "sdpa_ragged.npz", "sdpa_causal.npz",
                                  "sdpa_cross.npz"])
def test_sdpa_flash_dropin_vs_reference_fixture(aa, name):
    from anima_attn import _lib as L
    g = golden(name)
    q, k, v = g["q"], g["k"], g["v"]
    bh, sq, d = q.shape
    skv = k.shape[1]
    out = np.zeros_like(g["out"])
    ok = L.lib.anima_rt_run_sdpa_flash(q.ctypes.data, k.ctypes.data, v.ctypes.data,
                                       out.ctypes.data, bh, sq, skv, d,
                                       ct.c_float(1 / np.sqrt(d)), ct.c_bool(bool(g["causal"])))
    assert ok, L.last_error()
    _ok(out, g["out"])


def test_rope_dropin_bit_exact(aa):
    from anima_attn.compat import anima_rt_rope
    g = golden("rope.npz")
    assert np.array_equal(anima_rt_rope(g["t"], g["freqs"]), g["out_anima_rt"])


def test_rmsnorm_dropin(aa):
    from anima_attn.compat import NumpyRT
    g = golden("rmsnorm.npz")
    rt = NumpyRT({"blk.q_norm.weight": g["w"]})
    got = rt.run_rmsnorm(g["x"].reshape(2, 32, 128), "blk.q_norm").reshape(64, 128)
    assert max_abs(got, g["out_w"]) <= 2e-6
    assert rel_l2(got, g["out_w"]) <= 1e-6


def test_fused_host_entry_vs_reference_composition(aa):
    from anima_attn.compat import NumpyRT
    g = golden("prologue_sdpa.npz")
    rt = NumpyRT({"b.q_norm.weight": g["q_w"], "b.k_norm.weight": g["k_w"]})
    got = rt.run_attention(g["q"], g["k"], g["v"], "b", rope_emb=g["freqs"])
    _ok(got, g["out"].transpose(0, 2, 1, 3))


@pytest.mark.parametrize("B,H,Sq,Skv,masked", [(3, 6, 160, 200, True), (9, 1, 96, 96, False),
                                                (2, 16, 64, 64, False), (1, 8, 300, 200, True)])
def test_host_entry_chunks_vs_oracle(aa, O, B, H, Sq, Skv, masked):
    """anima_rt_run_attention pipelines the call over (batch rows x head group) chunks;
    odd B and H, a short last chunk (B=9, H=1 -> chunks of 2 rows), a last chunk split into
    g/2 + g/4 + g/4 heads (H=16 and H=8) and per-sample key padding all map back to the right
    output rows."""
    from anima_attn import _lib as L
    rng = np.random.default_rng(B * 100 + H)
    q = rng.standard_normal((B, Sq, H, 128), dtype=np.float32)
    k = rng.standard_normal((B, Skv, H, 128), dtype=np.float32)
    v = rng.standard_normal((B, Skv, H, 128), dtype=np.float32)
    qw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    valid = rng.integers(1, Skv + 1, size=B).astype(np.int32) if masked else None
    # a page-locked output where the head count lets the library split the last chunk
    keep = torch.zeros((B, Sq, H, 128), dtype=torch.float32, pin_memory=(H % 8 == 0))
    out = keep.numpy()
    ok = L.lib.anima_rt_run_attention(
        q.ctypes.data, k.ctypes.data, v.ctypes.data, qw.ctypes.data, None, None,
        None if valid is None else valid.ctypes.data, out.ctypes.data, B, Sq, Skv, H, 128,
        ct.c_float(1e-6), ct.c_float(128 ** -0.5), ct.c_uint(L.FLAG_QNORM))
    assert ok, L.last_error()
    rq, rk, rv = O.prologue(q, k, v, qw, None)  # [B, H, S, D]
    ref = O.sdpa_varlen(rq, rk, rv, valid) if masked else O.sdpa(rq, rk, rv)
    _ok(out.transpose(0, 2, 1, 3), ref)


def test_numpyrt_run_sdpa_shapes(aa):
    from anima_attn.compat import NumpyRT
    g = golden("sdpa_ragged.npz")
    rt = NumpyRT({})
    got = rt.run_sdpa(g["q"][None], g["k"][None], g["v"][None])
    _ok(got[0], g["out"])


# ------------------------------------------------------------------ device path
SHAPES = [  # (B, H, Sq, Skv, causal)
    (1, 1, 1, 1, False), (1, 2, 7, 7, False), (1, 1, 64, 64, False), (1, 2, 127, 129, False),
    (2, 2, 129, 127, False), (1, 3, 256, 256, False), (1, 1, 300, 1000, False),
    (1, 1, 513, 200, False), (1, 2, 256, 256, True), (1, 1, 200, 333, True),
]


@pytest.mark.parametrize("B,H,Sq,Skv,causal", SHAPES)
def test_attention_core_shapes(aa, O, B, H, Sq, Skv, causal):
    rng = np.random.default_rng(B * 1000 + Sq * 7 + Skv)
    q = rng.standard_normal((B, H, Sq, 128), dtype=np.float32)
    k = rng.standard_normal((B, H, Skv, 128), dtype=np.float32)
    v = rng.standard_normal((B, H, Skv, 128), dtype=np.float32)
    ref = O.sdpa(q, k, v, causal=causal)
    got = aa.sdpa(_dev(q), _dev(k), _dev(v), is_causal=causal)
    torch.cuda.synchronize()
    _ok(got.cpu().numpy(), ref)
    assert aa.status() == 0


@pytest.mark.parametrize("op_dtype", ["bf16", "f16"])
@pytest.mark.parametrize("out_dtype,layout", [("f32", "bshd"), ("bf16", "bshd"), ("f32", "bhsd")])
def test_operand_and_output_variants(aa, O, op_dtype, out_dtype, layout):
    rng = np.random.default_rng(5)
    B, H, S = 2, 3, 300
    q, k, v = (rng.standard_normal((B, S, H, 128), dtype=np.float32) for _ in range(3))
    qw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
    qh, kh, vh = aa.prologue(_dev(q), _dev(k), _dev(v), _dev(qw), _dev(kw), op_dtype=tdt[op_dtype])
    out = aa.attention_core(qh, kh, vh, B, H, out_layout=layout, out_dtype=tdt[out_dtype])
    torch.cuda.synchronize()
    rq, rk, rv = O.prologue(q, k, v, qw, kw)
    ref = O.sdpa(rq, rk, rv)  # [B,H,S,D]
    got = out.float().cpu().numpy()
    if layout == "bshd":
        got = got.transpose(0, 2, 1, 3)
    tol = 8e-3 if out_dtype == "bf16" else ATTN_REL_L2  # bf16 output adds 2^-9 rounding
    _ok(got, ref, rel=tol)


def test_prologue_matches_oracle_to_operand_rounding(aa, O):
    rng = np.random.default_rng(9)
    B, H, side = 2, 4, 10
    S = side * side
    q, k, v = (rng.standard_normal((B, S, H, 128), dtype=np.float32) for _ in range(3))
    qw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    fr = O.rope_freqs_3d(1, side, side)
    qh, kh, vh = aa.prologue(_dev(q), _dev(k), _dev(v), _dev(qw), _dev(kw), _dev(fr),
                             op_dtype=torch.float16)
    torch.cuda.synchronize()
    rq, rk, rv = O.prologue(q, k, v, qw, kw, fr)
    for got, ref in ((qh, rq), (kh, rk), (vh, rv)):
        g = got.float().cpu().numpy().reshape(ref.shape)
        # fp16 rounding of the fp32 oracle value: |err| <= 2^-11 |x| (+ tree-sum ulps)
        assert np.all(np.abs(g - ref) <= np.abs(ref) * 2.0 ** -10 + 1e-6)


@pytest.mark.parametrize("in_dtype", ["f16", "bf16"])
@pytest.mark.parametrize("H", [2, 6, 16])
def test_prologue_16bit_strided_views(aa, O, in_dtype, H):
    """16-bit projections read as strided views of one [B, S, 3, H, 128] GEMM output
    (the DiT's fused QKV projection), H not a multiple of the heads one pass covers."""
    rng = np.random.default_rng(30 + H)
    B, side = 2, 8
    S = side * side
    dt = torch.float16 if in_dtype == "f16" else torch.bfloat16
    qkv = torch.from_numpy(rng.standard_normal((B, S, 3, H, 128), dtype=np.float32)).to(dt)
    x = qkv.float().numpy()  # the values the kernel reads
    qw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    fr = O.rope_freqs_3d(1, side, side)
    d = qkv.cuda()
    qh, kh, vh = aa.prologue(d[:, :, 0], d[:, :, 1], d[:, :, 2], _dev(qw), _dev(kw), _dev(fr),
                             op_dtype=torch.float16)
    torch.cuda.synchronize()
    rq, rk, rv = O.prologue(*(np.ascontiguousarray(x[:, :, i]) for i in range(3)), qw, kw, fr)
    for got, ref in ((qh, rq), (kh, rk), (vh, rv)):
        g = got.float().cpu().numpy().reshape(ref.shape)
        assert np.all(np.abs(g - ref) <= np.abs(ref) * 2.0 ** -10 + 1e-6)


@pytest.mark.parametrize("H,grid,in_dtype", [(1, (1, 32, 32), "f32"), (2, (1, 64, 64), "f32"),
                                             (16, (1, 64, 64), "f32"), (40, (1, 16, 16), "f32"),
                                             (3, (10, 10, 10), "bf16"), (48, (2, 8, 8), "f16"),
                                             (64, (2, 8, 8), "f16")])
def test_prologue_layouts_and_head_counts(aa, O, H, grid, in_dtype):
    """The prologue over head counts that select each of its two kernels: few heads (fp32
    H <= 4, 16-bit H <= 8: several tokens per warp item, the head split over 4-16 GPUs) and
    one token per item otherwise.  Each runs on the usual [B, S, H, D] projection and on a
    head-major [B, H, S, D] tensor viewed as [B, S, H, D] (head stride S*D): the same bits
    from both layouts, and the oracle's operand-rounding bound.  S = 1000 with 3 heads (five
    tokens per item) ends on a partial item and runs items across sample boundaries."""
    rng = np.random.default_rng(H * 100 + grid[1])
    B = 2
    S = grid[0] * grid[1] * grid[2]
    dt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[in_dtype]
    x = [torch.from_numpy(rng.standard_normal((B, S, H, 128), dtype=np.float32)).to(dt)
         for _ in range(3)]
    vals = [t.float().numpy() for t in x]  # the values the kernels read
    qw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    fr = O.rope_freqs_3d(*grid)
    dense = [t.cuda() for t in x]
    head_major = [t.permute(0, 2, 1, 3).contiguous().cuda().permute(0, 2, 1, 3) for t in x]
    if H > 1:  # one head: torch gives the size-1 head axis stride 128
        assert head_major[0].stride(2) == S * 128 and dense[0].stride(2) == 128
    a = aa.prologue(*dense, _dev(qw), _dev(kw), _dev(fr), op_dtype=torch.bfloat16)
    b = aa.prologue(*head_major, _dev(qw), _dev(kw), _dev(fr), op_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert aa.status() == 0
    for u, w in zip(a, b):
        assert torch.equal(u, w)
    rq, rk, rv = O.prologue(*vals, qw, kw, fr)
    for got, ref in zip(a, (rq, rk, rv)):
        g = got.float().cpu().numpy().reshape(ref.shape)
        # bf16 rounding of the fp32 oracle value: |err| <= 2^-8 |x| (+ tree-sum ulps)
        assert np.all(np.abs(g - ref) <= np.abs(ref) * 2.0 ** -7 + 1e-6)


def test_masked_cross_attention(aa, O):
    rng = np.random.default_rng(21)
    B, H, Sq, Skv = 6, 2, 200, 512
    q = rng.standard_normal((B, H, Sq, 128), dtype=np.float32)
    k = rng.standard_normal((B, H, Skv, 128), dtype=np.float32)
    v = rng.standard_normal((B, H, Skv, 128), dtype=np.float32)
    valid = np.array([0, 1, 77, 128, 129, 512], dtype=np.int32)
    ref = O.sdpa_varlen(q, k, v, valid, threads=4)
    qh, kh, vh = (_dev(t).reshape(B * H, -1, 128).to(torch.bfloat16) for t in (q, k, v))
    out = aa.attention_core(qh, kh, vh, B, H, kv_valid_len=_dev(valid), out_layout="bhsd")
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert not got[0].any()  # zero valid keys -> zero output, like the oracle
    _ok(got, ref)


def test_masked_persistent_whole_units_match_unit_mode_and_oracle(aa, O):
    """Masked calls of more than one wave of short units run persistent whole units: here
    6 x 16 heads x 4 units of 250 rows against 512 keys (384 units on 148 SMs), valid
    lengths 0 (zero output), 1, 77, 128, 129 and 512 -- units of 0 to 4 key tiles dealt
    round-robin -- against one CTA per unit and the oracle."""
    from anima_attn import _lib as L
    rng = np.random.default_rng(23)
    B, H, Sq, Skv = 6, 16, 1000, 512
    assert L.lib.anima_attn_schedule(B, H, Sq, Skv, L.FLAG_MASK, 0) == L.SCHED_WHOLE
    q = rng.standard_normal((B, H, Sq, 128), dtype=np.float32)
    k = rng.standard_normal((B, H, Skv, 128), dtype=np.float32)
    v = rng.standard_normal((B, H, Skv, 128), dtype=np.float32)
    valid = np.array([0, 1, 77, 128, 129, 512], dtype=np.int32)
    qh, kh, vh = (_dev(t).reshape(B * H, -1, 128).to(torch.bfloat16) for t in (q, k, v))
    dvalid = _dev(valid)
    got = aa.attention_core(qh, kh, vh, B, H, kv_valid_len=dvalid, out_layout="bhsd")
    one = aa.attention_core(qh, kh, vh, B, H, kv_valid_len=dvalid, out_layout="bhsd",
                            schedule="unit")
    torch.cuda.synchronize()
    assert aa.status() == 0
    g = got.cpu().numpy()
    assert not g[0].any()
    assert np.array_equal(g, one.cpu().numpy())  # same tiles in the same order per row
    ref = O.sdpa_varlen(q, k, v, valid, threads=16)
    _ok(g, ref)


@pytest.mark.parametrize("Sq,Skv", [(1300, 700), (4000, 3000), (1280, 128), (4096, 4096)])
def test_schedules_match_each_other_and_oracle(aa, O, Sq, Skv):
    """More than one wave of 256-row units (B*H*ceil(Sq/256) > 148 SMs) in all three
    schedules: one CTA per unit (ANIMA_FLAG_UNIT), the persistent grid of whole units
    (ANIMA_FLAG_WHOLE; its last round leaves CTAs idle), and the persistent grid with the
    last round cut into key-tile slices merged in-kernel (ANIMA_FLAG_SPLIT).  Ragged Sq/Skv
    exercise partial query units and partial key tiles; (1280, 128) has one-tile units
    (nothing to cut); (4096, 4096) is the bench shape, whose 68 last-round units are each
    cut across about three CTAs."""
    from anima_attn import _lib as L
    B, H = 2, 16
    rng = np.random.default_rng(Sq + Skv)
    q = rng.standard_normal((B * H, Sq, 128), dtype=np.float32)
    k = rng.standard_normal((B * H, Skv, 128), dtype=np.float32)
    v = rng.standard_normal((B * H, Skv, 128), dtype=np.float32)
    assert L.lib.anima_attn_workspace_size(B, H, Sq, Skv, L.FLAG_SPLIT) > 0
    qh, kh, vh = (_dev(t).to(torch.bfloat16) for t in (q, k, v))
    split = aa.attention_core(qh, kh, vh, B, H, out_layout="bhsd", schedule="split")
    unit = aa.attention_core(qh, kh, vh, B, H, out_layout="bhsd", schedule="unit")
    whole = aa.attention_core(qh, kh, vh, B, H, out_layout="bhsd", schedule="whole")
    torch.cuda.synchronize()
    assert aa.status() == 0
    s_np, u_np = split.cpu().numpy(), unit.cpu().numpy()
    # Whole units compute exactly what one CTA per unit computes.
    assert np.array_equal(whole.cpu().numpy(), u_np)
    rows = np.sort(rng.choice(Sq, size=min(Sq, 160), replace=False))
    ref = O.sdpa(q[:, rows], k, v, threads=8).reshape(B, H, len(rows), 128)
    # Each schedule rounds P to bf16 relative to the running max its CTA saw, so the two
    # differ at the bf16 level; both must meet the bar against the fp32 oracle.
    _ok(s_np[:, :, rows], ref)
    _ok(u_np[:, :, rows], ref)
    assert rel_l2(s_np, u_np) < ATTN_REL_L2


@pytest.mark.parametrize("B,H,Sq,Skv,out", [(2, 2, 4096, 4096, "f32"), (1, 1, 1000, 3000, "f32"),
                                             (2, 2, 2048, 2048, "bf16"), (2, 1, 2500, 1300, "f16")])
def test_one_wave_cut_matches_unit_and_oracle(aa, O, B, H, Sq, Skv, out):
    """Calls of one wave of 256-row units that would leave most of the 148 SMs idle (a few
    heads per GPU, as the 8-GPU head split gives) run every unit cut into key-tile slices
    over all SMs, merged in-kernel; ANIMA_FLAG_UNIT keeps one CTA per unit.  Both against
    the oracle on sampled rows of every (b, h), and against each other.  Ragged shapes put a
    partial query unit and a partial key tile into slices that span two units."""
    from anima_attn import _lib as L
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    assert L.lib.anima_attn_schedule(B, H, Sq, Skv, 0, sm) == L.SCHED_CUT
    assert L.lib.anima_attn_schedule(B, H, Sq, Skv, L.FLAG_UNIT, sm) == L.SCHED_UNIT
    rng = np.random.default_rng(Sq * 7 + Skv + H)
    q = rng.standard_normal((B * H, Sq, 128), dtype=np.float32)
    k = rng.standard_normal((B * H, Skv, 128), dtype=np.float32)
    v = rng.standard_normal((B * H, Skv, 128), dtype=np.float32)
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[out]
    qh, kh, vh = (_dev(t).to(torch.bfloat16) for t in (q, k, v))
    for _ in range(2):  # the second call finds the arrival counters left at zero by the first
        cut = aa.attention_core(qh, kh, vh, B, H, out_layout="bhsd", out_dtype=tdt)
    unit = aa.attention_core(qh, kh, vh, B, H, out_layout="bhsd", out_dtype=tdt, schedule="unit")
    torch.cuda.synchronize()
    assert aa.status() == 0
    c_np, u_np = cut.float().cpu().numpy(), unit.float().cpu().numpy()
    rows = np.unique(np.concatenate([np.arange(0, 16), np.arange(Sq - 16, Sq),
                                     rng.choice(Sq, size=min(Sq, 96), replace=False)]))
    ref = O.sdpa(q[:, rows], k, v, threads=8).reshape(B, H, len(rows), 128)
    rel = ATTN_REL_L2 if out == "f32" else 8e-3  # 16-bit output adds its rounding
    _ok(c_np[:, :, rows], ref, rel=rel)
    _ok(u_np[:, :, rows], ref, rel=rel)
    assert rel_l2(c_np, u_np) < rel


KV64_CASES = [  # (B, H, Sq, Skv, causal, masked, schedule, out_dtype)
    (1, 1, 1, 1, False, False, "auto", "f32"), (1, 2, 7, 9, False, False, "auto", "f32"),
    (1, 2, 127, 65, False, False, "auto", "f32"), (2, 3, 300, 1000, False, False, "auto", "bf16"),
    (1, 2, 256, 256, True, False, "auto", "f32"), (1, 1, 200, 333, True, False, "auto", "f16"),
    (3, 2, 160, 200, False, True, "auto", "f32"),
    (2, 16, 1300, 700, False, False, "unit", "f32"), (2, 16, 1300, 700, False, False, "whole", "f32"),
    (2, 16, 1300, 700, False, False, "split", "f32"), (2, 16, 4096, 512, False, False, "auto", "f16"),
    (2, 16, 4096, 4096, False, False, "auto", "f32"), (2, 16, 1200, 777, False, False, "split", "bf16"),
]


@pytest.mark.parametrize("B,H,Sq,Skv,causal,masked,schedule,out_dtype", KV64_CASES)
def test_kv64_kernel_matches_oracle(aa, O, B, H, Sq, Skv, causal, masked, schedule, out_dtype):
    """The 64-key-tile kernel (ANIMA_FLAG_KV64: P in tensor-memory columns of its own, the
    next QK^T issued while the softmax runs): ragged and one-row shapes, causal and
    key-padding masks, the three schedules (the cut slices counted in 64-key tiles) and
    16-bit output, against the oracle on sampled rows and against the default kernel."""
    rng = np.random.default_rng(B * 7919 + Sq * 31 + Skv)
    q = rng.standard_normal((B * H, Sq, 128), dtype=np.float32)
    k = rng.standard_normal((B * H, Skv, 128), dtype=np.float32)
    v = rng.standard_normal((B * H, Skv, 128), dtype=np.float32)
    valid = rng.integers(1, Skv + 1, size=B).astype(np.int32) if masked else None
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[out_dtype]
    qh, kh, vh = (_dev(t).to(torch.bfloat16) for t in (q, k, v))
    kw = dict(out_layout="bhsd", out_dtype=tdt, causal=causal, schedule=schedule,
              kv_valid_len=None if valid is None else _dev(valid))
    got = aa.attention_core(qh, kh, vh, B, H, kv64=True, **kw)
    base = aa.attention_core(qh, kh, vh, B, H, **kw)
    torch.cuda.synchronize()
    assert aa.status() == 0
    g_np, b_np = got.float().cpu().numpy(), base.float().cpu().numpy()
    rows = np.unique(np.concatenate([np.arange(min(Sq, 48)), np.arange(max(0, Sq - 48), Sq),
                                     rng.choice(Sq, size=min(Sq, 64), replace=False)]))
    qr, kr, vr = (t.reshape(B, H, -1, 128) for t in (q, k, v))
    if masked:
        ref = O.sdpa_varlen(qr, kr, vr, valid)[:, :, rows]
    elif causal:
        ref = O.sdpa(qr, kr, vr, causal=True)[:, :, rows]
    else:
        ref = O.sdpa(q[:, rows], k, v, threads=8).reshape(B, H, len(rows), 128)
    tol = ATTN_REL_L2 if out_dtype == "f32" else 8e-3
    _ok(g_np[:, :, rows], ref, rel=tol)
    assert rel_l2(g_np, b_np) < tol


@pytest.mark.parametrize("out_dtype", ["bf16", "f16"])
def test_split_schedule_16bit_strided_output(aa, O, out_dtype):
    """Split schedule writing 16-bit output into a token-major [B, S, H, D] tensor (row
    stride H*D): the epilogue's staged block stores and the merge of cut units both write
    through it.  S_q = 1200 leaves the last unit's last warps with 16 and 0 valid rows, and
    S_kv = 777 a partial key tile."""
    from anima_attn import _lib as L
    B, H, Sq, Skv = 2, 16, 1200, 777
    rng = np.random.default_rng(11)
    q = rng.standard_normal((B * H, Sq, 128), dtype=np.float32)
    k = rng.standard_normal((B * H, Skv, 128), dtype=np.float32)
    v = rng.standard_normal((B * H, Skv, 128), dtype=np.float32)
    assert L.lib.anima_attn_workspace_size(B, H, Sq, Skv, L.FLAG_SPLIT) > 0
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16}[out_dtype]
    qh, kh, vh = (_dev(t).to(torch.bfloat16) for t in (q, k, v))
    split = aa.attention_core(qh, kh, vh, B, H, out_dtype=tdt, schedule="split")
    unit = aa.attention_core(qh, kh, vh, B, H, out_dtype=tdt, schedule="unit")
    torch.cuda.synchronize()
    assert aa.status() == 0
    s_np = split.float().cpu().numpy().transpose(0, 2, 1, 3)  # -> [B, H, S, D]
    u_np = unit.float().cpu().numpy().transpose(0, 2, 1, 3)
    rows = np.concatenate([np.arange(0, 40), np.arange(1140, 1200)])
    ref = O.sdpa(q[:, rows], k, v, threads=8).reshape(B, H, len(rows), 128)
    _ok(s_np[:, :, rows], ref, rel=8e-3)  # 16-bit output adds its rounding
    _ok(u_np[:, :, rows], ref, rel=8e-3)
    assert rel_l2(s_np, u_np) < 8e-3


# ------------------------------------------------------------------ benchmark configurations
def test_config1_self_attention_256(aa, O):
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((2, 16, 256, 128), dtype=np.float32) for _ in range(3))
    ref = O.sdpa(q, k, v, threads=8)
    got = aa.sdpa(_dev(q), _dev(k), _dev(v))
    torch.cuda.synchronize()
    _ok(got.cpu().numpy(), ref)


def test_config2_prologue_self_attention_1024(aa, O):
    rng = np.random.default_rng(1)
    B, S, H = 2, 1024, 16
    q, k, v = (rng.standard_normal((B, S, H, 128), dtype=np.float32) for _ in range(3))
    qw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    fr = O.rope_freqs_3d(1, 32, 32)
    out = aa.attention(_dev(q), _dev(k), _dev(v), _dev(qw), _dev(kw), _dev(fr))
    torch.cuda.synchronize()
    rq, rk, rv = O.prologue(q, k, v, qw, kw, fr)
    ref = O.sdpa(rq, rk, rv, threads=8)
    _ok(out.cpu().numpy().transpose(0, 2, 1, 3), ref)


def test_config3_masked_cross_attention(aa, O):
    rng = np.random.default_rng(2)
    B, Sq, Skv, H = 2, 4096, 512, 16
    q = rng.standard_normal((B, Sq, H, 128), dtype=np.float32)
    ctx = rng.standard_normal((B, Skv, 1024), dtype=np.float32)
    wk = (0.02 * rng.standard_normal((2048, 1024))).astype(np.float32)
    wv = (0.02 * rng.standard_normal((2048, 1024))).astype(np.float32)
    wk = torch.from_numpy(wk).bfloat16().float().numpy()
    wv = torch.from_numpy(wv).bfloat16().float().numpy()
    k = (ctx @ wk.T).reshape(B, Skv, H, 128).astype(np.float32)
    v = (ctx @ wv.T).reshape(B, Skv, H, 128).astype(np.float32)
    qw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    valid = rng.integers(32, 513, size=B).astype(np.int32)
    out = aa.attention(_dev(q), _dev(k), _dev(v), _dev(qw), None, None,
                       kv_valid_len=_dev(valid), norm_k=False)
    torch.cuda.synchronize()
    rq, rk, rv = O.prologue(q, k, v, qw, None)
    ref = O.sdpa_varlen(rq, rk, rv, valid, threads=8)
    _ok(out.cpu().numpy().transpose(0, 2, 1, 3), ref)


@pytest.mark.parametrize("L", [4096, 9216, 16384])
def test_long_sequence_rows_and_properties(aa, O, L):
    """Config 5 sizes (64x64, 96x96 and 128x128 latent grids): sampled query rows of every
    (batch, head) against all keys (rows are independent, so the sliced oracle is exact),
    plus size-independent properties of the full output."""
    side = int(np.sqrt(L))
    rng = np.random.default_rng(L)
    B, H = 2, 16
    q, k, v = (rng.standard_normal((B, L, H, 128), dtype=np.float32) for _ in range(3))
    qw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    fr = O.rope_freqs_3d(1, side, side)
    dq, dk, dv = _dev(q), _dev(k), _dev(v)
    out = aa.attention(dq, dk, dv, _dev(qw), _dev(kw), _dev(fr))
    torch.cuda.synchronize()
    got = out.cpu().numpy()  # [B, L, H, D]
    rq, rk, rv = O.prologue(q, k, v, qw, kw, fr)  # [B, H, L, D]
    # 24 rows of each of the 32 (b, h), a fresh sample per head, first and last rows included
    rows = np.stack([np.sort(np.concatenate([[0, L - 1], rng.choice(np.arange(1, L - 1), 22,
                                                                     replace=False)]))
                     for _ in range(B * H)])
    qs = np.stack([rq[bh // H, bh % H][rows[bh]] for bh in range(B * H)])  # [BH, 24, D]
    ref = O.sdpa(qs, rk.reshape(B * H, L, 128), rv.reshape(B * H, L, 128), threads=16)
    sel = np.stack([got[bh // H, rows[bh], bh % H] for bh in range(B * H)])
    _ok(sel, ref)
    # rows of softmax sum to one: V = 1 gives an all-ones output
    ones = torch.ones_like(dv)
    o1 = aa.attention(dq, dk, ones, _dev(qw), _dev(kw), _dev(fr))
    torch.cuda.synchronize()
    assert np.abs(o1.cpu().numpy() - 1.0).max() < 1e-2
    assert aa.status() == 0


def test_bounded_wait_reports_timeout_and_context_survives(aa, O):
    """Failure detection without a GPU fault: a wait on a flag nothing sets runs out
    after 20 ms, the status word reads ANIMA_ERR_TIMEOUT, and the next call works."""
    from anima_attn import _lib as L
    st = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.lib.anima_attn_status(st, 1) == 0
    assert L.lib.anima_attn_selftest_timeout(20000, st) == L.OK
    assert L.lib.anima_attn_status(st, 1) == L.ERR_TIMEOUT
    assert L.lib.anima_attn_status(st, 1) == 0  # cleared by the previous read
    assert L.lib.anima_attn_selftest_timeout(0, st) == L.ERR_ARG
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((1, 2, 200, 128), dtype=np.float32) for _ in range(3))
    got = aa.sdpa(_dev(q), _dev(k), _dev(v))
    torch.cuda.synchronize()
    _ok(got.cpu().numpy(), O.sdpa(q, k, v))
    assert aa.status() == 0


PAIR_SHAPES = [  # (B, H, Sq, Skv, causal, valid)
    (1, 1, 512, 128, False, None), (1, 2, 700, 300, False, None), (2, 3, 1000, 1000, False, None),
    (1, 2, 600, 600, True, None), (4, 2, 512, 512, False, [0, 5, 130, 512]),
    (1, 1, 1, 1, False, None),
]


@pytest.mark.parametrize("B,H,Sq,Skv,causal,valid", PAIR_SHAPES)
def test_cta_pair_kernel(aa, O, B, H, Sq, Skv, causal, valid):
    """The opt-in CTA-pair kernel (tcgen05.mma.cta_group::2, M = 256 over two SMs, each
    SM loading half of every K and V tile) against the oracle."""
    rng = np.random.default_rng(Sq * 7 + Skv)
    q = rng.standard_normal((B, H, Sq, 128), dtype=np.float32)
    k = rng.standard_normal((B, H, Skv, 128), dtype=np.float32)
    v = rng.standard_normal((B, H, Skv, 128), dtype=np.float32)
    qh, kh, vh = (_dev(t).reshape(B * H, -1, 128).to(torch.bfloat16) for t in (q, k, v))
    vl = None if valid is None else _dev(np.array(valid, np.int32))
    out = aa.attention_core(qh, kh, vh, B, H, kv_valid_len=vl, causal=causal, out_layout="bhsd",
                            pair=True)
    torch.cuda.synchronize()
    assert aa.status() == 0
    ref = (O.sdpa(q, k, v, causal=causal) if valid is None
           else O.sdpa_varlen(q, k, v, np.array(valid, np.int32)))
    _ok(out.cpu().numpy(), ref)


# ------------------------------------------------------------------ RoPE entry, predict2 patch
def test_apply_rope_device_entry_bit_exact(aa, O):
    """anima_attn_rope (predict2.apply_rotary_pos_emb on the device) against the restated
    reference RoPE: bit-exact on [B, S, H, D], on a strided head view and on [N, S, D]."""
    rng = np.random.default_rng(3)
    t = rng.standard_normal((2, 64, 6, 128), dtype=np.float32)
    fr = O.rope_freqs_3d(1, 8, 8)
    got = aa.apply_rope(_dev(t), _dev(fr))
    assert np.array_equal(got.cpu().numpy(), O.rope(t, fr))
    view = _dev(t)[:, :, ::2]  # heads 0, 2, 4: element strides (S*6*D, 6*D, 2*D)
    got = aa.apply_rope(view, _dev(fr))
    assert np.array_equal(got.cpu().numpy(), O.rope(np.ascontiguousarray(t[:, :, ::2]), fr))
    t3 = rng.standard_normal((5, 64, 128), dtype=np.float32)
    assert np.array_equal(aa.apply_rope(_dev(t3), _dev(fr)).cpu().numpy(), O.rope(t3, fr))
    tb = _dev(t).to(torch.bfloat16)  # computed in fp32, returned in t's dtype
    got = aa.apply_rope(tb, _dev(fr))
    assert got.dtype == torch.bfloat16
    ref = O.rope(tb.float().cpu().numpy(), fr)
    assert np.abs(got.float().cpu().numpy() - ref).max() <= 2 ** -7 * np.abs(ref).max()


def test_patched_predict2_attention_forward_on_gpu(aa):
    """The fused Attention.forward that patch_predict2 installs, with the library's GPU
    backend, on a module with predict2.Attention's attribute surface (the reference module
    itself is tested on CPU with stand-ins in tests/test_predict2_patch.py), for self- and
    cross-attention, against the same math in fp64 on the CPU."""
    import types
    import torch.nn as nn
    import torch.nn.functional as F
    from anima_attn import compat
    from dit_cpu_attention import rope as cpu_rope

    class Attention(nn.Module):  # predict2.Attention's fields (src/predict2.py:91-160)
        def __init__(self, dim, ctx_dim, heads, selfattn):
            super().__init__()
            self.n_heads, self.head_dim, self.is_selfattn = heads, 128, selfattn
            inner = heads * 128
            self.q_proj = nn.Linear(dim, inner, bias=False)
            self.k_proj = nn.Linear(ctx_dim, inner, bias=False)
            self.v_proj = nn.Linear(ctx_dim, inner, bias=False)
            self.q_norm, self.k_norm = nn.RMSNorm(128, eps=1e-6), nn.RMSNorm(128, eps=1e-6)
            self.output_proj = nn.Linear(inner, dim, bias=False)
            self.output_dropout = nn.Identity()

        def forward(self, *a, **kw):
            raise AssertionError("not patched")

    fake = types.SimpleNamespace(_scaled_dot_product_attention=None, apply_rotary_pos_emb=None,
                                 Attention=Attention)
    compat.patch_predict2(fake)
    torch.manual_seed(0)
    B, S, dim, H = 2, 144, 512, 4
    fr = torch.from_numpy(aa.rope_freqs_3d(1, 12, 12).cpu().numpy())
    for selfattn, Skv, cdim in ((True, S, dim), (False, 77, 256)):
        m = Attention(dim, cdim, H, selfattn)
        with torch.no_grad():
            for nrm in (m.q_norm, m.k_norm):
                nrm.weight.copy_(1 + 0.1 * torch.randn(128))
        x, ctx = torch.randn(B, S, dim), torch.randn(B, Skv, cdim)
        rope_emb = fr.reshape(1, S, 1, 64, 2, 2)  # predict2's broadcast shape
        with torch.no_grad():
            got = m.cuda()(x.cuda(), None if selfattn else ctx.cuda(), rope_emb=rope_emb.cuda())
            md = m.double().cpu()
            src = x.double() if selfattn else ctx.double()
            q = md.q_proj(x.double()).view(B, S, H, 128)
            k = md.k_proj(src).view(B, -1, H, 128)
            v = md.v_proj(src).view(B, -1, H, 128)
            q = F.rms_norm(q, (128,), md.q_norm.weight, 1e-6)
            k = F.rms_norm(k, (128,), md.k_norm.weight, 1e-6)
            if selfattn:
                q, k = cpu_rope(q, fr.double()).double(), cpu_rope(k, fr.double()).double()
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
            ref = md.output_proj(o.transpose(1, 2).reshape(B, S, H * 128))
        _ok(got.double().cpu().numpy(), ref.numpy())
