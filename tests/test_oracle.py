"""The CPU oracle, pinned against the reference (CPU only).

The golden fixtures were produced by the reference's own code (tests/golden/
make_golden.py); the restatement in oracle/anima_oracle.c must reproduce them exactly.
When the reference library was compiled here (oracle/_ref), it is compared directly too.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden, max_abs
from oracle import oracle as O


@pytest.fixture(scope="module", autouse=True)
def _built():
    O.build(ref=O.REF_TREE is not None)


@pytest.mark.parametrize("name", ["sdpa_square.npz", "sdpa_ragged.npz", "sdpa_causal.npz",
                                  "sdpa_cross.npz"])
def test_sdpa_matches_reference_fixture_bit_exact(name):
    g = golden(name)
    out = O.sdpa(g["q"], g["k"], g["v"], causal=bool(g["causal"]))
    assert np.array_equal(out, g["out"])


def test_rmsnorm_matches_reference_fixture_bit_exact():
    g = golden("rmsnorm.npz")
    assert np.array_equal(O.rmsnorm(g["x"], g["w"]), g["out_w"])
    assert np.array_equal(O.rmsnorm(g["x"], None), g["out_nw"])


def test_rope_matches_reference_fixture():
    g = golden("rope.npz")
    # anima_rt_run_rope restated: bit-exact
    assert np.array_equal(O.rope(g["t"], g["freqs"]), g["out_anima_rt"])
    # predict2.apply_rotary_pos_emb (torch) agrees to fp32 rounding
    assert max_abs(g["out_anima_rt"], g["out_predict2"]) < 1e-5
    # the numpy restatement of numpy_dit._numpy_rope (the CPU prologue baseline)
    assert np.array_equal(O.numpy_rope(g["t"], g["freqs"]), g["out_anima_rt"])
    assert max_abs(O.numpy_rope(g["t"], g["freqs"]), g["out_predict2"]) < 1e-5


def test_rope_table_matches_video_rope_3d():
    g = golden("rope.npz")
    assert max_abs(O.rope_freqs_3d(1, 16, 16), g["freqs"]) < 1e-6


def test_product_rope_table_matches_reference_fixture():
    import torch
    from anima_attn.rope import rope_freqs_3d
    g = golden("rope.npz")
    t = rope_freqs_3d(1, 16, 16, device="cpu").numpy()
    assert t.shape == g["freqs"].shape
    assert max_abs(t, g["freqs"]) < 1e-6


def test_prologue_composition_fixture():
    g = golden("prologue_sdpa.npz")
    qh, kh, vh = O.prologue(g["q"], g["k"], g["v"], g["q_w"], g["k_w"], g["freqs"])
    assert np.array_equal(qh, g["q_ready"]) and np.array_equal(kh, g["k_ready"])
    assert np.array_equal(O.sdpa(qh, kh, vh), g["out"])


def test_reference_known_answer_checksums():
    """scripts/archive/_verify_flash.py: seed-42 randn [2,16,256,128]."""
    import torch
    with open(os.path.join(GOLDEN, "verify_flash.json")) as f:
        ref = json.load(f)
    torch.manual_seed(42)
    q, k, v = (torch.randn(*ref["shape"]).numpy() for _ in range(3))
    out = O.sdpa(q, k, v, threads=8).astype(np.float64)
    assert abs(out.sum() - ref["ref_sum"]) < 1e-6 * ref["ref_abs_sum"]
    assert abs(np.sqrt((out ** 2).sum()) - ref["ref_l2"]) < 1e-9 * ref["ref_l2"] * 1e3
    assert np.allclose(out.reshape(-1)[:8], ref["ref_first8"], rtol=0, atol=0)
    assert ref["max_err_vs_torch_sdpa"] < 2e-6


def test_varlen_equals_per_sample_reference_calls():
    rng = np.random.default_rng(3)
    B, H, Sq, Skv, D = 2, 2, 40, 90, 128
    q = rng.standard_normal((B, H, Sq, D), dtype=np.float32)
    k = rng.standard_normal((B, H, Skv, D), dtype=np.float32)
    v = rng.standard_normal((B, H, Skv, D), dtype=np.float32)
    valid = np.array([33, 90], dtype=np.int32)
    out = O.sdpa_varlen(q, k, v, valid, threads=2)
    for b in range(B):
        n = valid[b]
        ref = O.sdpa(q[b], k[b][:, :n], v[b][:, :n])
        assert np.array_equal(out[b], ref)
    zero = O.sdpa_varlen(q, k, v, np.array([0, 5], np.int32))
    assert not zero[0].any()


@pytest.mark.skipif(not O.have_reference(), reason="reference library not compiled here")
def test_port_is_bit_exact_with_compiled_reference():
    rng = np.random.default_rng(11)
    for (bh, sq, skv, causal) in [(2, 300, 700, False), (1, 129, 129, True), (3, 33, 65, False)]:
        q = rng.standard_normal((bh, sq, 128), dtype=np.float32)
        k = rng.standard_normal((bh, skv, 128), dtype=np.float32)
        v = rng.standard_normal((bh, skv, 128), dtype=np.float32)
        a = O.sdpa(q, k, v, causal=causal, kind="port")
        b = O.sdpa(q, k, v, causal=causal, kind="reference")
        assert np.array_equal(a, b)
    x = rng.standard_normal((50, 2048), dtype=np.float32)
    w = rng.standard_normal(2048, dtype=np.float32)
    assert np.array_equal(O.rmsnorm(x, w, kind="port"), O.rmsnorm(x, w, kind="reference"))
