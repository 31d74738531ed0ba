"""DiT weights in the reference's safetensors format (anima_attn.checkpoint).

The reference reads its diffusion checkpoint with its own header parser
(anima_rt/scripts/phone_pipeline_anima_rt.py:99-141, prefix detection included) or with
safetensors.torch.load_file (scripts/pc_compare_dit_err.py:131-135).  These tests write
small checkpoints of the DiT's parameter names and check that the loader returns them bit
for bit, on the host and through the pinned double-buffered path to the GPU, and that its
files and the safetensors package's files read the same both ways."""
import struct

import pytest
import torch

from anima_attn.checkpoint import detect_prefix, load_dit_weights, read_header, save_weights
from anima_attn.dit import DiTConfig, make_weights, weight_spec

CFG = DiTConfig(hidden=256, heads=2, blocks=2, adaln_lora=32, ctx_dim=64)


def _same(a, b):
    assert a.dtype == b.dtype and a.shape == b.shape
    assert torch.equal(a.view(-1).view(torch.uint8).cpu(), b.view(-1).view(torch.uint8).cpu())


def _check(loaded, ref):
    assert set(loaded) == set(ref)
    for n, t in ref.items():
        _same(loaded[n], t)


@pytest.fixture
def weights():
    return make_weights(CFG, seed=3)


def test_round_trip_with_prefix_and_extra_keys(tmp_path, weights):
    stored = {n: (t.to(torch.bfloat16) if t.dtype == torch.float32 else t) for n, t in weights.items()}
    stored["pos_embedder.seq"] = torch.arange(7, dtype=torch.float32)
    stored["llm_adapter.proj.weight"] = torch.randn(3, 5).to(torch.bfloat16)
    path = str(tmp_path / "dit.safetensors")
    save_weights(path, stored, prefix="net.", metadata={"format": "pt"})
    header, start = read_header(path)
    assert detect_prefix(header.keys()) == "net."
    assert start % 8 == 0
    got = load_dit_weights(path, CFG, device="cpu")
    assert set(got) == {n for n, _, _ in weight_spec(CFG)}
    for n, _, kind in weight_spec(CFG):
        if kind == "one":
            assert got[n].dtype == torch.float32
            _same(got[n], stored[n].float())
        else:
            _same(got[n], stored[n])


def test_no_prefix_and_keep_filter(tmp_path, weights):
    path = str(tmp_path / "dit.safetensors")
    save_weights(path, weights)
    keep = lambda n: n.startswith("blocks.1.")
    got = load_dit_weights(path, CFG, device="cpu", keep=keep)
    _check(got, {n: t for n, t in weights.items() if keep(n)})


def test_fp32_linear_weights_become_bf16(tmp_path, weights):
    path = str(tmp_path / "dit.safetensors")
    save_weights(path, {n: t.float() for n, t in weights.items()})
    got = load_dit_weights(path, CFG, device="cpu")
    _check(got, weights)  # the stored fp32 values are bf16 values, so this is exact


def test_errors(tmp_path, weights):
    path = str(tmp_path / "dit.safetensors")
    w = dict(weights)
    del w["blocks.0.mlp.layer1.weight"]
    save_weights(path, w)
    with pytest.raises(KeyError, match="missing"):
        load_dit_weights(path, CFG, device="cpu")
    w = dict(weights)
    w["blocks.0.mlp.layer1.weight"] = w["blocks.0.mlp.layer1.weight"][:-1].contiguous()
    save_weights(path, w)
    with pytest.raises(ValueError, match="shape"):
        load_dit_weights(path, CFG, device="cpu")
    save_weights(path, weights)
    data = open(path, "rb").read()
    open(path, "wb").write(data[:-2])  # truncated data section
    with pytest.raises(ValueError, match="data_offsets"):
        read_header(path)
    open(path, "wb").write(struct.pack("<Q", 1 << 40))
    with pytest.raises(ValueError, match="header length"):
        read_header(path)


def test_interoperates_with_safetensors_package(tmp_path, weights):
    st = pytest.importorskip("safetensors.torch")
    ours = str(tmp_path / "ours.safetensors")
    save_weights(ours, weights, prefix="net.")
    theirs = st.load_file(ours)
    _check({k[len("net."):]: v for k, v in theirs.items()}, weights)
    path = str(tmp_path / "theirs.safetensors")
    st.save_file({"net." + n: t for n, t in weights.items()}, path)
    _check(load_dit_weights(path, CFG, device="cpu"), weights)


@pytest.mark.gpu
def test_load_to_device_through_pinned_chunks(tmp_path, weights):
    path = str(tmp_path / "dit.safetensors")
    save_weights(path, weights, prefix="net.")
    # 4 KiB chunks: most tensors take several, so both staging buffers are reused.
    got = load_dit_weights(path, CFG, device="cuda", chunk_bytes=4096)
    assert all(t.is_cuda for t in got.values())
    _check(got, weights)
