"""Anima DiT weights in the reference's on-disk format, loaded straight to the device.

The reference ships the diffusion model as one safetensors file of bf16 tensors and reads
it in two ways: a header parser over an mmap (SafetensorsReader,
anima_rt/scripts/phone_pipeline_anima_rt.py:99-125, which also strips a leading key prefix
such as "net.", lines 130-141) and safetensors.torch.load_file followed by dropping the
"net." prefix (scripts/pc_compare_dit_err.py:131-135).  Both produce MiniTrainDIT
state-dict keys, the names anima_attn.dit.weight_spec lists.

The format: an 8-byte little-endian header length, a JSON header mapping each tensor name
to {"dtype", "shape", "data_offsets": [begin, end]} (offsets relative to the end of the
header; an optional "__metadata__" entry), then the raw little-endian tensor bytes.

load_dit_weights reads only the tensors the DiT step uses, in file order, through two
page-locked staging buffers: the file read of one chunk overlaps the host-to-device copy of
the previous one, and the tensors land in device memory in their stored type (bf16 stays
bf16, bit for bit).  Norm weights are returned as fp32 (exact for bf16/f16 values, as the
reference's bit-widening at phone_pipeline_anima_rt.py:160-168).
"""
from __future__ import annotations

import json
import os
import struct
from typing import Callable, Dict, Iterable, Optional, Tuple

import torch

from .dit import DiTConfig, weight_spec

_DTYPES = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}
_NAMES = {v: k for k, v in _DTYPES.items()}
# First name components of MiniTrainDIT's own keys; anything else in front is a prefix
# (phone_pipeline_anima_rt.py:133-137).
_ROOTS = ("blocks", "x_embedder", "t_embedder", "final_layer", "t_embedding_norm",
          "pos_embedder", "extra_pos_embedder", "llm_adapter")


def read_header(path: str) -> Tuple[Dict[str, dict], int]:
    """(header without "__metadata__", byte offset of the data section)."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file (shorter than 8 bytes)")
        (n,) = struct.unpack("<Q", raw)
        size = os.fstat(f.fileno()).st_size
        if n > size - 8:
            raise ValueError(f"{path}: header length {n} exceeds the file")
        header = json.loads(f.read(n).decode("utf-8"))
    header.pop("__metadata__", None)
    data_len = size - 8 - n
    for k, info in header.items():
        b, e = info["data_offsets"]
        if info["dtype"] not in _DTYPES:
            raise ValueError(f"{path}: tensor {k!r} has unsupported dtype {info['dtype']}")
        count = 1
        for d in info["shape"]:
            count *= d
        if not (0 <= b <= e <= data_len) or e - b != count * _DTYPES[info["dtype"]].itemsize:
            raise ValueError(f"{path}: tensor {k!r} has inconsistent data_offsets {b}..{e}")
    return header, 8 + n


def detect_prefix(keys: Iterable[str]) -> str:
    """The key prefix in front of MiniTrainDIT's names ("" or e.g. "net.")."""
    for k in keys:
        head = k.split(".", 1)[0]
        return "" if head in _ROOTS or "." not in k else head + "."
    return ""


class _Staging:
    """Two page-locked buffers; chunk k's host->device copy overlaps chunk k+1's read."""

    def __init__(self, nbytes: int, device: torch.device):
        self.bufs = [torch.empty(nbytes, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        self.events = [None, None]
        self.stream = torch.cuda.Stream(device=device)
        self.k = 0

    def copy(self, f, nbytes: int, dst: torch.Tensor) -> None:
        """Reads nbytes at f's position into the flat uint8 device tensor dst."""
        off, cap = 0, self.bufs[0].numel()
        while off < nbytes:
            n = min(cap, nbytes - off)
            buf, ev = self.bufs[self.k], self.events[self.k]
            if ev is not None:
                ev.synchronize()  # the copy that last used this buffer is done
            got = f.readinto(memoryview(buf.numpy())[:n])
            if got != n:
                raise IOError(f"short read: {got} of {n} bytes")
            with torch.cuda.stream(self.stream):
                dst[off:off + n].copy_(buf[:n], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.stream)
            self.events[self.k] = ev
            self.k ^= 1
            off += n

    def finish(self) -> None:
        self.stream.synchronize()


def load_dit_weights(path: str, cfg: Optional[DiTConfig] = None, device="cuda",
                     keep: Optional[Callable[[str], bool]] = None,
                     chunk_bytes: int = 64 << 20) -> Dict[str, torch.Tensor]:
    """The DiT step's weights from a safetensors checkpoint, as anima_attn.dit.AnimaDiT
    takes them: Linear weights in their stored 16-bit type (fp32 ones become bf16), norm
    weights fp32.  ``keep`` filters names (a rank may skip weights it never uses).

    Raises KeyError for a missing tensor and ValueError for a shape that does not match
    ``cfg`` (default DiTConfig(), the 2B model)."""
    cfg = cfg or DiTConfig()
    device = torch.device(device)
    header, start = read_header(path)
    prefix = detect_prefix(header.keys())
    want = [(n, s, kind) for n, s, kind in weight_spec(cfg) if keep is None or keep(n)]
    missing = [n for n, _, _ in want if prefix + n not in header]
    if missing:
        raise KeyError(f"{path}: {len(missing)} DiT tensors missing, e.g. {missing[:3]}")
    for n, shape, _ in want:
        got = tuple(header[prefix + n]["shape"])
        if got != tuple(shape):
            raise ValueError(f"{path}: {n} has shape {got}, the config needs {tuple(shape)}")
    want.sort(key=lambda t: header[prefix + t[0]]["data_offsets"][0])  # file order
    staging = _Staging(chunk_bytes, device) if device.type == "cuda" else None
    out: Dict[str, torch.Tensor] = {}
    with open(path, "rb", buffering=0) as f:
        for n, shape, kind in want:
            info = header[prefix + n]
            b, e = info["data_offsets"]
            t = torch.empty(tuple(shape), dtype=_DTYPES[info["dtype"]], device=device)
            flat = t.view(-1).view(torch.uint8)
            f.seek(start + b)
            if staging is not None:
                staging.copy(f, e - b, flat)
            else:
                got = f.readinto(memoryview(flat.numpy()))
                if got != e - b:
                    raise IOError(f"{path}: short read of {n}")
            out[n] = t
        if staging is not None:
            staging.finish()
    for n, _, kind in want:
        t = out[n]
        if kind == "one":
            out[n] = t.float()
        elif t.dtype == torch.float32:
            out[n] = t.to(torch.bfloat16)
    return out


def save_weights(path: str, weights: Dict[str, torch.Tensor], prefix: str = "",
                 metadata: Optional[Dict[str, str]] = None) -> None:
    """Writes ``weights`` (any device) as a safetensors file, names prefixed by ``prefix``
    (the released checkpoint uses "net.").  Tensors are laid out in name order with the
    header padded to 8 bytes."""
    names = sorted(weights)
    header: Dict[str, dict] = {}
    off = 0
    for n in names:
        t = weights[n]
        if t.dtype not in _NAMES:
            raise ValueError(f"{n}: dtype {t.dtype} not representable")
        nb = t.numel() * t.element_size()
        header[prefix + n] = {"dtype": _NAMES[t.dtype], "shape": list(t.shape),
                              "data_offsets": [off, off + nb]}
        off += nb
    if metadata:
        header["__metadata__"] = dict(metadata)
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hb += b" " * ((-len(hb)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for n in names:
            t = weights[n].detach().contiguous().cpu()
            f.write(t.view(-1).view(torch.uint8).numpy().tobytes())
