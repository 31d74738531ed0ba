"""Reference-facing drop-ins: the Python call sites of the reference, backed by B200.

Each name here mirrors a reference binding with the same arguments and return layout,
so the reference's pipelines and tests switch by changing one import:

  NumpyRT            scripts/phone_pipeline_nd.py:46-68 (run_rmsnorm, run_sdpa), plus
                     run_attention: NumpyAttention.forward's norm/RoPE/SDPA in one call
  anima_rt_sdpa      anima_rt/scripts/anima_rt_ops.py:89-111
  anima_rt_rope      anima_rt/scripts/anima_rt_ops.py:127-143
  AnimaRTRMSNorm     anima_rt/scripts/anima_rt_ops.py:57-72
  patch_predict2     the monkeypatch points used by
                     anima_rt/scripts/phone_pipeline_anima_rt.py:224-252
                     (_scaled_dot_product_attention, apply_rotary_pos_emb) and a fused
                     Attention.forward (src/predict2.py:167-214)

Where the reference falls back to torch on a false return (anima_rt_ops.py:108-109),
these raise AnimaError: the B200 path never silently degrades to a CPU computation.
"""
from __future__ import annotations

import ctypes as ct
import math

import numpy as np
import torch
import torch.nn as nn

from . import _lib as L
from . import ops


def _f32c(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _fail(what: str):
    raise L.AnimaError(f"{what} failed: {L.last_error()}")


def _ensure_init():
    if not L.lib.anima_rt_init():
        _fail("anima_rt_init")


class NumpyRT:
    """numpy front end with the interface of the reference's NumpyRT.

    ``nw`` maps '<prefix>.q_norm.weight' etc. to fp32 arrays, as in the reference.
    """

    def __init__(self, nw: dict):
        _ensure_init()
        self._nw = nw

    def _kw(self, k):
        w = self._nw.get(k)
        return _f32c(w) if w is not None else None

    def run_rmsnorm(self, x, key):
        *b, D = x.shape
        M = int(np.prod(b)) if b else 1
        xf = _f32c(x.reshape(M, D))
        w = self._kw(key + ".weight")
        o = np.zeros((M, D), dtype=np.float32)
        if not L.lib.anima_rt_run_rmsnorm(xf.ctypes.data, None if w is None else w.ctypes.data,
                                          o.ctypes.data, M, D, ct.c_float(1e-6)):
            _fail("anima_rt_run_rmsnorm")
        return o.reshape(*b, D)

    def run_sdpa(self, q, k, v):
        B, H, Sq, D = q.shape
        Skv = k.shape[2]
        qf = _f32c(q.reshape(B * H, Sq, D))
        kf = _f32c(k.reshape(B * H, Skv, D))
        vf = _f32c(v.reshape(B * H, Skv, D))
        o = np.zeros((B * H, Sq, D), dtype=np.float32)
        s = 1.0 / np.sqrt(D)
        if not L.lib.anima_rt_run_sdpa_flash(qf.ctypes.data, kf.ctypes.data, vf.ctypes.data,
                                             o.ctypes.data, B * H, Sq, Skv, D, ct.c_float(s),
                                             ct.c_bool(False)):
            _fail("anima_rt_run_sdpa_flash")
        return o.reshape(B, H, Sq, D)

    def run_attention(self, q, k, v, prefix, rope_emb=None, kv_valid=None):
        """q [B,S,H,D], k/v [B,S_kv,H,D] projections -> [B,S,H,D] attention output:
        q/k RMSNorm with '<prefix>.q_norm' / '.k_norm', RoPE when ``rope_emb`` is given
        (self-attention), SDPA; the body of NumpyAttention.forward (numpy_dit.py:285-294)
        between its projection and o-proj GEMMs."""
        B, Sq, H, D = q.shape
        Skv = k.shape[1]
        qf, kf, vf = _f32c(q), _f32c(k), _f32c(v)
        qw, kw = self._kw(prefix + ".q_norm.weight"), self._kw(prefix + ".k_norm.weight")
        fr = None if rope_emb is None else _f32c(rope_emb).reshape(-1)
        vl = None if kv_valid is None else np.ascontiguousarray(kv_valid, dtype=np.int32)
        flags = L.FLAG_QNORM | L.FLAG_KNORM | (L.FLAG_ROPE if fr is not None else 0)
        o = np.zeros((B, Sq, H, D), dtype=np.float32)
        ptr = lambda a: None if a is None else a.ctypes.data
        if not L.lib.anima_rt_run_attention(ptr(qf), ptr(kf), ptr(vf), ptr(qw), ptr(kw), ptr(fr),
                                            ptr(vl), ptr(o), B, Sq, Skv, H, D, ct.c_float(1e-6),
                                            ct.c_float(1.0 / math.sqrt(D)), flags):
            _fail("anima_rt_run_attention")
        return o


def anima_rt_sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """F.scaled_dot_product_attention replacement on [B, H, S, D]; returns [B, H, S_q, D]
    on q's device and dtype.  CUDA tensors stay on the device; CPU tensors go through the
    host-pointer ABI (anima_rt_run_sdpa_flash)."""
    if q.is_cuda:
        return ops.sdpa(q, k, v)
    B, H, Sq, D = q.shape
    Skv = k.shape[2]
    qf = _f32c(q.reshape(B * H, Sq, D).float().numpy())
    kf = _f32c(k.reshape(B * H, Skv, D).float().numpy())
    vf = _f32c(v.reshape(B * H, Skv, D).float().numpy())
    out = np.zeros((B * H, Sq, D), dtype=np.float32)
    if not L.lib.anima_rt_run_sdpa_flash(qf.ctypes.data, kf.ctypes.data, vf.ctypes.data,
                                         out.ctypes.data, B * H, Sq, Skv, D,
                                         ct.c_float(1.0 / np.sqrt(D)), ct.c_bool(False)):
        _fail("anima_rt_run_sdpa_flash")
    return torch.from_numpy(out).to(dtype=q.dtype).reshape(B, H, Sq, D)


def anima_rt_rope(t_np, freqs_np):
    """apply_rotary_pos_emb on t [B, S, H, D] or [N, S, D] fp32 with freqs [S, D/2, 2, 2]."""
    if t_np.ndim == 4:
        B, S, H, D = t_np.shape
        N = B * H
        t_flat = _f32c(np.transpose(t_np, (0, 2, 1, 3)).reshape(N, S, D))
    else:
        N, S, D = t_np.shape
        t_flat = _f32c(t_np)
    f = _f32c(freqs_np)
    out = np.zeros((N, S, D), dtype=np.float32)
    if not L.lib.anima_rt_run_rope(t_flat.ctypes.data, f.ctypes.data, out.ctypes.data, N, S, D):
        _fail("anima_rt_run_rope")
    if t_np.ndim == 4:
        return np.ascontiguousarray(out.reshape(B, H, S, D).transpose(0, 2, 1, 3))
    return out


class AnimaRTRMSNorm(nn.RMSNorm):
    """nn.RMSNorm whose forward runs the B200 kernel through anima_rt_run_rmsnorm."""

    def forward(self, x):
        _ensure_init()
        *batch, D = x.shape
        M = int(np.prod(batch)) if batch else 1
        xf = _f32c(x.detach().reshape(M, D).cpu().float().numpy())
        w = None if self.weight is None else _f32c(self.weight.detach().cpu().float().numpy())
        out = np.zeros((M, D), dtype=np.float32)
        eps = self.eps if self.eps is not None else torch.finfo(torch.float32).eps
        if not L.lib.anima_rt_run_rmsnorm(xf.ctypes.data, None if w is None else w.ctypes.data,
                                          out.ctypes.data, M, D, ct.c_float(eps)):
            _fail("anima_rt_run_rmsnorm")
        res = torch.from_numpy(out).to(device=x.device, dtype=x.dtype)
        return res.reshape(*batch, D) if batch else res.squeeze(0)


class Predict2Backend:
    """The three operations patch_predict2 installs.  The default is this library on the
    GPU; CPU tests pass stand-ins with the same signatures to check the patch's plumbing
    against the reference model (the GPU kernels are tested on the GPU on their own).
      sdpa(q, k, v)                      [B, H, S, D] -> [B, H, S_q, D], q's dtype
      rope(t, freqs)                     t [B, S, H, D], freqs [S, D/2, 2, 2] -> t's shape
      attention(q, k, v, q_norm_w, k_norm_w, rope_freqs, eps=..., out_dtype=...)
                                         ops.attention's signature"""

    def __init__(self, sdpa=None, rope=None, attention=None):
        self.sdpa = sdpa or ops.sdpa
        self.rope = rope or _rope_any_device
        self.attention = attention or ops.attention


def _rope_any_device(t, freqs):
    """apply_rotary_pos_emb on CUDA tensors through anima_attn_rope; on host tensors through
    the reference-facing host ABI (anima_rt_run_rope)."""
    if t.is_cuda:
        return ops.apply_rope(t, freqs)
    S, D = t.shape[1], t.shape[-1]
    f = np.ascontiguousarray(freqs.detach().float().reshape(S, D // 2, 2, 2).numpy())
    out = anima_rt_rope(t.detach().float().numpy(), f)
    return torch.from_numpy(out).to(dtype=t.dtype).reshape(t.shape)


def _freqs_per_token(rope_emb, S, D):
    """predict2 hands the blocks the 3D RoPE table as [1, S, 1, D/2, 2, 2] (a broadcast
    shape, no batch; src/predict2.py:885).  Returns it as [S, D/2, 2, 2]; a table of another
    size (for instance with a real batch dimension) is rejected rather than misread."""
    if rope_emb.numel() != S * D * 2:
        raise ValueError(f"rope_emb of shape {tuple(rope_emb.shape)} does not hold one "
                         f"[{D // 2}, 2, 2] entry per token of a {S}-token sequence")
    return rope_emb.reshape(S, D // 2, 2, 2)


def patch_predict2(p2, backend: "Predict2Backend" = None, fused: bool = True) -> dict:
    """Route a loaded ``predict2`` module's attention through the B200 library.

    The reference's own patch points (anima_rt/scripts/phone_pipeline_anima_rt.py:224-252):
    * ``_scaled_dot_product_attention(q, k, v, heads, skip_reshape)`` (predict2.py:25-29)
      -> backend.sdpa, reshaped as the reference does;
    * ``apply_rotary_pos_emb(t, freqs)`` (predict2.py:31-38) -> backend.rope;
    and, going further than the reference, ``Attention.forward`` (predict2.py:201-214): the
    module's own projections, then ONE fused call (q/k RMSNorm with the module's weights,
    RoPE for self-attention, SDPA), then ``output_proj``.  fused=False patches only the
    reference's two points.  Returns the replaced originals (restore them with
    unpatch_predict2)."""
    be = backend or Predict2Backend()
    orig = {"_scaled_dot_product_attention": p2._scaled_dot_product_attention,
            "apply_rotary_pos_emb": p2.apply_rotary_pos_emb,
            "Attention.forward": p2.Attention.forward}

    def _sdpa(q, k, v, heads, skip_reshape=False, transformer_options=None):
        out = be.sdpa(q, k, v)
        if skip_reshape:
            return out.transpose(1, 2).reshape(q.shape[0], -1, heads * q.shape[-1])
        return out.reshape(q.shape[0], q.shape[2], heads * q.shape[-1])

    def _rope(t, freqs):
        return be.rope(t, _freqs_per_token(freqs, t.shape[1], t.shape[-1]))

    def _forward(self, x, context=None, rope_emb=None, transformer_options={}):
        ctx = x if context is None else context
        B, Sq = x.shape[0], x.shape[1]
        Skv = ctx.shape[1]
        H, D = self.n_heads, self.head_dim
        q = self.q_proj(x).view(B, Sq, H, D)
        k = self.k_proj(ctx).view(B, Skv, H, D)
        v = self.v_proj(ctx).view(B, Skv, H, D)
        freqs = None
        if self.is_selfattn and rope_emb is not None:
            freqs = _freqs_per_token(rope_emb, Sq, D)
        eps = self.q_norm.eps if getattr(self.q_norm, "eps", None) is not None else 1e-6
        o = be.attention(q, k, v, self.q_norm.weight, self.k_norm.weight, freqs, eps=eps,
                         out_dtype=torch.float32 if x.dtype == torch.float32 else torch.bfloat16)
        o = o.reshape(B, Sq, H * D).to(x.dtype)
        return self.output_dropout(self.output_proj(o))

    p2._scaled_dot_product_attention = _sdpa
    p2.apply_rotary_pos_emb = _rope
    if fused:
        p2.Attention.forward = _forward
    return orig


def unpatch_predict2(p2, orig: dict) -> None:
    """Undo patch_predict2 with the originals it returned."""
    p2._scaled_dot_product_attention = orig["_scaled_dot_product_attention"]
    p2.apply_rotary_pos_emb = orig["apply_rotary_pos_emb"]
    p2.Attention.forward = orig["Attention.forward"]
