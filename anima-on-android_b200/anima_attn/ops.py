"""Torch-tensor front end of the B200 attention library.

All tensors are CUDA tensors on the current device; every call is enqueued on the
current torch stream and returns without synchronising.  The kernels run in
libanima_attn.so (sm_100a); there is no PyTorch or CPU fallback.

Layouts follow the reference call sites:
  * projections q/k/v as produced by ``rearrange(t, "b s (h d) -> b s h d")``
    (src/predict2.py:177-180, anima_rt/scripts/numpy_dit.py:283): [B, S, H, D];
  * operands of the attention core: [B*H, S, D] 16-bit (the anima_rt [BH, S, D]
    layout, anima_rt/src/anima_rt.cpp:142-145);
  * output [B, S, H, D] (what the o-proj consumes, numpy_dit.py:294) or [B, H, S, D]
    (what F.scaled_dot_product_attention returns, predict2.py:25-29).
"""
from __future__ import annotations

import ctypes as ct
import math
from typing import Optional

import torch

from . import _lib as L

L_ = L

_TORCH_DT = {torch.float32: L.DTYPE_F32, torch.bfloat16: L.DTYPE_BF16, torch.float16: L.DTYPE_F16}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ct.c_void_p(t.data_ptr())


def _check_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("anima_attn ops take CUDA tensors")


def _as_weight(w: Optional[torch.Tensor], device) -> Optional[torch.Tensor]:
    if w is None:
        return None
    return w.detach().to(device=device, dtype=torch.float32).contiguous()


def prologue(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
             q_norm_w: Optional[torch.Tensor] = None, k_norm_w: Optional[torch.Tensor] = None,
             rope_freqs: Optional[torch.Tensor] = None, eps: float = 1e-6,
             norm_q: bool = True, norm_k: bool = True, op_dtype=torch.bfloat16,
             out: Optional[tuple] = None):
    """Fused per-head RMSNorm + 3D RoPE + cast + transpose, one HBM pass.

    q [B, S_q, H, D], k/v [B, S_kv, H, D] (fp32/bf16/fp16, any strides with D
    contiguous) -> (q, k, v) [B*H, S, D] in ``op_dtype``.  ``norm_q``/``norm_k`` apply
    RMSNorm (weights may be None = 1); ``rope_freqs`` [S, D/2, 2, 2] fp32 rotates q and k.
    Replaces numpy_dit.py:285-291 / predict2.py:182-193.
    q = None, or k = v = None, runs one side only and returns None for the other (a side
    whose operands are kept across calls, e.g. the K/V of a constant text context).
    """
    ref = q if q is not None else k
    if ref is None or (k is None) != (v is None):
        raise ValueError("pass q, or k and v, or all three")
    _check_cuda(q, k, v)
    B, _, H, D = ref.shape
    Sq = 0 if q is None else q.shape[1]
    Skv = 0 if k is None else k.shape[1]
    present = [t for t in (q, k, v) if t is not None]
    if q is not None and q.shape != (B, Sq, H, D):
        raise ValueError("q must be [B, S_q, H, D]")
    if k is not None and (k.shape != (B, Skv, H, D) or v.shape != k.shape):
        raise ValueError("k and v must be [B, S_kv, H, D] matching q")
    if ref.dtype not in _TORCH_DT or any(t.dtype != ref.dtype for t in present):
        raise ValueError("q, k, v must share one of float32/bfloat16/float16")
    for t in present:
        if t.stride(3) != 1:
            raise ValueError("the head dimension must be contiguous")
    dev = ref.device
    if out is None:
        qo = None if q is None else torch.empty((B * H, Sq, D), device=dev, dtype=op_dtype)
        ko = None if k is None else torch.empty((B * H, Skv, D), device=dev, dtype=op_dtype)
        vo = None if v is None else torch.empty((B * H, Skv, D), device=dev, dtype=op_dtype)
    else:
        qo, ko, vo = out
    qw, kw = _as_weight(q_norm_w, dev), _as_weight(k_norm_w, dev)
    fr = None
    flags = (L.FLAG_QNORM if norm_q else 0) | (L.FLAG_KNORM if norm_k else 0)
    if rope_freqs is not None:
        fr = rope_freqs.detach().to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
        if fr.numel() != Sq * D * 2:
            raise ValueError("rope_freqs must hold [S_q, D/2, 2, 2] values")
        flags |= L.FLAG_ROPE
    a = L.PrologueArgs()
    a.q, a.k, a.v = _ptr(q), _ptr(k), _ptr(v)
    a.in_dtype = _TORCH_DT[ref.dtype]
    for name, t in (("q_stride", q), ("k_stride", k), ("v_stride", v)):
        getattr(a, name)[:] = [0, 0, 0] if t is None else [t.stride(0), t.stride(1), t.stride(2)]
    a.B, a.H, a.S_q, a.S_kv, a.D = B, H, Sq, Skv, D
    a.q_norm_w, a.k_norm_w = _ptr(qw), _ptr(kw)
    a.eps = float(eps)
    a.rope_freqs = _ptr(fr)
    a.flags = flags
    a.q_out, a.k_out, a.v_out = _ptr(qo), _ptr(ko), _ptr(vo)
    a.op_dtype = _TORCH_DT[op_dtype]
    # qw/kw/fr may be freed on return: the caching allocator hands their blocks only to
    # work enqueued later on this stream, which runs after the kernel.
    L.check(L.lib.anima_attn_prologue(ct.byref(a), ct.c_void_p(_stream())), "anima_attn_prologue")
    return qo, ko, vo


_WORKSPACES: dict = {}


def _workspace(device: torch.device, nbytes: int) -> Optional[torch.Tensor]:
    """Grow-only, zero-filled scratch per (device, stream) for the split schedule.  The
    kernel leaves its arrival counters at zero, so the buffer is reused as is."""
    if nbytes == 0:
        return None
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def attention_core(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, B: int, H: int,
                   scale: Optional[float] = None, kv_valid_len: Optional[torch.Tensor] = None,
                   causal: bool = False, out: Optional[torch.Tensor] = None,
                   out_layout: str = "bshd", out_dtype=torch.float32,
                   schedule: str = "auto", pair: bool = False,
                   kv64: bool = False, peers: Optional[list] = None,
                   scatter: Optional[tuple] = None) -> torch.Tensor:
    """tcgen05 flash attention on 16-bit head-major operands.

    q [B*H, S_q, 128], k/v [B*H, S_kv, 128] contiguous bf16/fp16.  Returns (or fills)
    ``out`` in ``out_layout`` "bshd" [B, S_q, H, D] or "bhsd" [B, H, S_q, D].
    ``kv_valid_len`` int32 [B] masks keys >= kv_valid_len[b] (cross-attention padding).
    ``schedule`` for calls of more than one wave of 256-row units: "auto" lets the library
    choose (a cached workspace is passed for the cut last round); "unit" one CTA per unit;
    "whole" a persistent grid of whole units; "split" the persistent grid with the last
    round cut into key-tile slices.
    ``pair`` runs the CTA-pair kernel (2-SM MMA, one pair per 512-row unit).
    ``kv64`` runs the 64-key-tile kernel, whose P has tensor-memory columns of its own so a
    query tile's next QK^T overlaps its softmax.
    ``peers``: device addresses (one per rank, this rank's included) that each receive every
    output block, with ``out``'s strides and dtype (anima_attn_fwd_gather): the all-gather
    of head outputs done by the epilogue; ``out`` is then this rank's own destination.
    ``scatter`` = (dest, rows_per_dest, row_stride, head0): the output rows go to the ranks
    that own them (anima_attn_fwd_scatter_rows): global row b*S_q + s to dest[g //
    rows_per_dest] at row g % rows_per_dest, columns of heads head0.. of rows row_stride
    elements long; nothing is returned (``out`` is not used).
    """
    _check_cuda(q, k, v)
    BH, Sq, D = q.shape
    Skv = k.shape[1]
    if BH != B * H or k.shape != (BH, Skv, D) or v.shape != k.shape:
        raise ValueError("operands must be [B*H, S, D]")
    if q.dtype not in (torch.bfloat16, torch.float16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("operands must be bfloat16 or float16")
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
        raise ValueError("operands must be contiguous")
    if out is None and scatter is not None:  # strides only; the kernel stores to `scatter`
        out = torch.empty((1, 1, 1, D), device=q.device, dtype=out_dtype).expand(B, Sq, H, D)
    if out is None:
        shape = (B, Sq, H, D) if out_layout == "bshd" else (B, H, Sq, D)
        out = torch.empty(shape, device=q.device, dtype=out_dtype)
    if out_layout == "bshd":
        st = (out.stride(0), out.stride(2), out.stride(1))
    elif out_layout == "bhsd":
        st = (out.stride(0), out.stride(1), out.stride(2))
    else:
        raise ValueError("out_layout must be 'bshd' or 'bhsd'")
    if out.stride(3) != 1:
        raise ValueError("output head dimension must be contiguous")
    flags = (L.FLAG_CAUSAL if causal else 0) | (L.FLAG_PAIR if pair else 0)
    if kv64:
        flags |= L.FLAG_KV64
    if schedule not in ("auto", "unit", "whole", "split"):
        raise ValueError("schedule must be 'auto', 'unit', 'whole' or 'split'")
    flags |= {"auto": 0, "unit": L.FLAG_UNIT, "whole": L.FLAG_WHOLE,
              "split": L.FLAG_SPLIT}[schedule]
    vl = None
    if kv_valid_len is not None:
        vl = kv_valid_len.to(device=q.device, dtype=torch.int32).contiguous()
        if vl.numel() != B:
            raise ValueError("kv_valid_len must have B entries")
        flags |= L.FLAG_MASK
    a = L.AttnArgs()
    a.q, a.k, a.v = _ptr(q), _ptr(k), _ptr(v)
    a.op_dtype = _TORCH_DT[q.dtype]
    a.out = _ptr(out)
    a.out_dtype = _TORCH_DT[out.dtype]
    a.out_stride[:] = list(st)
    a.B, a.H, a.S_q, a.S_kv, a.D = B, H, Sq, Skv, D
    a.scale = float(1.0 / math.sqrt(D) if scale is None else scale)
    a.flags = flags
    a.kv_valid_len = _ptr(vl)
    ws = None
    if schedule in ("auto", "split") and not pair:
        ws = _workspace(q.device, int(L.lib.anima_attn_workspace_size(B, H, Sq, Skv, flags)))
    a.workspace = _ptr(ws)
    a.workspace_bytes = 0 if ws is None else ws.numel()
    if scatter is not None:
        dest, rows_per_dest, row_stride, head0 = scatter
        arr = (ct.c_void_p * len(dest))(*dest)
        L.check(L.lib.anima_attn_fwd_scatter_rows(ct.byref(a), arr, len(dest), int(rows_per_dest),
                                                  int(row_stride), int(head0),
                                                  ct.c_void_p(_stream())),
                "anima_attn_fwd_scatter_rows")
        return None
    if peers:
        arr = (ct.c_void_p * len(peers))(*peers)
        L.check(L.lib.anima_attn_fwd_gather(ct.byref(a), arr, len(peers), ct.c_void_p(_stream())),
                "anima_attn_fwd_gather")
    else:
        L.check(L.lib.anima_attn_fwd(ct.byref(a), ct.c_void_p(_stream())), "anima_attn_fwd")
    return out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
              q_norm_w: Optional[torch.Tensor] = None, k_norm_w: Optional[torch.Tensor] = None,
              rope_freqs: Optional[torch.Tensor] = None,
              kv_valid_len: Optional[torch.Tensor] = None, norm_q: bool = True,
              norm_k: bool = True, causal: bool = False, scale: Optional[float] = None,
              eps: float = 1e-6, out_dtype=torch.float32, op_dtype=torch.bfloat16,
              workspace: Optional[tuple] = None, out: Optional[torch.Tensor] = None):
    """The attention of one DiT block from projections to o-proj input.

    q [B, S_q, H, D], k/v [B, S_kv, H, D] pre-norm projections -> [B, S_q, H, D]:
    q/k RMSNorm, RoPE (self-attention), SDPA with optional key-padding mask.  This is
    NumpyAttention.forward between the projection and o-proj GEMMs
    (numpy_dit.py:285-294) and predict2 Attention.compute_qkv's norm/RoPE plus
    torch_attention_op (predict2.py:182-193, 61-88).
    """
    B, Sq, H, D = q.shape
    qh, kh, vh = prologue(q, k, v, q_norm_w, k_norm_w, rope_freqs, eps, norm_q, norm_k,
                          op_dtype, out=workspace)
    return attention_core(qh, kh, vh, B, H, scale, kv_valid_len, causal, out=out,
                          out_layout="bshd", out_dtype=out_dtype)


def attention_cached_kv(q: torch.Tensor, kh: torch.Tensor, vh: torch.Tensor,
                        q_norm_w: Optional[torch.Tensor] = None, norm_q: bool = True,
                        kv_valid_len: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                        eps: float = 1e-6, out_dtype=torch.float32,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Cross-attention whose K/V operands were prepared earlier: q [B, S_q, H, D] pre-norm
    projection -> [B, S_q, H, D].  kh/vh [B*H, S_kv, D] 16-bit head-major, as prologue(None,
    k, v) returns them.  Runs the q side of the prologue and the attention core only."""
    B, Sq, H, D = q.shape
    qh, _, _ = prologue(q, None, None, q_norm_w, None, None, eps, norm_q, False, kh.dtype)
    return attention_core(qh, kh, vh, B, H, scale, kv_valid_len, False, out=out,
                          out_layout="bshd", out_dtype=out_dtype)


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None,
         is_causal: bool = False, op_dtype=torch.bfloat16) -> torch.Tensor:
    """F.scaled_dot_product_attention on [B, H, S, D] tensors (predict2.py:25-29).

    Returns [B, H, S_q, D] in q's dtype (fp32 for fp32 inputs)."""
    B, H, Sq, D = q.shape
    Skv = k.shape[2]
    # [B, H, S, D] viewed as [B, S, H, D] with swapped strides: the prologue reads any
    # strides, so no transpose copy is made.
    qv, kv, vv = (t.transpose(1, 2) for t in (q, k, v))
    if q.dtype not in _TORCH_DT:
        raise ValueError("unsupported dtype")
    qh, kh, vh = prologue(qv, kv, vv, norm_q=False, norm_k=False, op_dtype=op_dtype)
    out_dtype = torch.bfloat16 if q.dtype == torch.bfloat16 else torch.float32
    o = attention_core(qh, kh, vh, B, H, scale, None, is_causal, out_layout="bhsd",
                       out_dtype=out_dtype)
    return o if o.dtype == q.dtype else o.to(q.dtype)


def qkv_projection(x: torch.Tensor, w: torch.Tensor, H: int, n_tensors: int = 3,
                   first_tensor: int = 0, q_norm_w: Optional[torch.Tensor] = None,
                   k_norm_w: Optional[torch.Tensor] = None,
                   rope_freqs: Optional[torch.Tensor] = None, eps: float = 1e-6,
                   norm_q: bool = True, norm_k: bool = True):
    """Projection GEMM with the attention prologue in its epilogue (anima_qkv_projection).

    x [B, L, K] 16-bit contiguous, w [n_tensors*H*128, K] in x's dtype (rows: tensor, head,
    128; tensors q, k, v from ``first_tensor``).  Returns the attention core's operands
    (q, k, v) [B*H, L, 128] in x's dtype, None for tensors not computed: q/k RMSNorm over the
    fp32 accumulator, RoPE on q and k when ``rope_freqs`` [L, 64, 2, 2] is given."""
    _check_cuda(x, w)
    B, L, K = x.shape
    if x.dtype not in (torch.float16, torch.bfloat16) or w.dtype != x.dtype:
        raise ValueError("x and w must share float16 or bfloat16")
    if w.shape != (n_tensors * H * 128, K) or not (x.is_contiguous() and w.is_contiguous()):
        raise ValueError("w must be [n_tensors*H*128, K]; x and w contiguous")
    outs = [None, None, None]
    for c in range(first_tensor, first_tensor + n_tensors):
        outs[c] = torch.empty((B * H, L, 128), device=x.device, dtype=x.dtype)
    qw, kw = _as_weight(q_norm_w, x.device), _as_weight(k_norm_w, x.device)
    fr = None
    flags = (L_.FLAG_QNORM if norm_q else 0) | (L_.FLAG_KNORM if norm_k else 0)
    if rope_freqs is not None:
        fr = rope_freqs.detach().to(device=x.device, dtype=torch.float32).reshape(-1).contiguous()
        if fr.numel() != L * 256:
            raise ValueError("rope_freqs must hold [L, 64, 2, 2] values")
        flags |= L_.FLAG_ROPE
    a = L_.QkvProjArgs()
    a.x, a.w = _ptr(x), _ptr(w)
    a.dtype = _TORCH_DT[x.dtype]
    a.B, a.L, a.H, a.K = B, L, H, K
    a.n_tensors, a.first_tensor = n_tensors, first_tensor
    a.q_norm_w, a.k_norm_w = _ptr(qw), _ptr(kw)
    a.eps = float(eps)
    a.rope_freqs = _ptr(fr)
    a.flags = flags
    a.q_out, a.k_out, a.v_out = (_ptr(t) for t in outs)
    L_.check(L_.lib.anima_qkv_projection(ct.byref(a), ct.c_void_p(_stream())), "anima_qkv_projection")
    return tuple(outs)


def qkv_projection_scatter(x: torch.Tensor, w: torch.Tensor, B: int, L: int, H: int, row0: int,
                           dest: list, n_tensors: int = 3, first_tensor: int = 0,
                           q_norm_w: Optional[torch.Tensor] = None,
                           k_norm_w: Optional[torch.Tensor] = None,
                           rope_freqs: Optional[torch.Tensor] = None, eps: float = 1e-6,
                           norm_q: bool = True, norm_k: bool = True) -> None:
    """qkv_projection for the token rows x [rows, K] (global rows row0.. of the [B, L] token
    grid) and all heads of a split over len(dest) ranks with H heads each, every head's
    operand rows stored into its rank's buffers (anima_qkv_projection_scatter): dest[d] =
    (q, k, v) device addresses of rank d's head-major [B*H, L, 128] buffers (0 for tensors
    not computed).  w [n_tensors*len(dest)*H*128, K] in (tensor, global head, dim) row order."""
    _check_cuda(x, w)
    if x.dtype not in (torch.float16, torch.bfloat16) or w.dtype != x.dtype:
        raise ValueError("x and w must share float16 or bfloat16")
    if x.dim() != 2 or not (x.is_contiguous() and w.is_contiguous()):
        raise ValueError("x must be [rows, K]; x and w contiguous")
    rows, K = x.shape
    if w.shape != (n_tensors * len(dest) * H * 128, K):
        raise ValueError("w must be [n_tensors*ranks*H*128, K]")
    qw, kw = _as_weight(q_norm_w, x.device), _as_weight(k_norm_w, x.device)
    fr = None
    flags = (L_.FLAG_QNORM if norm_q else 0) | (L_.FLAG_KNORM if norm_k else 0)
    if rope_freqs is not None:
        fr = rope_freqs.detach().to(device=x.device, dtype=torch.float32).reshape(-1).contiguous()
        if fr.numel() != L * 256:
            raise ValueError("rope_freqs must hold [L, 64, 2, 2] values")
        flags |= L_.FLAG_ROPE
    a = L_.QkvProjArgs()
    a.x, a.w = _ptr(x), _ptr(w)
    a.dtype = _TORCH_DT[x.dtype]
    a.B, a.L, a.H, a.K = B, L, H, K
    a.n_tensors, a.first_tensor = n_tensors, first_tensor
    a.q_norm_w, a.k_norm_w = _ptr(qw), _ptr(kw)
    a.eps = float(eps)
    a.rope_freqs = _ptr(fr)
    a.flags = flags
    flat = [int(p) for d3 in dest for p in d3]
    arr = (ct.c_void_p * len(flat))(*flat)
    L_.check(L_.lib.anima_qkv_projection_scatter(ct.byref(a), rows, row0, arr, len(dest),
                                                 ct.c_void_p(_stream())),
             "anima_qkv_projection_scatter")


def gemm_gelu(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """GELU(x @ w.T) in one tcgen05 GEMM, the exact GELU applied to the fp32 accumulator
    (anima_gemm_gelu; the MLP's first layer and activation, src/predict2.py:45).

    x [..., K] and w [N, K] contiguous float16 or bfloat16 of one type; returns [..., N] of
    that type."""
    _check_cuda(x, w)
    if x.dtype not in (torch.float16, torch.bfloat16) or w.dtype != x.dtype:
        raise ValueError("x and w must share float16 or bfloat16")
    if not (x.is_contiguous() and w.is_contiguous()) or w.dim() != 2 or x.shape[-1] != w.shape[1]:
        raise ValueError("x [..., K] and w [N, K] must be contiguous")
    K, N = w.shape[1], w.shape[0]
    M = x.numel() // K
    if out is None:
        out = torch.empty(x.shape[:-1] + (N,), device=x.device, dtype=x.dtype)
    L_.check(L_.lib.anima_gemm_gelu(_ptr(x), _ptr(w), _ptr(out), M, N, K, _TORCH_DT[x.dtype],
                                    ct.c_void_p(_stream())), "anima_gemm_gelu")
    return out


def apply_rope(t: torch.Tensor, freqs: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """predict2.apply_rotary_pos_emb (src/predict2.py:31-38) on the GPU.

    t [B, S, H, D] (any strides, D contiguous) or [N, S, D]; freqs holding [S, D/2, 2, 2]
    values (predict2's [1, S, 1, D/2, 2, 2] broadcast shape is accepted).  Computes in fp32
    and returns t's dtype, like the reference."""
    _check_cuda(t, freqs)
    if t.dim() == 3:
        tv = t.unsqueeze(2)
    elif t.dim() == 4:
        tv = t
    else:
        raise ValueError("t must be [B, S, H, D] or [N, S, D]")
    O, S, Hn, D = tv.shape
    fr = freqs.detach().to(device=t.device, dtype=torch.float32).reshape(-1).contiguous()
    if fr.numel() != S * D * 2:
        raise ValueError(f"freqs must hold [S={S}, {D // 2}, 2, 2] values, got {freqs.shape}")
    src = tv if tv.dtype == torch.float32 else tv.float()
    if src.stride(3) != 1:
        src = src.contiguous()
    res = torch.empty((O, S, Hn, D), device=t.device, dtype=torch.float32) if out is None else out
    ts = (ct.c_int64 * 3)(src.stride(0), src.stride(1), src.stride(2))
    os_ = (ct.c_int64 * 3)(res.stride(0), res.stride(1), res.stride(2))
    L.check(L.lib.anima_attn_rope(_ptr(src), ts, _ptr(fr), _ptr(res), os_, O, S, Hn, D,
                                  ct.c_void_p(_stream())), "anima_attn_rope")
    res = res.view(t.shape) if t.dim() == 3 else res
    return res if res.dtype == t.dtype else res.to(t.dtype)


def ln_modulate(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, eps: float = 1e-6,
                out_dtype=torch.float16) -> torch.Tensor:
    """LayerNorm(x) * (1 + scale) + shift -> out_dtype, one pass (DiT block, predict2.py:512).
    x [B, L, D] fp32 contiguous; scale/shift [B, 1, D] fp32 views with D contiguous."""
    _check_cuda(x, scale, shift)
    B, Lr, D = x.shape
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("x must be contiguous float32")
    y = torch.empty((B, Lr, D), device=x.device, dtype=out_dtype)
    if scale.stride(-1) != 1 or shift.stride(-1) != 1 or scale.stride(0) != shift.stride(0):
        raise ValueError("scale/shift rows must be contiguous with a common batch stride")
    L.check(L.lib.anima_dit_ln_modulate(_ptr(x), _ptr(scale), _ptr(shift), scale.stride(0), _ptr(y),
                                        _TORCH_DT[out_dtype], B * Lr, Lr, D, float(eps),
                                        ct.c_void_p(_stream())), "anima_dit_ln_modulate")
    return y


def gate_residual_(x: torch.Tensor, gate: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """x += gate * y in place; x, y [B, L, D] fp32 contiguous, gate [B, 1, D] view."""
    _check_cuda(x, gate, y)
    B, Lr, D = x.shape
    if gate.stride(-1) != 1 or not y.is_contiguous() or not x.is_contiguous():
        raise ValueError("contiguous operands expected")
    if x.dtype != torch.float32 or y.dtype != torch.float32 or y.shape != x.shape:
        raise ValueError("x and y must be float32 of one shape")
    L.check(L.lib.anima_dit_gate_residual(_ptr(x), _ptr(gate), gate.stride(0), _ptr(y), B * Lr, Lr,
                                          D, ct.c_void_p(_stream())), "anima_dit_gate_residual")
    return x


def gate_residual_ln_modulate_(x: torch.Tensor, gate: torch.Tensor, y: torch.Tensor,
                               scale: torch.Tensor, shift: torch.Tensor, eps: float = 1e-6,
                               out_dtype=torch.float16) -> torch.Tensor:
    """x += gate * y in place, then LayerNorm(x) * (1 + scale) + shift -> out_dtype, in one
    pass.  x [B, L, D] fp32 contiguous, y of x's shape (fp32, fp16 or bf16) contiguous;
    gate/scale/shift [B, 1, D] views with D contiguous (scale and shift with a common batch
    stride)."""
    _check_cuda(x, gate, y, scale, shift)
    B, Lr, D = x.shape
    if not (x.is_contiguous() and y.is_contiguous()) or x.dtype != torch.float32 or \
            y.dtype not in _TORCH_DT or y.shape != x.shape:
        raise ValueError("x (float32) and y must be contiguous tensors of one shape")
    if gate.stride(-1) != 1 or scale.stride(-1) != 1 or shift.stride(-1) != 1 or \
            scale.stride(0) != shift.stride(0):
        raise ValueError("gate/scale/shift rows must be contiguous, scale/shift one batch stride")
    h = torch.empty((B, Lr, D), device=x.device, dtype=out_dtype)
    L.check(L.lib.anima_dit_gate_residual_ln_modulate(
        _ptr(x), _ptr(gate), gate.stride(0), _ptr(y), _TORCH_DT[y.dtype], _ptr(scale), _ptr(shift),
        scale.stride(0),
        _ptr(h), _TORCH_DT[out_dtype], B * Lr, Lr, D, float(eps), ct.c_void_p(_stream())),
        "anima_dit_gate_residual_ln_modulate")
    return h


def gelu_(x: torch.Tensor) -> torch.Tensor:
    """Exact GELU in place on a contiguous fp16/bf16 CUDA tensor (numel a multiple of 8)."""
    _check_cuda(x)
    if x.dtype not in (torch.float16, torch.bfloat16) or not x.is_contiguous():
        raise ValueError("x must be a contiguous float16/bfloat16 tensor")
    L.check(L.lib.anima_dit_gelu(_ptr(x), _ptr(x), _TORCH_DT[x.dtype], x.numel(),
                                 ct.c_void_p(_stream())), "anima_dit_gelu")
    return x


def status(reset: bool = True) -> int:
    """Synchronise the current stream and return the device status word (0 = clean).
    A non-zero status drops the cached workspaces (an aborted kernel may have left
    arrival counters non-zero)."""
    rc = L.lib.anima_attn_status(ct.c_void_p(_stream()), int(reset))
    if rc != 0:
        _WORKSPACES.clear()
    return rc


def device_info():
    sm, cc = ct.c_int(0), ct.c_int(0)
    L.check(L.lib.anima_attn_device_info(ct.byref(sm), ct.byref(cc)), "anima_attn_device_info")
    return sm.value, cc.value


def version() -> str:
    return L.lib.anima_attn_version().decode()
