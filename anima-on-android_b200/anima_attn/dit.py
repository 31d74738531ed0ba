"""One denoising step of the Anima 2B DiT on B200, head-parallel over N GPUs.

This restates, for inference, the reference model and sampler step around the attention
library:
  MiniTrainDIT._forward   src/predict2.py:841-908  (patch embed, RoPE table, timestep
                          embedding with adaLN-LoRA, blocks, final layer, unpatchify)
  Block.forward           src/predict2.py:469-583  (adaLN-modulated self-attention,
                          cross-attention and GELU MLP with gated residuals)
  Attention               src/predict2.py:91-214   (q/k/v projections, per-head q/k
                          RMSNorm, RoPE on self-attention, SDPA, o-proj)
  EulerSampler step       anima_rt/scripts/sampling.py:115-140 (CFG pair, Euler update)
The attention of every block (norm, RoPE, SDPA) runs in this library's kernels, and so do
the HBM passes around it: each gated residual update fused with the LayerNorm + adaLN
modulation + 16-bit cast that follows it (anima_dit_gate_residual_ln_modulate; the first
LayerNorm of the step alone, anima_dit_ln_modulate) and the exact GELU of the MLP
(anima_dit_gelu).  The q/k/v projections run as this library's projection GEMM with the
attention prologue in its epilogue (anima_qkv_projection, fused_qkv=True; outside the tokens
layout); the other GEMMs run in PyTorch (cuBLAS).  The residual stream stays fp32; GEMMs take
16-bit operands with fp32 accumulation.  The projections, MLP layers and o-proj write 16-bit output (their
consumers are the attention prologue, GELU, the next GEMM, or the fused residual pass, which
adds them into the fp32 residual stream); the adaLN and final-layer GEMMs write fp32.
The operand type is fp16 by default: the weights are bf16 values (exact in fp16 unless
below 2^-14), the GEMM inputs are normalised activations, and fp16's 10-bit mantissa
keeps the step's latent within 1.1e-3 rel-L2 of the fp32 reference model at 2 blocks,
where bf16 operands give 8.5e-3.  The attention runs on fp16 operands for the same
reason (q and k are RMS-normalised; v is a projection of normalised activations).

Multi-GPU (N ranks; the attention is split by heads in both modes, rank r owning heads
[r*16/N, (r+1)*16/N)):
  shard="heads"   the layout specified for this step: every rank holds the whole residual
                  stream, projects q/k/v for its heads only, runs their attention, and one
                  all_gather_into_tensor per attention collects every rank's head outputs
                  before the o-proj (one transpose copy to [B, S, hidden], one GEMM).  o-proj,
                  MLP, adaLN and final layer are replicated, so only the attention's share of
                  the step shrinks with N.
  shard="tokens"  (default) the same head-parallel attention, with everything else split by
                  tokens (sequence parallelism): rank r owns rows [r*R/N, (r+1)*R/N) of the
                  R = B*L token rows.  It projects q/k/v for all heads on its rows, one
                  all_to_all_single hands every rank its heads for all rows, attention runs
                  per head, and a second all_to_all_single returns all heads' outputs for its
                  own rows before the o-proj -- the part of the all-gather a rank uses.  The
                  o-proj, MLP, LayerNorm/adaLN passes and final layer run on its rows only.
                  Cross-attention K/V come from the (replicated, 512-token) context.  With
                  peer_a2a (default on CUDA) both exchanges are stores from the producing
                  kernels into the other ranks' buffers over NVLink (peer.PeerBuffers).

Weights follow the reference's parameter names (state-dict keys of MiniTrainDIT with
use_adaln_lora=True), so the same seeded weights load into the reference model for the
CPU oracle.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F


@dataclass
class DiTConfig:
    hidden: int = 2048
    heads: int = 16
    blocks: int = 28
    mlp_ratio: float = 4.0
    adaln_lora: int = 256
    in_channels: int = 16
    out_channels: int = 16
    patch: int = 2
    patch_t: int = 1
    ctx_dim: int = 1024
    eps: float = 1e-6
    rope_h_ratio: float = 4.0
    rope_w_ratio: float = 4.0
    rope_t_ratio: float = 1.0
    gemm_dtype: torch.dtype = torch.float16   # 16-bit operand type of GEMMs and attention

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def weight_spec(cfg: DiTConfig) -> List[Tuple[str, tuple, str]]:
    """(reference parameter name, shape, kind) in a fixed order; kind 'w' = Linear
    weight drawn N(0, 0.02) and stored bf16, 'one' = norm weight, fp32 ones."""
    D, H, hd, L = cfg.hidden, cfg.heads, cfg.head_dim, cfg.adaln_lora
    cin = (cfg.in_channels + 1) * cfg.patch * cfg.patch * cfg.patch_t  # + padding mask
    spec = [("x_embedder.proj.1.weight", (D, cin), "w"),
            ("t_embedder.1.linear_1.weight", (D, D), "w"),
            ("t_embedder.1.linear_2.weight", (3 * D, D), "w"),
            ("t_embedding_norm.weight", (D,), "one")]
    mlp = int(D * cfg.mlp_ratio)
    for b in range(cfg.blocks):
        p = f"blocks.{b}."
        for att, kv_in in (("self_attn", D), ("cross_attn", cfg.ctx_dim)):
            spec += [(p + att + ".q_proj.weight", (D, D), "w"),
                     (p + att + ".q_norm.weight", (hd,), "one"),
                     (p + att + ".k_proj.weight", (D, kv_in), "w"),
                     (p + att + ".k_norm.weight", (hd,), "one"),
                     (p + att + ".v_proj.weight", (D, kv_in), "w"),
                     (p + att + ".output_proj.weight", (D, D), "w")]
        spec += [(p + "mlp.layer1.weight", (mlp, D), "w"),
                 (p + "mlp.layer2.weight", (D, mlp), "w")]
        for m in ("self_attn", "cross_attn", "mlp"):
            spec += [(p + f"adaln_modulation_{m}.1.weight", (L, D), "w"),
                     (p + f"adaln_modulation_{m}.2.weight", (3 * D, L), "w")]
    pout = cfg.patch * cfg.patch * cfg.patch_t * cfg.out_channels
    spec += [("final_layer.linear.weight", (pout, D), "w"),
             ("final_layer.adaln_modulation.1.weight", (L, D), "w"),
             ("final_layer.adaln_modulation.2.weight", (2 * D, L), "w")]
    return spec


def make_weights(cfg: DiTConfig, seed: int = 0, device="cpu", rng_device="cpu",
                 keep: Optional[Callable[[str], bool]] = None) -> Dict[str, torch.Tensor]:
    """Seeded random weights: Linear ~ N(0, 0.02) rounded to bf16, norm weights 1.

    With rng_device='cpu' the values are identical on every machine (used by the parity
    tests and the reference oracle); 'cuda' draws them on the GPU (fast, for benches).
    ``keep`` filters names (a rank may skip weights it never uses)."""
    g = torch.Generator(device=rng_device).manual_seed(seed)
    out = {}
    for name, shape, kind in weight_spec(cfg):
        if kind == "one":
            t = torch.ones(shape, dtype=torch.float32)
        else:
            t = torch.empty(shape, dtype=torch.float32, device=rng_device).normal_(0.0, 0.02, generator=g)
            t = t.to(torch.bfloat16)
        if keep is None or keep(name):
            out[name] = t.to(device)
    return out


def timestep_sinusoid(t: torch.Tensor, channels: int) -> torch.Tensor:
    """Timesteps.forward (predict2.py:222-235): [B] -> [B, 1, channels] = [cos | sin]."""
    half = channels // 2
    exponent = -math.log(10000) * torch.arange(half, dtype=torch.float32, device=t.device)
    exponent = exponent / (half - 0.0)
    emb = t.float()[:, None] * torch.exp(exponent)[None, :]
    return torch.cat([torch.cos(emb), torch.sin(emb)], dim=-1)[:, None, :]


# CUDA-event regions of one profiled step (profile_step): None outside it.
_REGIONS: Optional[list] = None


class _region:
    """Brackets the work of one category (gemm, attention, fused, collective) on the current
    stream with CUDA events while a step is being profiled; a no-op otherwise."""
    __slots__ = ("cat", "e0")

    def __init__(self, cat: str):
        self.cat = cat

    def __enter__(self):
        if _REGIONS is not None:
            self.e0 = torch.cuda.Event(enable_timing=True)
            self.e0.record()

    def __exit__(self, *exc):
        if _REGIONS is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
            _REGIONS.append((self.cat, self.e0, e1))


def _linear(x: torch.Tensor, w: torch.Tensor, out_dtype=torch.float32) -> torch.Tensor:
    """x [..., K] @ w[N, K]^T: operands in w's 16-bit type, fp32 accumulation, output in
    ``out_dtype`` (fp32, or w's type)."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    if x.is_cuda:
        with _region("gemm"):
            if out_dtype == w.dtype:
                y = torch.mm(x2.to(w.dtype), w.t())
            else:
                y = torch.mm(x2.to(w.dtype), w.t(), out_dtype=out_dtype)
    else:  # CPU tests of the sharding logic: same operand rounding, fp32 math
        y = (x2.to(w.dtype).float() @ w.float().t()).to(out_dtype)
    return y.reshape(*shp[:-1], w.shape[0])


AttnFn = Callable[..., torch.Tensor]
_SUBBLOCKS = ("self_attn", "cross_attn", "mlp")  # adaLN-modulated sub-blocks of a block


class AnimaDiT:
    """Inference forward of the Anima DiT with this library's attention.

    ``weights`` is a make_weights() dict (full model; a rank slices what it needs).
    ``rank`` / ``world`` / ``group``: this rank, the number of ranks and their
    torch.distributed process group (world 1 = one GPU, no collectives).
    ``shard``: "tokens" (default) or "heads", the multi-GPU layouts of the module
    docstring; both split the attention by head.
    ``attn_fn`` replaces the attention op (signature of anima_attn.attention); tests on
    CPU pass a reference implementation, the product uses the B200 kernels.
    ``fused_qkv``: with the library attention on CUDA, the MLP's first layer and GELU run as
    one GEMM (anima_gemm_gelu), and outside the tokens layout the q/k/v
    projections run as anima_qkv_projection (the GEMM with q/k RMSNorm, RoPE and the
    head-major 16-bit store in its epilogue) followed by the attention core, instead of a
    cuBLAS GEMM whose output the attention prologue reads back.
    ``peer_a2a``: tokens layout with fused_qkv: the projection GEMM stores each head's
    operand rows into the owning rank's buffers and the attention stores each output row into
    its token owner's buffer over NVLink (anima_qkv_projection_scatter,
    anima_attn_fwd_scatter_rows), with one-element all-reduces ordering the ranks, instead of
    two NCCL all-to-alls and the prologue per attention.
    ``peer_gather``: heads layout on N > 1 GPUs with fused_qkv: the attention kernel stores
    its head outputs into every rank's gather buffer over NVLink (anima_attn_fwd_gather) and a
    one-element all-reduce orders the ranks, instead of an NCCL all-gather.  The buffers are
    allocated by a collective call on the first step (every rank, before graph capture);
    ``close()`` releases the peer mappings (every rank, before the process group goes).
    """

    def __init__(self, cfg: DiTConfig, weights: Dict[str, torch.Tensor], rank: int = 0,
                 world: int = 1, group=None, attn_fn: Optional[AttnFn] = None,
                 shard: str = "tokens", fused_qkv: bool = True, peer_gather: bool = True,
                 peer_a2a: bool = True):
        if cfg.heads % world:
            raise ValueError("heads must divide evenly over ranks")
        if shard not in ("tokens", "heads"):
            raise ValueError("shard must be 'tokens' or 'heads'")
        self.cfg, self.rank, self.world, self.group = cfg, rank, world, group
        self.seq = shard == "tokens" and world > 1
        self.h_local = cfg.heads // world
        self.w = {}
        cols = self.h_local * cfg.head_dim
        lo, hi = rank * cols, (rank + 1) * cols
        for name, t in weights.items():
            if t.dtype == torch.bfloat16:
                t = t.to(cfg.gemm_dtype)  # GEMM operand type
            self.w[name] = t
        # One GEMM per input: self-attention [Wq; Wk; Wv] on x, cross-attention [Wk; Wv]
        # on the context.  The prologue reads q/k/v as strided views of its output.
        #  heads mode: only this rank's heads ([3*cols, D] and [2*cols, ctx]).
        #  tokens mode: self-attention and cross q for every head, grouped by owning rank
        #  ([N, 3*cols, D] and [N, cols, D]) so one batched GEMM writes the all-to-all's
        #  send buffer; cross k/v for this rank's heads only.
        N = world
        for b in range(cfg.blocks):
            p = f"blocks.{b}."
            sa, ca = p + "self_attn.", p + "cross_attn."
            if sa + "q_proj.weight" not in self.w:
                continue
            wq, wk, wv = (self.w.pop(sa + f"{c}_proj.weight") for c in "qkv")
            if self.seq:
                D = wq.shape[1]
                self.w[sa + "qkv"] = torch.cat([t.view(N, cols, D) for t in (wq, wk, wv)], 1).contiguous()
                cq = self.w.pop(ca + "q_proj.weight")
                self.w[ca + "q_by_rank"] = cq.view(N, cols, cq.shape[1]).contiguous()
                if peer_a2a and self.w[sa + "qkv"].is_cuda:  # (tensor, global head, dim) rows
                    self.w[sa + "qkv_all"] = torch.cat([wq, wk, wv]).contiguous()
                    self.w[ca + "q_all"] = cq.contiguous()
            else:
                self.w[sa + "qkv"] = torch.cat([wq[lo:hi], wk[lo:hi], wv[lo:hi]]).contiguous()
                self.w[ca + "q_proj.weight"] = self.w[ca + "q_proj.weight"][lo:hi].contiguous()
            ck, cv = (self.w.pop(ca + f"{c}_proj.weight") for c in "kv")
            self.w[ca + "kv"] = torch.cat([ck[lo:hi], cv[lo:hi]]).contiguous()
        # The adaLN-LoRA modulations depend only on the timestep embedding, so on CUDA all
        # blocks' are computed at once per forward (_all_mods: one GEMM for the 84 first
        # layers, one batched GEMM for the 84 second layers) instead of 336 small launches.
        # The per-block entries become views of the two stacks, so no weight is held twice.
        self._mod_w, self._mod_all = None, None
        mnames = [(f"blocks.{b}.adaln_modulation_{m}.1.weight",
                   f"blocks.{b}.adaln_modulation_{m}.2.weight")
                  for b in range(cfg.blocks) for m in _SUBBLOCKS]
        if all(n1 in self.w and n2 in self.w for n1, n2 in mnames) and \
                self.w[mnames[0][0]].is_cuda:
            w1 = torch.cat([self.w[n1] for n1, _ in mnames]).contiguous()   # [84 * Lr, D]
            w2 = torch.stack([self.w[n2] for _, n2 in mnames]).contiguous()  # [84, 3D, Lr]
            lr = self.w[mnames[0][0]].shape[0]
            for i, (n1, n2) in enumerate(mnames):
                self.w[n1], self.w[n2] = w1[i * lr:(i + 1) * lr], w2[i]
            self._mod_w = (w1, w2)
        from .ops import attention as _lib_attention
        if attn_fn is None:
            attn_fn = _lib_attention
        self.attn_fn = attn_fn
        self.fused_qkv = bool(fused_qkv) and attn_fn is _lib_attention
        # heads layout over N > 1 GPUs: the attention stores its head outputs straight into
        # every rank's gather buffer over NVLink (peer.GatherBuffers), replacing the NCCL
        # all-gather and the transpose before the o-proj
        self.peer_gather = bool(peer_gather) and self.fused_qkv and world > 1 and not self.seq
        self._gather = None
        # tokens layout: the q/k/v projection stores each head's operand rows into its owner's
        # buffers and the attention stores each output row into its token owner's buffer,
        # over NVLink (anima_qkv_projection_scatter, anima_attn_fwd_scatter_rows), in place of
        # the two NCCL all-to-alls and the prologue on the received projections
        self.peer_a2a = bool(peer_a2a) and self.fused_qkv and self.seq
        self._a2a_bufs, self._a2a_key = None, None
        self._freqs_cache = {}
        self._w32 = {}

    # ------------------------------------------------------------------ pieces
    def _rope(self, T, Hp, Wp, device):
        key = (T, Hp, Wp, str(device))
        if key not in self._freqs_cache:
            from .rope import rope_freqs_3d
            self._freqs_cache[key] = rope_freqs_3d(
                T, Hp, Wp, self.cfg.head_dim, self.cfg.rope_h_ratio, self.cfg.rope_w_ratio,
                self.cfg.rope_t_ratio, device=device)
        return self._freqs_cache[key]

    def _ln_mod(self, x, scale, shift):
        """LayerNorm(x) * (1 + scale) + shift as the next GEMM's 16-bit operand."""
        if x.is_cuda:
            from .ops import ln_modulate
            with _region("fused"):
                return ln_modulate(x, scale, shift, self.cfg.eps, out_dtype=self.cfg.gemm_dtype)
        h = F.layer_norm(x, (x.shape[-1],), eps=self.cfg.eps) * (1 + scale) + shift
        return h.to(self.cfg.gemm_dtype)

    def _add_ln(self, x, pending, scale, shift):
        """Apply a pending gated residual (gate, y) to x, then LayerNorm + modulate it:
        returns (x, h).  Every gated residual of a block is followed by the next sub-block's
        (or the final layer's) LayerNorm, so on CUDA the two run as one pass over the
        residual stream with x updated in place (x is this forward's own buffer)."""
        if pending is None:
            return x, self._ln_mod(x, scale, shift)
        gate, y = pending
        if x.is_cuda:
            from .ops import gate_residual_ln_modulate_
            with _region("fused"):
                return x, gate_residual_ln_modulate_(x, gate, y, scale, shift, self.cfg.eps,
                                                     out_dtype=self.cfg.gemm_dtype)
        x = x + gate * y
        return x, self._ln_mod(x, scale, shift)

    @staticmethod
    def _gelu(h):
        """Exact GELU (nn.GELU, predict2.py:45) on the 16-bit MLP hidden layer, in place on
        CUDA; fp32 arithmetic either way."""
        if h.is_cuda and h.numel() % 8 == 0 and h.is_contiguous():
            from .ops import gelu_
            with _region("fused"):
                return gelu_(h)
        return F.gelu(h.float()).to(h.dtype)

    def _all_mods(self, emb, lora):
        """Every block's adaLN-LoRA modulation at once, [blocks * 3, B, 3 * hidden] fp32 in
        (block, sub-block) order: the same operand rounding as _mods (16-bit SiLU(emb) and
        hidden layer, fp32 accumulation), one GEMM and one batched GEMM."""
        w1, w2 = self._mod_w
        dt, B = w1.dtype, emb.shape[0]
        with _region("gemm"):
            h = torch.mm(F.silu(emb).reshape(B, -1).to(dt), w1.t(), out_dtype=torch.float32)
            h = h.view(B, w2.shape[0], -1).transpose(0, 1).to(dt)  # [84, B, Lr]
            y = torch.bmm(h, w2.transpose(1, 2), out_dtype=torch.float32)  # [84, B, 3D]
        return y + lora.reshape(1, B, -1)

    def _mods(self, p, emb, lora):
        """adaLN-LoRA modulation (shift, scale, gate) of the three sub-blocks of block p."""
        if self._mod_all is not None:  # computed for every block by this forward
            b = int(p.split(".")[1])
            return tuple(self._mod_all[3 * b + j].unsqueeze(1).chunk(3, dim=-1)
                         for j in range(3))
        w = self.w

        def mods(m):
            h = _linear(F.silu(emb), w[p + f"adaln_modulation_{m}.1.weight"])
            return (_linear(h, w[p + f"adaln_modulation_{m}.2.weight"]) + lora).chunk(3, dim=-1)

        return tuple(mods(m) for m in _SUBBLOCKS)

    def _mlp(self, p, h):
        dt = self.cfg.gemm_dtype
        w1 = self.w[p + "mlp.layer1.weight"]
        if self.fused_qkv and h.is_cuda and h.dtype == dt and h.is_contiguous():
            from .ops import gemm_gelu  # layer 1 + GELU in one GEMM (fp32 accumulator)
            with _region("gemm"):
                hid = gemm_gelu(h, w1)
        else:
            hid = self._gelu(_linear(h, w1, dt))
        return _linear(hid, self.w[p + "mlp.layer2.weight"], dt)

    # ---------------------------------------------------------- tokens mode (rows)
    def _segments(self, lo: int, hi: int, L: int):
        """Pieces (start, end, sample) of global rows [lo, hi), one sample each, with
        start/end relative to lo."""
        segs, r = [], lo
        while r < hi:
            b = r // L
            e = min(hi, (b + 1) * L)
            segs.append((r - lo, e - lo, b))
            r = e
        return segs

    def _ln_mod_rows(self, x, scale, shift, segs):
        """_ln_mod on local rows x [n, D] whose samples are given by segs."""
        parts = [self._ln_mod(x[s0:s1].unsqueeze(0), scale[b:b + 1], shift[b:b + 1])[0]
                 for s0, s1, b in segs]
        return parts[0] if len(parts) == 1 else torch.cat(parts)

    def _add_ln_rows(self, x, pending, scale, shift, segs):
        """_add_ln on local rows x [n, D] whose samples are given by segs."""
        if pending is None:
            return x, self._ln_mod_rows(x, scale, shift, segs)
        gate, y = pending
        if not x.is_cuda:
            x = torch.cat([x[s0:s1] + gate[b, 0] * y[s0:s1] for s0, s1, b in segs])
            return x, self._ln_mod_rows(x, scale, shift, segs)
        parts = [self._add_ln(x[s0:s1].unsqueeze(0), (gate[b:b + 1], y[s0:s1].unsqueeze(0)),
                              scale[b:b + 1], shift[b:b + 1])[1][0] for s0, s1, b in segs]
        return x, parts[0] if len(parts) == 1 else torch.cat(parts)

    def _by_rank_linear(self, h, w):
        """h [n, K] @ w[r]^T for every rank r -> [N, n, M] (the all-to-all send buffer)."""
        if h.is_cuda:
            with _region("gemm"):
                return torch.matmul(h.to(w.dtype), w.transpose(1, 2))
        return (h.to(w.dtype).float() @ w.float().transpose(1, 2)).to(w.dtype)

    def _a2a(self, t: torch.Tensor) -> torch.Tensor:
        """all_to_all_single over dim 0 (destination rank in, source rank out)."""
        import torch.distributed as dist
        out = torch.empty_like(t)
        t = t.contiguous()
        with _region("collective"):
            dist.all_to_all_single(out, t, group=self.group)
        return out

    def _a2a_buffers(self, B: int, L: int, device):
        """The peer buffers of the tokens layout for a [B, L] token grid (collective on first
        use and on a shape change): q/k/v operands of this rank's heads for self-attention
        (q0, k0, v0), the query of cross-attention (q1), and this rank's rows of all heads'
        attention outputs (o0 self, o1 cross)."""
        from .peer import PeerBuffers
        cfg, hl, hd, dt = self.cfg, self.h_local, self.cfg.head_dim, self.cfg.gemm_dtype
        n = B * L // self.world
        if self._a2a_bufs is None or self._a2a_key != (B, L):
            if self._a2a_bufs is not None:
                self._a2a_bufs.close()
            op = ((B * hl, L, hd), dt)
            out = ((n, cfg.heads * hd), dt)
            self._a2a_bufs = PeerBuffers({"q0": op, "k0": op, "v0": op, "q1": op, "o0": out,
                                          "o1": out}, device, self.group, self.rank, self.world)
            self._a2a_key = (B, L)
        return self._a2a_bufs

    def _attention_rows_peer(self, p, h_loc, B, L, ctx, freqs):
        """_attention_rows with the all-to-alls folded into the projection's and the
        attention's epilogues: projection GEMM (all heads, this rank's rows) -> each head's
        rows into its owner's q/k/v buffers -> barrier -> attention on this rank's heads ->
        each output row into its token owner's buffer -> barrier -> o-proj of this rank's
        rows."""
        from .ops import attention_core, qkv_projection_scatter
        cfg, N, r = self.cfg, self.world, self.rank
        hl, hd, dt = self.h_local, cfg.head_dim, cfg.gemm_dtype
        n = h_loc.shape[0]
        g = self._a2a_buffers(B, L, h_loc.device)
        h16 = h_loc.to(dt).contiguous()
        qw = self._norm32(p + ".q_norm.weight")
        if ctx is None:
            dest = [(g.ptr("q0", d), g.ptr("k0", d), g.ptr("v0", d)) for d in range(N)]
            with _region("qkv_fused"):
                qkv_projection_scatter(h16, self.w[p + ".qkv_all"], B, L, hl, r * n, dest, 3, 0,
                                       qw, self._norm32(p + ".k_norm.weight"), freqs, cfg.eps)
            qh, kh, vh, o = g.local["q0"], g.local["k0"], g.local["v0"], "o0"
        else:
            dest = [(g.ptr("q1", d), 0, 0) for d in range(N)]
            with _region("qkv_fused"):
                qkv_projection_scatter(h16, self.w[p + ".q_all"], B, L, hl, r * n, dest, 1, 0,
                                       qw, None, None, cfg.eps, True, False)
            entry = ctx if isinstance(ctx, dict) else self._context_entry(p, ctx, True)
            qh, kh, vh, o = g.local["q1"], entry["kh"], entry["vh"], "o1"
        with _region("collective"):
            g.barrier()
        with _region("attention"):
            attention_core(qh, kh, vh, B, hl, out_dtype=dt,
                           scatter=(g.ptrs(o), n, cfg.heads * hd, r * hl))
        with _region("collective"):
            g.barrier()
        return _linear(g.local[o], self.w[p + ".output_proj.weight"], dt)

    def _attention_rows(self, p, h_loc, B, L, ctx, freqs):
        """Head-parallel attention for local token rows h_loc [n, D] -> o-proj [n, D]."""
        if (self.peer_a2a and h_loc.is_cuda and L % 32 == 0 and h_loc.shape[0] % 32 == 0
                and (ctx is None or not isinstance(ctx, dict) or "kh" in ctx)):
            return self._attention_rows_peer(p, h_loc, B, L, ctx, freqs)
        cfg, N = self.cfg, self.world
        hl, hd, dt = self.h_local, cfg.head_dim, cfg.gemm_dtype
        n = h_loc.shape[0]
        if ctx is None:
            qkv = self._a2a(self._by_rank_linear(h_loc, self.w[p + ".qkv"]))  # [N, n, 3*hl*hd]
            qkv = qkv.view(B, L, 3, hl, hd)  # rows in global order: source rank r = rows r
            q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
            o = self._cross_or_self(p, q, None, freqs, (k, v))
        else:
            q = self._a2a(self._by_rank_linear(h_loc, self.w[p + ".q_by_rank"])).view(B, L, hl, hd)
            o = self._cross_or_self(p, q, ctx, None, None)
        # [B, L, hl, hd] = [N, n, hl*hd] by destination rank -> [N (source heads), n, hl*hd]
        o = self._a2a(o.reshape(N, n, hl * hd))
        o = o.permute(1, 0, 2).reshape(n, N * hl * hd)  # my rows, heads in order
        return _linear(o, self.w[p + ".output_proj.weight"], dt)

    def _block_rows(self, b, x, pending, emb, lora, ctx, freqs, B, L, segs):
        """One block on local rows.  pending: the previous block's MLP residual (gate, y),
        applied together with this block's first LayerNorm; returns (x, pending)."""
        p = f"blocks.{b}."
        (sh_sa, sc_sa, g_sa), (sh_ca, sc_ca, g_ca), (sh_m, sc_m, g_m) = self._mods(p, emb, lora)
        x, h = self._add_ln_rows(x, pending, sc_sa, sh_sa, segs)
        y = self._attention_rows(p + "self_attn", h, B, L, None, freqs)
        x, h = self._add_ln_rows(x, (g_sa, y), sc_ca, sh_ca, segs)
        y = self._attention_rows(p + "cross_attn", h, B, L, self._ctx_for(p, ctx), None)
        x, h = self._add_ln_rows(x, (g_ca, y), sc_m, sh_m, segs)
        return x, (g_m, self._mlp(p, h))

    # ---------------------------------------------------------- heads mode
    def _gather_oproj(self, o_local: torch.Tensor, w_o: torch.Tensor) -> torch.Tensor:
        """o_local [B, S, H/N, hd] -> o-proj of all heads [B, S, hidden] (fp32)."""
        B, S = o_local.shape[:2]
        cols = self.h_local * self.cfg.head_dim
        if self.world == 1:
            return _linear(o_local.reshape(B, S, cols), w_o, self.cfg.gemm_dtype)
        import torch.distributed as dist
        # gathered along dim 0 ([world * B, S, H/N, hd]); viewed as [world, B, ...]
        full = torch.empty((self.world * B,) + tuple(o_local.shape[1:]), dtype=o_local.dtype,
                           device=o_local.device)
        o_local = o_local.contiguous()
        with _region("collective"):
            dist.all_gather_into_tensor(full, o_local, group=self.group)
        # [world, B, S, H/N, hd] -> [B, S, hidden], rank r's heads at columns r*cols (the
        # order of w_o's input columns), then one GEMM with K = hidden: one transpose copy
        # instead of `world` GEMMs of K = cols summed in fp32.
        full = full.view((self.world,) + tuple(o_local.shape)).permute(1, 2, 0, 3, 4)
        return _linear(full.reshape(B, S, self.world * cols), w_o, self.cfg.gemm_dtype)

    def _gather_buffers(self, B: int, S: int, device):
        """The peer gather buffers for [B, S] tokens (collective on first use and on a shape
        change: every rank reaches it at the same attention)."""
        from .peer import GatherBuffers
        shape = (B, S, self.cfg.heads, self.cfg.head_dim)
        if self._gather is None or tuple(self._gather.bufs[0].shape) != shape:
            if self._gather is not None:
                self._gather.close()
            self._gather = GatherBuffers(shape, self.cfg.gemm_dtype, device, self.group,
                                         self.rank, self.world)
        return self._gather

    def close(self) -> None:
        """Releases the peer mappings of the gather / all-to-all buffers (N > 1)."""
        if self._gather is not None:
            self._gather.close()
            self._gather = None
        if self._a2a_bufs is not None:
            self._a2a_bufs.close()
            self._a2a_bufs, self._a2a_key = None, None

    def _fused(self, x: torch.Tensor) -> bool:
        """Whether x [B, S, K] can feed anima_qkv_projection (token count a multiple of 32)."""
        return self.fused_qkv and x.is_cuda and x.shape[1] % 32 == 0

    def _norm32(self, name: str) -> torch.Tensor:
        """An RMSNorm weight as the fp32 vector the fused kernels read (made once)."""
        t = self._w32.get(name)
        if t is None:
            t = self._w32[name] = self.w[name].float().contiguous()
        return t

    def _attention(self, p: str, x: torch.Tensor, ctx, freqs):
        """ctx: None (self-attention), the context tensor, or this block's entry of a
        context_cache (cross-attention K/V prepared for the whole sampling run)."""
        cfg = self.cfg
        B, S = x.shape[:2]
        hl, hd, dt = self.h_local, cfg.head_dim, cfg.gemm_dtype
        entry = None
        if ctx is not None and self._fused(x):
            entry = ctx if isinstance(ctx, dict) else self._context_entry(p, ctx, True)
        if self._fused(x) and (ctx is None or "kh" in entry):
            from .ops import attention_core, qkv_projection
            x16 = x.to(dt).contiguous()
            qw = self._norm32(p + ".q_norm.weight")
            with _region("qkv_fused"):
                if ctx is None:
                    qh, kh, vh = qkv_projection(x16, self.w[p + ".qkv"], hl, 3, 0, qw,
                                                self._norm32(p + ".k_norm.weight"), freqs,
                                                cfg.eps)
                else:
                    qh, _, _ = qkv_projection(x16, self.w[p + ".q_proj.weight"], hl, 1, 0, qw,
                                              None, None, cfg.eps, True, False)
                    kh, vh = entry["kh"], entry["vh"]
            if self.peer_gather and x.is_cuda:
                g = self._gather_buffers(B, S, x.device)
                i = 0 if ctx is None else 1  # self- and cross-attention alternate buffers
                mine = g.bufs[i][:, :, self.rank * hl:(self.rank + 1) * hl]
                with _region("attention"):
                    attention_core(qh, kh, vh, B, hl, out=mine, out_dtype=dt,
                                   peers=g.destinations(i, self.rank * hl * hd))
                with _region("collective"):
                    g.barrier()
                return _linear(g.bufs[i].view(B, S, cfg.hidden), self.w[p + ".output_proj.weight"],
                               dt)
            with _region("attention"):
                o = attention_core(qh, kh, vh, B, hl, out_dtype=dt)
            return self._gather_oproj(o, self.w[p + ".output_proj.weight"])
        if ctx is None:
            qkv = _linear(x, self.w[p + ".qkv"], dt).view(B, S, 3, hl, hd)
            q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        else:
            q = _linear(x, self.w[p + ".q_proj.weight"], dt).view(B, S, hl, hd)
        o = self._cross_or_self(p, q, None if ctx is None else ctx, freqs,
                                (k, v) if ctx is None else None)
        return self._gather_oproj(o, self.w[p + ".output_proj.weight"])

    def _cross_or_self(self, p, q, ctx, freqs, kv):
        """The attention call of one block: self-attention on (k, v) = kv, or
        cross-attention on ctx (a context tensor, or a cached entry)."""
        cfg = self.cfg
        dt = cfg.gemm_dtype
        qw, kw = self.w[p + ".q_norm.weight"], self.w[p + ".k_norm.weight"]
        if ctx is None:
            k, v = kv
            with _region("attention"):
                return self.attn_fn(q, k, v, qw, kw, freqs, eps=cfg.eps, out_dtype=dt, op_dtype=dt)
        entry = ctx if isinstance(ctx, dict) else self._context_entry(p, ctx)
        if "kh" in entry:  # operands already in the attention core's layout (GPU)
            from .ops import attention_cached_kv
            with _region("attention"):
                return attention_cached_kv(q, entry["kh"], entry["vh"], qw, eps=cfg.eps,
                                           out_dtype=dt)
        with _region("attention"):
            return self.attn_fn(q, entry["k"], entry["v"], qw, kw, None, eps=cfg.eps,
                                out_dtype=dt, op_dtype=dt)

    def _context_entry(self, p, ctx, keep_operands=False):
        """Cross-attention K/V of block prefix p for context ctx [B, N, ctx_dim]: the
        projection of this rank's heads, and with keep_operands (GPU, library attention)
        also their k-norm + head-major 16-bit operands, which then replace the K/V side of
        the prologue in every step."""
        cfg = self.cfg
        B, Skv = ctx.shape[:2]
        if keep_operands and self._fused(ctx):
            from .ops import qkv_projection
            with _region("qkv_fused"):
                _, kh, vh = qkv_projection(ctx.to(cfg.gemm_dtype).contiguous(), self.w[p + ".kv"],
                                           self.h_local, 2, 1, None,
                                           self._norm32(p + ".k_norm.weight"), None, cfg.eps,
                                           False, True)
            return {"kh": kh, "vh": vh}
        kv = _linear(ctx, self.w[p + ".kv"], cfg.gemm_dtype).view(B, Skv, 2, self.h_local,
                                                                 cfg.head_dim)
        entry = {"k": kv[:, :, 0], "v": kv[:, :, 1]}
        if keep_operands:
            from .ops import prologue
            _, kh, vh = prologue(None, entry["k"], entry["v"], None, self.w[p + ".k_norm.weight"],
                                 None, cfg.eps, False, True, cfg.gemm_dtype)
            entry = {"kh": kh, "vh": vh}
        return entry

    def context_cache(self, ctx_cond: torch.Tensor, ctx_uncond: torch.Tensor) -> Dict[str, dict]:
        """Cross-attention K/V of every block for the CFG pair's contexts (stacked [uncond,
        cond], the order euler_cfg_step uses).  The text context is the same in every step of
        a sampling run (anima_rt/scripts/sampling.py:127), while the reference projects and
        normalises its K/V in every step and block (numpy_dit.py:276-286); with the cache a
        step runs only the query side of each cross-attention."""
        from .ops import attention as _lib_attention
        ctx = torch.cat([ctx_uncond, ctx_cond], dim=0).float()
        keep = ctx.is_cuda and self.attn_fn is _lib_attention
        return {f"blocks.{b}.cross_attn": self._context_entry(f"blocks.{b}.cross_attn", ctx, keep)
                for b in range(self.cfg.blocks)}

    def _block(self, b: int, x, pending, emb, lora, ctx, freqs):
        """One block on the whole residual stream [B, L, D]; pending as in _block_rows."""
        p = f"blocks.{b}."
        (sh_sa, sc_sa, g_sa), (sh_ca, sc_ca, g_ca), (sh_m, sc_m, g_m) = self._mods(p, emb, lora)
        x, h = self._add_ln(x, pending, sc_sa, sh_sa)
        y = self._attention(p + "self_attn", h, None, freqs)
        x, h = self._add_ln(x, (g_sa, y), sc_ca, sh_ca)
        y = self._attention(p + "cross_attn", h, self._ctx_for(p, ctx), None)
        x, h = self._add_ln(x, (g_ca, y), sc_m, sh_m)
        return x, (g_m, self._mlp(p, h))

    @staticmethod
    def _ctx_for(p, ctx):
        """This block's context: the tensor itself, or its entry of a context_cache."""
        return ctx[p + "cross_attn"] if isinstance(ctx, dict) else ctx

    # ------------------------------------------------------------------ forward
    def forward(self, x: torch.Tensor, timesteps: torch.Tensor, context):
        """x [B, C, T, H, W] latent, timesteps [B], context [B, N, ctx_dim] (or the
        context_cache of that context) -> v, x's shape."""
        cfg, w = self.cfg, self.w
        B, C, T, Hh, Ww = x.shape
        ps, pt = cfg.patch, cfg.patch_t
        if Hh % ps or Ww % ps or T % pt:
            raise ValueError("latent must be a multiple of the patch size")
        mask = torch.zeros(B, 1, T, Hh, Ww, dtype=x.dtype, device=x.device)
        xm = torch.cat([x, mask], dim=1)
        Tp, Hp, Wp = T // pt, Hh // ps, Ww // ps
        # "b c (t r) (h m) (w n) -> b t h w (c r m n)"
        xp = xm.reshape(B, C + 1, Tp, pt, Hp, ps, Wp, ps).permute(0, 2, 4, 6, 1, 3, 5, 7)
        xp = xp.reshape(B, Tp * Hp * Wp, (C + 1) * pt * ps * ps)
        freqs = self._rope(Tp, Hp, Wp, x.device)
        sample = timestep_sinusoid(timesteps, cfg.hidden)  # [B, 1, hidden]
        lora = _linear(F.silu(_linear(sample, w["t_embedder.1.linear_1.weight"])),
                       w["t_embedder.1.linear_2.weight"])
        emb = F.rms_norm(sample, (cfg.hidden,), w["t_embedding_norm.weight"], cfg.eps)
        self._mod_all = (self._all_mods(emb, lora) if self._mod_w is not None and x.is_cuda
                         else None)
        ctx = context if isinstance(context, dict) else context.float()
        fm = _linear(_linear(F.silu(emb), w["final_layer.adaln_modulation.1.weight"]),
                     w["final_layer.adaln_modulation.2.weight"])
        shift, scale = (fm + lora[:, :, :2 * cfg.hidden]).chunk(2, dim=-1)
        L = Tp * Hp * Wp
        if self.seq:
            R = B * L
            if R % self.world:
                raise ValueError("B * tokens must divide evenly over ranks")
            n = R // self.world
            lo = self.rank * n
            segs = self._segments(lo, lo + n, L)
            h = _linear(xp.reshape(R, -1)[lo:lo + n], w["x_embedder.proj.1.weight"])  # [n, hidden]
            pending = None
            for b in range(cfg.blocks):
                h, pending = self._block_rows(b, h, pending, emb, lora, ctx, freqs, B, L, segs)
            h = self._add_ln_rows(h, pending, scale, shift, segs)[1]
            part = _linear(h, w["final_layer.linear.weight"])  # [n, p*p*t*C]
            import torch.distributed as dist
            out = torch.empty((R, part.shape[1]), dtype=part.dtype, device=part.device)
            part = part.contiguous()
            with _region("collective"):
                dist.all_gather_into_tensor(out, part, group=self.group)
            out = out.view(B, L, -1)
        else:
            h = _linear(xp, w["x_embedder.proj.1.weight"])  # [B, L, hidden]
            pending = None
            for b in range(cfg.blocks):
                h, pending = self._block(b, h, pending, emb, lora, ctx, freqs)
            h = self._add_ln(h, pending, scale, shift)[1]
            out = _linear(h, w["final_layer.linear.weight"])  # [B, L, p*p*t*C]
        # "B T H W (p1 p2 t C) -> B C (T t) (H p1) (W p2)"
        out = out.reshape(B, Tp, Hp, Wp, ps, ps, pt, cfg.out_channels)
        out = out.permute(0, 7, 1, 6, 2, 4, 3, 5).reshape(B, cfg.out_channels, T, Hh, Ww)
        return out

    def euler_cfg_step(self, x: torch.Tensor, sigma, sigma_next, ctx_cond: torch.Tensor,
                       ctx_uncond: torch.Tensor, cfg_scale: float, ctx_cache: dict = None):
        """One EulerSampler step (sampling.py:121-138): CFG pair [uncond, cond] in one
        batch, v = v_u + cfg (v_c - v_u), x' = x + v (sigma_next - sigma).
        x [1, C, H, W] -> [1, C, H, W].  sigma / sigma_next are numbers or one-element
        device tensors (a captured step then serves every step of a schedule);
        ctx_cache: context_cache(ctx_cond, ctx_uncond), used instead of the contexts."""
        xb = x[:, :, None].expand(2, -1, -1, -1, -1).contiguous()
        ctx = ctx_cache if ctx_cache is not None else torch.cat([ctx_uncond, ctx_cond], dim=0)
        if torch.is_tensor(sigma):
            t = sigma.reshape(1).float().expand(2)
        else:
            t = torch.full((2,), sigma, dtype=torch.float32, device=x.device)
        v = self.forward(xb, t, ctx)
        v_cfg = v[0:1] + cfg_scale * (v[1:2] - v[0:1])
        return x + v_cfg[:, :, 0] * (sigma_next - sigma)


class StepGraph:
    """One ``AnimaDiT.euler_cfg_step`` captured as a CUDA graph.

    A step issues about fifty launches per block (GEMMs, the library's kernels, torch
    elementwise ops and, on N GPUs, the collectives); once the per-GPU work of a step drops
    to a few milliseconds, issuing them from Python costs more than running them.  Replaying
    the captured graph issues the whole step at once.  The graph owns static copies of the
    latent and both contexts: ``__call__`` copies new values into them (on the current
    stream), replays, and returns the static output tensor (overwritten by the next call).
    ``sigma``, ``sigma_next`` and ``cfg_scale`` are fixed at capture.  On N ranks every rank
    must build and replay its graph in the same order (the collectives are captured), and
    drop it before the process group is destroyed."""

    def __init__(self, model: "AnimaDiT", x, sigma: float, sigma_next: float, ctx_cond,
                 ctx_uncond, cfg_scale: float, warmup: int = 2):
        self.x, self.cc, self.cu = x.clone(), ctx_cond.clone(), ctx_uncond.clone()
        args = (sigma, sigma_next)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # first calls allocate caches outside the capture
            for _ in range(warmup):
                model.euler_cfg_step(self.x, *args, self.cc, self.cu, cfg_scale)
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = model.euler_cfg_step(self.x, *args, self.cc, self.cu, cfg_scale)

    def __call__(self, x=None, ctx_cond=None, ctx_uncond=None):
        for dst, src in ((self.x, x), (self.cc, ctx_cond), (self.cu, ctx_uncond)):
            if src is not None:
                dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.out



def profile_step(model: "AnimaDiT", x, sigma: float, sigma_next: float, ctx_cond, ctx_uncond,
                 cfg_scale: float) -> dict:
    """One eager ``euler_cfg_step`` with CUDA events around every GEMM, attention call (fused
    prologue + attention kernels), fused LayerNorm/residual/GELU pass and collective.
    Returns the step's device time and each category's total in ms and as a share of it;
    "other" is the rest (torch elementwise ops, launch gaps, waits).  A collective's time
    includes its wait for the slowest rank.  Event pairs add a little overhead, so these are
    shares of an eager step, not of the graph-replayed one."""
    global _REGIONS
    torch.cuda.synchronize()
    _REGIONS = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        e0.record()
        model.euler_cfg_step(x, sigma, sigma_next, ctx_cond, ctx_uncond, cfg_scale)
        e1.record()
        torch.cuda.synchronize()
        regions, _REGIONS = _REGIONS, None
    finally:
        _REGIONS = None
    total = e0.elapsed_time(e1)
    cats: Dict[str, float] = {}
    counts: Dict[str, int] = {}
    for cat, a, b in regions:
        cats[cat] = cats.get(cat, 0.0) + a.elapsed_time(b)
        counts[cat] = counts.get(cat, 0) + 1
    cats["other"] = max(0.0, total - sum(cats.values()))
    return {"step_ms": round(total, 3),
            "ms": {k: round(v, 3) for k, v in cats.items()},
            "share": {k: round(v / total, 4) for k, v in cats.items()},
            "calls": counts}
