"""CPU stand-in for the attention op, for CPU tests of the DiT harness only.

Same signature as anima_attn.attention; computes q/k RMSNorm, the reference RoPE
(src/predict2.py:31-38) and fp32 torch SDPA.  Test infrastructure: the product path has
no CPU attention."""
import torch
import torch.nn.functional as F


def rope(t, freqs):
    # predict2.apply_rotary_pos_emb on t [B, S, H, D] with freqs [S, D/2, 2, 2]
    f = freqs[None, :, None]
    t_ = t.reshape(*t.shape[:-1], 2, -1).movedim(-2, -1).unsqueeze(-2)
    t_ = t_ if t_.dtype == torch.float64 else t_.float()
    f = f.to(t_.dtype)
    out = f[..., 0] * t_[..., 0] + f[..., 1] * t_[..., 1]
    return out.movedim(-1, -2).reshape(*t.shape)


def cpu_attention(q, k, v, q_norm_w=None, k_norm_w=None, rope_freqs=None, kv_valid_len=None,
                  norm_q=True, norm_k=True, causal=False, scale=None, eps=1e-6,
                  out_dtype=torch.float32, **_):
    d = q.shape[-1]
    q = F.rms_norm(q.float(), (d,), q_norm_w, eps) if norm_q else q.float()
    k = F.rms_norm(k.float(), (d,), k_norm_w, eps) if norm_k else k.float()
    if rope_freqs is not None:
        q, k = rope(q, rope_freqs), rope(k, rope_freqs)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                       v.float().transpose(1, 2), scale=scale)
    return o.transpose(1, 2).contiguous().to(out_dtype)
