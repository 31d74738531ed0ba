"""3D (t, h, w) rotary table of the Anima DiT, built on the device.

Restates VideoRopePosition3DEmb (src/position_embedding.py:80-98 for the frequency
split and NTK factors, 100-163 for generate_embeddings) in fp32 torch ops of the same
order, so the table matches the reference's to within one fp32 ulp of cos/sin:

  head_dim 128 -> dim_h = dim_w = 42, dim_t = 44 (21 + 21 + 22 = 64 pairs)
  ntk_axis   = ratio_axis ** (dim_axis / (dim_axis - 2))
  freq_axis  = 1 / (theta * ntk_axis) ** (arange(0, dim_axis, 2) / dim_axis)
  token s = (t * H + h) * W + w (w fastest); pair blocks ordered [t | h | w]
  entry [s, p] = [[cos, -sin], [sin, cos]] of angle (position * freq)

The Anima pipeline uses h/w extrapolation ratio 4.0, t ratio 1.0, theta 10000 and
no fps modulation (image case), which are the defaults here.
"""
from __future__ import annotations

import torch


def rope_freqs_3d(T: int, H: int, W: int, head_dim: int = 128, h_ratio: float = 4.0,
                  w_ratio: float = 4.0, t_ratio: float = 1.0, theta: float = 10000.0,
                  device=None) -> torch.Tensor:
    """Returns the fp32 table [(T*H*W), head_dim/2, 2, 2]."""
    dim_h = head_dim // 6 * 2
    dim_w = dim_h
    dim_t = head_dim - 2 * dim_h
    sp = torch.arange(0, dim_h, 2, device=device)[: dim_h // 2].float() / dim_h
    tp = torch.arange(0, dim_t, 2, device=device)[: dim_t // 2].float() / dim_t
    h_theta = theta * h_ratio ** (dim_h / (dim_h - 2))
    w_theta = theta * w_ratio ** (dim_w / (dim_w - 2))
    t_theta = theta * t_ratio ** (dim_t / (dim_t - 2))
    fh = 1.0 / (h_theta ** sp)
    fw = 1.0 / (w_theta ** sp)
    ft = 1.0 / (t_theta ** tp)
    seq = torch.arange(max(H, W, T), dtype=torch.float, device=device)

    def rot(ang):  # [n, pairs] -> [n, pairs, 4] = cos, -sin, sin, cos
        c, s = torch.cos(ang), torch.sin(ang)
        return torch.stack([c, -s, s, c], dim=-1)

    eh = rot(torch.outer(seq[:H], fh))  # [H, 21, 4]
    ew = rot(torch.outer(seq[:W], fw))  # [W, 21, 4]
    et = rot(torch.outer(seq[:T], ft))  # [T, 22, 4]
    full = torch.cat([
        et[:, None, None].expand(T, H, W, et.shape[1], 4),
        eh[None, :, None].expand(T, H, W, eh.shape[1], 4),
        ew[None, None, :].expand(T, H, W, ew.shape[1], 4),
    ], dim=-2)
    return full.reshape(T * H * W, head_dim // 2, 2, 2).contiguous()
