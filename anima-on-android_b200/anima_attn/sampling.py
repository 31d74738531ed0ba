"""The denoising loop of the reference sampler, on the device.

Restates, around AnimaDiT:
  ZImageScheduler.get_sigmas   anima_rt/scripts/sampling.py:69-87   sigma schedule
                               sigma = shift * t / (1 + (shift - 1) t), t = linspace(d, 0, n+1)
  EulerSampler.sample          anima_rt/scripts/sampling.py:110-140 CFG pair per step,
                               x += (v_u + cfg (v_c - v_u)) (sigma_next - sigma)
  run_ksampler                 anima_rt/scripts/sampling.py:183-209 schedule + seeded noise
                               + sampler

EulerCFGSampler keeps the latent on the device for the whole run.  The text contexts do
not change between steps, so the cross-attention K/V of every block are projected and
normalised once per run (AnimaDiT.context_cache) instead of once per step as in the
reference (numpy_dit.py:276-286).  With graph=True one Euler+CFG step is captured as a CUDA
graph whose sigma pair is read from device memory and whose result overwrites the latent
in place, so every step of the schedule replays the same graph.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch


def z_image_sigmas(steps: int, denoise: float = 1.0, shift: float = 3.0) -> np.ndarray:
    """ZImageScheduler.get_sigmas (sampling.py:69-87): steps + 1 fp32 sigmas, descending to 0,
    computed in fp32 numpy as the reference does, so the values are the same bits."""
    start = np.float32(0.0) + (np.float32(1.0) - np.float32(0.0)) * np.float32(denoise)
    t = np.linspace(start, 0.0, steps + 1, dtype=np.float32)
    return (np.float32(shift) * t / (np.float32(1.0) + (np.float32(shift) - 1.0) * t)).astype(np.float32)


def seeded_noise(seed: int, H: int, W: int, channels: int = 16) -> np.ndarray:
    """The starting latent of run_ksampler (sampling.py:198-199)."""
    return np.random.default_rng(seed).standard_normal((1, channels, H, W), dtype=np.float32)


class EulerCFGSampler:
    """EulerSampler.sample for an AnimaDiT: latent [1, C, H, W] and both contexts [1, N,
    ctx_dim] on the model's device.  ``cfg_scale`` is fixed per sampler (as in a captured
    graph).  On N ranks every rank builds and runs its sampler in the same order (the
    collectives are captured), and drops it before the process group is destroyed."""

    def __init__(self, model, ctx_cond: torch.Tensor, ctx_uncond: torch.Tensor, cfg_scale: float,
                 latent_shape, graph: bool = True, cache_context: bool = True,
                 warmup: int = 2):
        self.model, self.cfg_scale = model, float(cfg_scale)
        dev = ctx_cond.device
        self.cc, self.cu = ctx_cond.clone(), ctx_uncond.clone()
        self.x = torch.zeros(latent_shape, device=dev, dtype=torch.float32)
        self.sig = torch.zeros(1, device=dev, dtype=torch.float32)
        self.sig_next = torch.zeros(1, device=dev, dtype=torch.float32)
        self.cache = model.context_cache(self.cc, self.cu) if cache_context else None
        self.graph = self.ctx_graph = None
        if graph:
            if not self.x.is_cuda:
                raise ValueError("graph capture needs CUDA tensors")
            self.sig.fill_(1.0)
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):  # first calls allocate caches outside the capture
                for _ in range(warmup):
                    self._step(self.x.clone())
                    if self.cache is not None:
                        self._fill_cache()
            torch.cuda.current_stream().wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.x.copy_(self._step(self.x))
            if self.cache is not None:  # the per-run precompute, replayed in one launch too
                self.ctx_graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.ctx_graph):
                    self._fill_cache()

    def _fill_cache(self):
        fresh = self.model.context_cache(self.cc, self.cu)
        for key, entry in fresh.items():
            for name, t in entry.items():
                self.cache[key][name].copy_(t)

    def _step(self, x):
        return self.model.euler_cfg_step(x, self.sig, self.sig_next, self.cc, self.cu,
                                         self.cfg_scale, ctx_cache=self.cache)

    def refresh_context(self, ctx_cond: torch.Tensor, ctx_uncond: torch.Tensor) -> None:
        """New prompts for the next run: copies them into the sampler's buffers and rebuilds
        the K/V cache in place (the captured graph keeps reading the same tensors)."""
        self.cc.copy_(ctx_cond)
        self.cu.copy_(ctx_uncond)
        if self.ctx_graph is not None:
            self.ctx_graph.replay()
        elif self.cache is not None:
            self._fill_cache()

    def sample(self, noise: torch.Tensor, sigmas) -> torch.Tensor:
        """Run the loop over ``sigmas`` (steps + 1 values) from ``noise`` [1, C, H, W];
        returns the final latent (the sampler's own buffer, overwritten by the next call)."""
        sig = torch.as_tensor(np.asarray(sigmas, dtype=np.float32)).to(self.x.device)
        self.x.copy_(noise)
        for i in range(sig.numel() - 1):
            self.sig.copy_(sig[i:i + 1])
            self.sig_next.copy_(sig[i + 1:i + 2])
            if self.graph is not None:
                self.graph.replay()
            else:
                self.x.copy_(self._step(self.x))
        return self.x


def run_ksampler(model, ctx_cond: torch.Tensor, ctx_uncond: torch.Tensor, H: int, W: int,
                 steps: int = 3, cfg: float = 5.0, seed: int = 6666, denoise: float = 1.0,
                 shift: float = 3.0, graph: bool = True,
                 sampler: Optional[EulerCFGSampler] = None) -> torch.Tensor:
    """run_ksampler (sampling.py:183-209) with the z_image schedule and the Euler sampler:
    seeded noise, the sigma schedule, then the loop.  Returns [1, 16, H, W] fp32."""
    dev = ctx_cond.device
    noise = torch.from_numpy(seeded_noise(seed, H, W)).to(dev)
    s = sampler or EulerCFGSampler(model, ctx_cond, ctx_uncond, cfg, noise.shape, graph=graph)
    return s.sample(noise, z_image_sigmas(steps, denoise, shift)).clone()
