"""Seeded synthetic fixed-camera streams for benchmarks and tests.

Stand-in for real camera footage (no dataset is used).  Per stream:

* background: uniform noise U(0, 255) blurred with a Gaussian of sigma 3, kept in float;
* every frame: background + N(0, 2) sensor noise, then ``n_rects`` filled rectangles with
  sides 40-120 px moving 2-8 px per frame and bouncing off the borders, clipped and
  rounded to uint8 RGB.

``normalise`` turns uint8 RGB frames into the engine input exactly as Sarbon's
``SarbonVideo._prep`` does (sarbon/inference/video.py:22-23, 96-99, 108):
``(x - MEAN) / STD`` in fp32, then rounded to fp16.

``forced_change`` builds the change-rate sweep: a new frame whose blocks, chosen by a
seeded random block mask covering an exact fraction of blocks, hold uniform random
uint8 content.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

MEAN = np.array([0.485, 0.456, 0.406], np.float32) * 255
STD = np.array([0.229, 0.224, 0.225], np.float32) * 255


def normalise(frames_u8_rgb, dtype=torch.float16):
    """uint8 RGB [..., 3] -> (x - MEAN) / STD in fp32 -> dtype."""
    mean = torch.as_tensor(MEAN, device=frames_u8_rgb.device)
    std = torch.as_tensor(STD, device=frames_u8_rgb.device)
    return ((frames_u8_rgb.float() - mean) / std).to(dtype)


def _gauss_blur(x, sigma):
    r = int(math.ceil(3 * sigma))
    t = torch.arange(-r, r + 1, device=x.device, dtype=torch.float32)
    k = torch.exp(-0.5 * (t / sigma) ** 2)
    k = (k / k.sum()).view(1, 1, 1, -1)
    c = x.shape[1]
    x = F.pad(x, (r, r, 0, 0), mode="reflect")
    x = F.conv2d(x, k.expand(c, 1, 1, -1), groups=c)
    x = F.pad(x, (0, 0, r, r), mode="reflect")
    return F.conv2d(x, k.view(1, 1, -1, 1).expand(c, 1, -1, 1), groups=c)


class Streams:
    """``n`` independent camera streams of ``h x w`` RGB frames (uint8 [n, h, w, 3])."""

    def __init__(self, n, h, w, seed=0, n_rects=3, noise=2.0, device="cpu"):
        self.n, self.h, self.w, self.noise = n, h, w, noise
        self.dev = torch.device(device)
        self.gen = torch.Generator(device=self.dev).manual_seed(seed)
        g = self.gen
        bg = torch.rand(n, 3, h, w, generator=g, device=self.dev) * 255.0
        self.bg = _gauss_blur(bg, 3.0).permute(0, 2, 3, 1).contiguous()  # [n, h, w, 3] float
        self.size = torch.randint(40, 121, (n, n_rects, 2), generator=g, device=self.dev)
        lim = torch.tensor([h, w], device=self.dev) - self.size
        self.pos = torch.rand(n, n_rects, 2, generator=g, device=self.dev) * lim
        speed = 2.0 + torch.rand(n, n_rects, 2, generator=g, device=self.dev) * 6.0
        sign = torch.where(torch.rand(n, n_rects, 2, generator=g, device=self.dev) < 0.5, -1.0, 1.0)
        self.vel = speed * sign
        self.color = torch.randint(0, 256, (n, n_rects, 3), generator=g, device=self.dev).float()

    def next(self):
        """Advance every stream by one frame; returns uint8 [n, h, w, 3] RGB."""
        lim = (torch.tensor([self.h, self.w], device=self.dev) - self.size).float()
        self.pos += self.vel
        bounce = (self.pos < 0) | (self.pos > lim)
        self.vel = torch.where(bounce, -self.vel, self.vel)
        self.pos = torch.minimum(torch.clamp(self.pos, min=0.0), lim)
        f = self.bg.clone()
        if self.noise:
            f += torch.randn(f.shape, generator=self.gen, device=self.dev) * self.noise
        pos = self.pos.round().long().tolist()
        size = self.size.tolist()
        for s in range(self.n):
            for r, ((y, x), (hh, ww)) in enumerate(zip(pos[s], size[s])):
                f[s, y:y + hh, x:x + ww] = self.color[s, r]
        return f.clamp_(0, 255).round_().to(torch.uint8)


def forced_change(prev_u8, frac, block, seed):
    """Copy of ``prev_u8`` [n, h, w, 3] where exactly round(frac * n_blocks) blocks, chosen
    by a seeded permutation, hold fresh uniform random uint8 content.  Returns
    (frames, block_mask [n, hb, wb] bool)."""
    n, h, w, _ = prev_u8.shape
    hb, wb = h // block, w // block
    nb = n * hb * wb
    g = torch.Generator(device="cpu").manual_seed(seed)
    k = int(round(frac * nb))
    pick = torch.randperm(nb, generator=g)[:k]
    mask = torch.zeros(nb, dtype=torch.bool)
    mask[pick] = True
    mask = mask.view(n, hb, wb)
    out = prev_u8.clone()
    noise = torch.randint(0, 256, prev_u8.shape, generator=g, dtype=torch.uint8).to(prev_u8.device)
    m = mask.to(prev_u8.device).repeat_interleave(block, 1).repeat_interleave(block, 2)[..., None]
    out = torch.where(m, noise, out)
    return out, mask
