"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The reference publishes no dataset for this path; these generators stand in
for real activations.  Everything is drawn on the CPU from an explicit
``torch.Generator`` seed (so every machine gets the same values) and then
moved to the requested device.

* ``config1_qkv``: B1 H2 S2048 D64 fp32, q/k/v ~ N(0,1)/sqrt(D) drawn in the
  order q, k, v from one generator (seed 0).
* ``video_qkv``: CogVideoX-shaped q/k/v.  Text rows ~ N(0,1).  Video q and k
  are a smooth random field plus noise: N(0,1) values on a coarse
  (2, 4, 4)-cell grid, nearest-upsampled to the (t, h, w) grid, plus
  0.5 * N(0,1).  v ~ N(0,1).
* ``video_hidden``: [B, video_len, C] hidden states from the same recipe.
"""
from __future__ import annotations

import math

import torch

from .geometry import VideoGeometry

CELL = (2, 4, 4)


def config1_qkv(device="cpu", seed: int = 0, B=1, H=2, S=2048, D=64):
    g = torch.Generator().manual_seed(seed)
    scale = 1.0 / math.sqrt(D)
    q = torch.randn(B, H, S, D, generator=g) * scale
    k = torch.randn(B, H, S, D, generator=g) * scale
    v = torch.randn(B, H, S, D, generator=g) * scale
    return q.to(device), k.to(device), v.to(device)


def _smooth_field(g: torch.Generator, lead: tuple, geo: VideoGeometry, D: int) -> torch.Tensor:
    """[*lead, video_len, D] nearest-upsampled coarse N(0,1) field + 0.5 N(0,1)."""
    ct, ch, cw = (math.ceil(geo.frames / CELL[0]), math.ceil(geo.height / CELL[1]),
                  math.ceil(geo.width / CELL[2]))
    coarse = torch.randn(*lead, ct, ch, cw, D, generator=g)
    it = torch.arange(geo.frames) // CELL[0]
    ih = torch.arange(geo.height) // CELL[1]
    iw = torch.arange(geo.width) // CELL[2]
    fine = coarse[..., it, :, :, :][..., :, ih, :, :][..., :, :, iw, :]
    fine = fine.reshape(*lead, geo.video_len, D)
    return fine + 0.5 * torch.randn(*lead, geo.video_len, D, generator=g)


def video_qkv(geo: VideoGeometry, B=2, H=30, D=64, dtype=torch.bfloat16, device="cpu",
              seed: int = 1234):
    """q, k, v [B, H, text+video, D] in ``dtype`` on ``device``."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for name in ("q", "k", "v"):
        text = torch.randn(B, H, geo.text_len, D, generator=g)
        if name == "v":
            video = torch.randn(B, H, geo.video_len, D, generator=g)
        else:
            video = _smooth_field(g, (B, H), geo, D)
        out.append(torch.cat([text, video], dim=2).to(dtype).to(device))
    return tuple(out)


def video_hidden(geo: VideoGeometry, B=2, C=1920, dtype=torch.bfloat16, device="cpu",
                 seed: int = 4321):
    """[B, video_len, C] hidden states (smooth field + noise)."""
    g = torch.Generator().manual_seed(seed)
    return _smooth_field(g, (B,), geo, C).to(dtype).to(device)
