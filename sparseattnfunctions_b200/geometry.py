"""Token geometry of CogVideoX-style DiT attention.

The reference hard-codes the CogVideoX-2B layout (226 text tokens, then a
13 x 30 x 45 (t, h, w) video grid: MergeAttention.py:16,26-31,
merge_unmerge.py:83,121, SmartAttention.py:15-26, mask_related.py:100-101)
and the 1.5-5B one (224 text, 11 x 48 x 85: combined_attn.py:17-41,
partern_attention.py:10-16).  Every shape constant here is derived from one
``VideoGeometry`` instead.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass(frozen=True)
class VideoGeometry:
    text_len: int = 226
    frames: int = 13
    height: int = 30
    width: int = 45

    @property
    def frame_len(self) -> int:
        return self.height * self.width

    @property
    def video_len(self) -> int:
        return self.frames * self.frame_len

    @property
    def seq_len(self) -> int:
        return self.text_len + self.video_len

    def text_blocks(self, block: int) -> int:
        """Blocks that contain at least one text token (text comes first)."""
        return math.ceil(self.text_len / block)

    def num_blocks(self, block: int) -> int:
        return math.ceil(self.seq_len / block)


COGVIDEOX_2B = VideoGeometry(226, 13, 30, 45)
COGVIDEOX_2B_LONG = VideoGeometry(226, 25, 30, 45)   # 33976 tokens
COGVIDEOX_15_5B = VideoGeometry(224, 11, 48, 85)


# --------------------------------------------------------------------------- frame-band masks

def frame_band_ranges(geo: VideoGeometry, diag: int = 1, device="cpu"):
    """int32 [S, 4] key intervals of the frame-band (block-tridiagonal) mask
    of SmartAttention (SmartAttention.py:30-43 mask_mod; :130-143 per-frame
    key sets): text rows see every key; a video row of frame i sees
    [0, text + frame_len) (the text and the first frame) and the frames
    i - diag .. i + diag.  Row r sees keys [x, y) U [z, w)."""
    import torch

    S, T, F = geo.seq_len, geo.text_len, geo.frame_len
    r = torch.zeros(S, 4, dtype=torch.int64)
    r[:, 1] = S
    fr = (torch.arange(T, S) - T) // F
    r[T:, 1] = min(S, T + F)
    r[T:, 2] = (T + (fr - diag) * F).clamp(0, S)
    r[T:, 3] = (T + (fr + diag + 1) * F).clamp(0, S)
    return r.to(torch.int32).to(device)


def video_token_perm(geo: VideoGeometry, device="cpu"):
    """(perm, inv) int32 [S]: ``perm[p]`` is the natural index of the token
    at position p of the (h, w, t)-ordered sequence (text first, unchanged);
    ``inv`` the inverse.  x[perm] is SmartAttention's ``process`` (video
    tokens (t h w) -> (h w t), SmartAttention.py:9-14), x[inv] its
    ``process_back`` (:16-27)."""
    import torch

    T, HW, F = geo.text_len, geo.frame_len, geo.frames
    p = torch.arange(geo.video_len)
    hw, t = p // F, p % F            # position p = hw * frames + t
    perm = torch.cat([torch.arange(T), T + t * HW + hw])
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel())
    return perm.to(torch.int32).to(device), inv.to(torch.int32).to(device)


def ranges_block_mask(ranges, Sk: int, block_m: int, block_n: int):
    """bool [ceil(Sq/block_m), ceil(Sk/block_n)]: key blocks that some row of
    the query block can see under ``ranges`` (int32 [Sq, 4])."""
    import torch

    r = ranges.to(torch.int64)
    Sq = r.shape[0]
    nbq, nbk = -(-Sq // block_m), -(-Sk // block_n)
    cols = torch.arange(nbk, device=r.device)
    cover = torch.zeros(Sq, nbk, dtype=torch.bool, device=r.device)
    for lo, hi in ((r[:, 0], r[:, 1]), (r[:, 2], r[:, 3])):
        hi = hi.clamp(max=Sk)
        ok = (hi > lo)[:, None]
        cover |= ok & (cols[None] >= (lo // block_n)[:, None]) & (cols[None] <= ((hi - 1) // block_n)[:, None])
    pad = nbq * block_m - Sq
    if pad:
        cover = torch.cat([cover, torch.zeros(pad, nbk, dtype=torch.bool, device=r.device)])
    return cover.view(nbq, block_m, nbk).any(dim=1)
