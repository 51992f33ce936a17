"""Drop-in for special_attentions/SildingTileAttention.py: sliding tile
attention (STA).

The reference (SildingTileAttention.py:18-140) reorders the video tokens tile
by tile (tiles of 13 x 3 x 3 tokens on the 13 x 30 x 45 CogVideoX-2B grid),
lets every video query see the text and the tiles inside a 1 x 9 x 9 tile
window around its own tile (the window centre clamped away from the canvas
edges), lets text queries see everything, and runs flex_attention with that
block mask.

Here every 117-token tile is placed in its own 128-row block and the text in
the first blocks (``saf_permute_tokens`` with zero-filled padding rows), so
the tile window is an exact block list: the block-sparse sm_100a kernel runs
it with a -inf bias on the padding key columns, and the output rows are
gathered back to the original order.  The layout and block list are built
once per device.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .. import kernels

DEFAULT_CONFIG = {"kernel_size": (1, 9, 9), "tile_size": (13, 3, 3), "img_size": (13, 30, 45),
                  "text_length": 226}


def sta_layout(config: dict, block: int = 128):
    """(pad_perm, unpad_perm, key_bias, block_mask) of the padded tile layout.

    pad_perm [S_pad]: original token index at each padded position (-1 for
    padding); unpad_perm [S]: padded position of each original token;
    key_bias [S_pad]: 0 / -inf; block_mask [nb, nb]: the tile-window mask."""
    T, Hc, W = config["img_size"]
    tt, th, tw = config["tile_size"]
    kt, kh, kw = config["kernel_size"]
    L = config["text_length"]
    nt, nh, nw = T // tt, Hc // th, W // tw
    n_tile = tt * th * tw
    if n_tile > block or nt * tt != T or nh * th != Hc or nw * tw != W:
        raise ValueError("tiles must divide the canvas and fit in one block")
    Lp = -(-L // block) * block
    tiles = nt * nh * nw
    S, S_pad = L + T * Hc * W, Lp + tiles * block
    idx = torch.arange(T * Hc * W).reshape(nt, tt, nh, th, nw, tw).permute(0, 2, 4, 1, 3, 5).reshape(tiles, n_tile)
    pad_perm = torch.full((S_pad,), -1, dtype=torch.int64)
    pad_perm[:L] = torch.arange(L)
    slots = Lp + torch.arange(tiles)[:, None] * block + torch.arange(n_tile)[None, :]
    pad_perm[slots.reshape(-1)] = L + idx.reshape(-1)
    unpad_perm = torch.empty(S, dtype=torch.int64)
    real = pad_perm >= 0
    unpad_perm[pad_perm[real]] = torch.nonzero(real).reshape(-1)
    key_bias = torch.where(real, 0.0, float("-inf")).to(torch.float32)
    tb = Lp // block
    nb = tb + tiles
    k = torch.arange(tiles)
    t_t, t_h, t_w = k // (nh * nw), (k % (nh * nw)) // nw, k % nw
    clamp = lambda x, lo, hi: torch.minimum(torch.maximum(x, torch.tensor(lo)), torch.tensor(hi))
    ct, ch, cw = clamp(t_t, kt // 2, (nt - 1) - kt // 2), clamp(t_h, kh // 2, (nh - 1) - kh // 2), \
        clamp(t_w, kw // 2, (nw - 1) - kw // 2)
    win = ((ct[:, None] - t_t[None, :]).abs() <= kt // 2) & ((ch[:, None] - t_h[None, :]).abs() <= kh // 2) & \
          ((cw[:, None] - t_w[None, :]).abs() <= kw // 2)
    mask = torch.zeros(nb, nb, dtype=torch.bool)
    mask[:tb, :] = True       # text queries see every key
    mask[tb:, :tb] = True     # video queries see the text
    mask[tb:, tb:] = win
    return pad_perm.to(torch.int32), unpad_perm.to(torch.int32), key_bias, mask


class SildingTileAttention:
    def __init__(self, config: Optional[dict] = None, block: int = 128):
        self.config = dict(config or DEFAULT_CONFIG)
        self.block = block
        self._static = {}

    def _layout(self, dev, B, H):
        key = (dev, B, H)
        if key not in self._static:
            pad_perm, unpad_perm, bias, mask = sta_layout(self.config, self.block)
            nb = mask.shape[0]
            csr = kernels.mask_to_csr(mask.to(dev)[None, None].expand(B, H, nb, nb).contiguous(), self.block,
                                      self.block, dense_rows=-(-self.config["text_length"] // self.block))
            self._static[key] = (pad_perm.to(dev), unpad_perm.to(dev), bias.to(dev), csr)
        return self._static[key]

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        B, H, S, D = q.shape
        pad_perm, unpad_perm, bias, csr = self._layout(q.device, B, H)
        if S != unpad_perm.numel():
            raise ValueError(f"sequence length {S} does not match the configuration ({unpad_perm.numel()})")
        qp, kp, vp = (kernels.permute_tokens(t, pad_perm) for t in (q, k, v))
        op = kernels.bsa_fwd(qp, kp, vp, csr, 1.0 / math.sqrt(D), kv_bias=bias)
        return kernels.permute_tokens(op, unpad_perm)

    def __call__(self, q, k, v):
        return self.forward(q, k, v)
