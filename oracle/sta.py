"""SildingTileAttention restated on the CPU -- TEST INFRASTRUCTURE ONLY.

Follows special_attentions/SildingTileAttention.py:
  token_order   preprocess (:106-126): video tokens reordered from
                (nt tp nh hp nw wp) to (nt nh nw tp hp wp), i.e. tile by tile
  sta_mask      generate_sta_mask's mask_mod (:18-92) on reordered indices:
                text queries see every key; video queries see the text and
                the video tiles whose tile coordinates lie within the kernel
                half-widths of the query tile's kernel centre (the centre
                clamped kernel//2 away from the canvas edges)
  sta_attention forward (:137-140): attention in the reordered order under
                that mask, output reordered back (process_out_back)
Pinned by tests/golden/sta_layout.npz (the reference's own mask_mod and
preprocess evaluated on the CPU).
"""
from __future__ import annotations

import math

import numpy as np

from .smart import masked_attention


def token_order(canvas, tile, text: int) -> np.ndarray:
    """perm: the original token index at every position after preprocess."""
    T, Hc, W = canvas
    tt, th, tw = tile
    nt, nh, nw = T // tt, Hc // th, W // tw
    idx = np.arange(T * Hc * W).reshape(nt, tt, nh, th, nw, tw)
    video = idx.transpose(0, 2, 4, 1, 3, 5).reshape(-1)
    return np.concatenate([np.arange(text), text + video])


def sta_mask(canvas, kernel, tile, text: int, rows=None) -> np.ndarray:
    """bool [S, S] over reordered token indices (only ``rows`` when given)."""
    T, Hc, W = canvas
    kt, kh, kw = kernel
    tt, th, tw = tile
    nt, nh, nw = T // tt, Hc // th, W // tw
    S = text + T * Hc * W
    idx = np.arange(S)
    tid = np.floor_divide(idx - text, tt * th * tw)
    t_t, t_h, t_w = tid // (nh * nw), (tid % (nh * nw)) // nw, tid % nw
    ct = np.minimum(np.maximum(t_t, kt // 2), (nt - 1) - kt // 2)
    ch = np.minimum(np.maximum(t_h, kh // 2), (nh - 1) - kh // 2)
    cw = np.minimum(np.maximum(t_w, kw // 2), (nw - 1) - kw // 2)
    r = idx if rows is None else np.asarray(rows)
    q, k = r[:, None], idx[None, :]
    win = ((np.abs(ct[r][:, None] - t_t[None, :]) <= kt // 2) & (np.abs(ch[r][:, None] - t_h[None, :]) <= kh // 2) &
           (np.abs(cw[r][:, None] - t_w[None, :]) <= kw // 2))
    image = (q >= text) & (k >= text)
    return (image & win) | ((q >= text) & (k < text)) | (q < text)


def sta_attention(q, k, v, canvas, kernel, tile, text: int) -> np.ndarray:
    """[B, H, S, D] in the original token order -> fp64 output, same order."""
    perm = token_order(canvas, tile, text)
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.size)
    mask = sta_mask(canvas, kernel, tile, text)
    D = q.shape[-1]
    out = masked_attention(q[:, :, perm], k[:, :, perm], v[:, :, perm], mask, 1 / math.sqrt(D))
    return out[:, :, inv]
