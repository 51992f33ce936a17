"""SmartAttention restated on the CPU in fp64 -- TEST INFRASTRUCTURE ONLY.

Follows special_attentions/SmartAttention.py:
  band_mask        generate_block_tridiagonal_mask_mod (:30-43): query q sees
                   key k when k < text + frame_len, q < text, or
                   |frame(q) - frame(k)| <= diag, frame(x) = floor((x - text) / frame_len)
  token_order      process / process_back (:9-27): video tokens (t, h, w) <-> (h, w, t)
  band_attention   attention_with_mask (:130-143): text rows attend every key, the
                   rows of frame i the key set of the band row at the frame's start
  probe            choose_strategy (:97-108) on given sampled rows: squared distance of
                   the band outputs (natural and reordered mask) to full attention
  smart_attention  forward (:153-166) with a given per-(b, h) strategy
Pinned by tests/golden/smart_layout.npz (the reference's own mask_mod,
per-frame key sets and process / process_back outputs).
"""
from __future__ import annotations

import math

import numpy as np

from .selection import to_f64


def band_mask(text: int, frames: int, frame_len: int, diag: int = 1) -> np.ndarray:
    S = text + frames * frame_len
    idx = np.arange(S)
    fr = np.floor_divide(idx - text, frame_len)
    q, k = idx[:, None], idx[None, :]
    return (k < text + frame_len) | (q < text) | (np.abs(fr[:, None] - fr[None, :]) <= diag)


def token_order(text: int, frames: int, height: int, width: int):
    """(perm, inv): x[perm] is process(x), x[inv] is process_back(x)."""
    hw = height * width
    nat = np.arange(frames * hw).reshape(frames, height, width)      # (t, h, w) -> natural index
    perm_video = nat.transpose(1, 2, 0).reshape(-1)                    # (h, w, t) order
    perm = np.concatenate([np.arange(text), text + perm_video])
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.size)
    return perm, inv


def _attend(q, k, v, allowed, scale):
    s = (q @ k.T) * scale
    s = np.where(allowed, s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    return (p / p.sum(axis=-1, keepdims=True)) @ v


def band_attention(q, k, v, text: int, frames: int, frame_len: int, diag: int = 1):
    """[B,H,S,D] -> fp64 [B,H,S,D] under the band mask (natural order)."""
    q, k, v = to_f64(q), to_f64(k), to_f64(v)
    B, H, S, D = q.shape
    allowed = band_mask(text, frames, frame_len, diag)
    out = np.empty_like(q)
    for b in range(B):
        for h in range(H):
            out[b, h] = _attend(q[b, h], k[b, h], v[b, h], allowed, 1 / math.sqrt(D))
    return out


def probe(q, k, v, idx, text, frames, height, width, diag: int = 1):
    """(spatial_diff, temporal_diff, full, spatial, temporal) for the sampled
    query rows ``idx``; the temporal mask is the band in (h, w, t) order
    mapped back to natural order (process_mask_back, :44-51)."""
    q, k, v = to_f64(q), to_f64(k), to_f64(v)
    B, H, S, D = q.shape
    band = band_mask(text, frames, height * width, diag)
    perm, inv = token_order(text, frames, height, width)
    temporal_mask = band[inv][:, inv]
    idx = np.asarray(idx)
    full = np.empty((B, H, idx.size, D))
    sp, tp = np.empty_like(full), np.empty_like(full)
    ones = np.ones((idx.size, S), dtype=bool)
    for b in range(B):
        for h in range(H):
            qs = q[b, h, idx]
            full[b, h] = _attend(qs, k[b, h], v[b, h], ones, 1 / math.sqrt(D))
            sp[b, h] = _attend(qs, k[b, h], v[b, h], band[idx], 1 / math.sqrt(D))
            tp[b, h] = _attend(qs, k[b, h], v[b, h], temporal_mask[idx], 1 / math.sqrt(D))
    sd = ((sp - full) ** 2).sum(axis=(-1, -2))
    td = ((tp - full) ** 2).sum(axis=(-1, -2))
    return sd, td, full, sp, tp


def smart_attention(q, k, v, strategy, text, frames, height, width, diag: int = 1):
    """forward with a given bool [B, H] strategy (True = natural order)."""
    q, k, v = to_f64(q), to_f64(k), to_f64(v)
    perm, inv = token_order(text, frames, height, width)
    out = np.empty_like(q)
    fl = height * width
    nat = band_attention(q, k, v, text, frames, fl, diag)
    reo = band_attention(q[:, :, perm], k[:, :, perm], v[:, :, perm], text, frames, fl, diag)[:, :, inv]
    strategy = np.asarray(strategy, dtype=bool)
    out[strategy] = nat[strategy]
    out[~strategy] = reo[~strategy]
    return out


def ranges_mask(ranges, Sk: int) -> np.ndarray:
    """bool [Sq, Sk] of per-row key intervals [x, y) U [z, w) (the
    ``row_ranges`` argument of saf_bsa_fwd_ranges)."""
    r = np.asarray(ranges, dtype=np.int64)
    k = np.arange(Sk)[None, :]
    return ((k >= r[:, 0:1]) & (k < r[:, 1:2])) | ((k >= r[:, 2:3]) & (k < r[:, 3:4]))


def masked_attention(q, k, v, allowed, scale: float) -> np.ndarray:
    """fp64 attention of [B,H,Sq,D] under a token mask allowed [Sq, Sk] or
    [B, H, Sq, Sk]; rows with no allowed key are NaN."""
    q, k, v = to_f64(q), to_f64(k), to_f64(v)
    B, H, Sq, D = q.shape
    allowed = np.broadcast_to(np.asarray(allowed, dtype=bool), (B, H, Sq, k.shape[2]))
    out = np.full(q.shape, np.nan)
    for b in range(B):
        for h in range(H):
            rows = allowed[b, h].any(axis=1)
            if rows.any():
                out[b, h, rows] = _attend(q[b, h, rows], k[b, h], v[b, h], allowed[b, h, rows], scale)
    return out
