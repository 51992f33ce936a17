"""Frame-scope block mask oracle (test infrastructure; see ``oracle/__init__.py``).

Restates ``generate_attention_mask_frame_scope``
(special_attentions/utils/mask_related.py:194-245) in numpy fp64, with the
random spatial sample passed in instead of drawn:

* keys and queries sampled at every text token and, in every frame, the
  same ``n`` spatial positions (:198-203): index list
  ``[0..T) ++ [T + f*FL + s for f in frames for s in spatial]``;
* logits = q_s k_s^T * scale with ``log(n / FL)`` (computed in fp32, as the
  reference's float32 ``torch.tensor``) added on the text key columns
  (:205-212), softmax over all sampled keys;
* frame x frame map = sum over each (query frame, key frame) pair of the
  video-video probabilities divided by n (:214-220);
* per head, the flattened map sorted in descending order, cumulative sum,
  the first position whose cumulative sum reaches ``threshold`` times the
  total (the last position if none does), and every entry ranked at or
  before it kept (:222-243).

The attention side (``BlockSparseAttention.forward_backup``,
block_mask_attn.py:11-20) keeps text rows and text key columns dense and
lets a video query of frame f1 see the video keys of frame f2 when
mask[f1, f2]; here that is applied on the unpadded sequence, token by token
(the reference pads q per frame and randomly truncates k / v,
mask_related.py:87-167, and its inner-frame mask with threshold 1 keeps
every block in exact arithmetic).
"""
from __future__ import annotations

import math

import numpy as np

from .selection import to_f64


def sample_index(spatial, text_len: int, frames: int, frame_len: int) -> np.ndarray:
    spatial = np.asarray(spatial, dtype=np.int64)
    vid = (text_len + np.arange(frames)[:, None] * frame_len + spatial[None, :]).reshape(-1)
    return np.concatenate([np.arange(text_len), vid])


def composition(n: int, frame_len: int) -> float:
    """log(n / FL) as the reference evaluates it: a float32 tensor."""
    return float(np.log(np.float32(n / frame_len)))


def frame_map(q, k, spatial, text_len: int, frames: int, frame_len: int, scale: float = 0.125) -> np.ndarray:
    """[B, H, F, F] fp64 frame x frame attention map from the sampled tokens."""
    q, k = to_f64(q), to_f64(k)
    n = len(spatial)
    idx = sample_index(spatial, text_len, frames, frame_len)
    qs, ks = q[:, :, idx], k[:, :, idx]
    logits = np.einsum("bhid,bhjd->bhij", qs, ks) * scale
    logits[..., :text_len] += np.float64(np.float32(composition(n, frame_len)))
    logits -= logits.max(axis=-1, keepdims=True)
    p = np.exp(logits)
    p /= p.sum(axis=-1, keepdims=True)
    vv = p[:, :, text_len:, text_len:]
    B, H = vv.shape[:2]
    return vv.reshape(B, H, frames, n, frames, n).sum(axis=(3, 5)) / n


def frame_select(fmap: np.ndarray, threshold: float = 0.9) -> np.ndarray:
    """bool [B, H, F, F]: the reference's global energy rule per head."""
    B, H, F, _ = fmap.shape
    flat = fmap.reshape(B, H, F * F)
    out = np.zeros_like(flat, dtype=bool)
    for b in range(B):
        for h in range(H):
            order = np.argsort(-flat[b, h], kind="stable")
            cum = np.cumsum(flat[b, h][order])
            over = cum >= threshold * cum[-1]
            over[-1] = True
            kk = int(np.argmax(over))
            out[b, h, order[:kk + 1]] = True
    return out.reshape(B, H, F, F)


def frame_of(tok: np.ndarray, text_len: int, frame_len: int) -> np.ndarray:
    """Frame index of each token, -1 for text."""
    tok = np.asarray(tok)
    return np.where(tok < text_len, -1, (tok - text_len) // frame_len)


def token_allowed(fmask_bh: np.ndarray, rows, cols, text_len: int, frame_len: int) -> np.ndarray:
    """bool [len(rows), len(cols)]: text rows and text key columns see
    everything; a video row of frame f1 sees the video keys of the frames f2
    with fmask[f1, f2]."""
    fr = frame_of(np.asarray(rows), text_len, frame_len)
    fc = frame_of(np.asarray(cols), text_len, frame_len)
    ok = np.zeros((fr.size, fc.size), dtype=bool)
    vr, vc = fr >= 0, fc >= 0
    ok[~vr, :] = True
    ok[:, ~vc] = True
    sub = fmask_bh[np.ix_(fr[vr], fc[vc])]
    ok[np.ix_(vr, vc)] = sub
    return ok


def frame_block_mask(fmask: np.ndarray, text_len: int, frame_len: int, S: int, block_m: int,
                     block_n: int) -> np.ndarray:
    """bool [B, H, nbq, nbk]: a block is live when some of its token pairs
    are allowed."""
    B, H = fmask.shape[:2]
    nbq, nbk = -(-S // block_m), -(-S // block_n)
    out = np.zeros((B, H, nbq, nbk), dtype=bool)
    rows_f = frame_of(np.arange(S), text_len, frame_len)
    for b in range(B):
        for h in range(H):
            for i in range(nbq):
                fr = np.unique(rows_f[i * block_m:min(S, (i + 1) * block_m)])
                for j in range(nbk):
                    fc = np.unique(rows_f[j * block_n:min(S, (j + 1) * block_n)])
                    if (fr < 0).any() or (fc < 0).any():
                        out[b, h, i, j] = True
                    else:
                        out[b, h, i, j] = fmask[b, h][np.ix_(fr, fc)].any()
    return out


def frame_attention_rows(q, k, v, fmask, text_len: int, frame_len: int, sm_scale: float, heads,
                         rows) -> np.ndarray:
    """fp64 attention of the query ``rows`` of the flat heads ``heads`` under
    the token-level frame mask; [len(heads), len(rows), D]."""
    B, H, S, D = q.shape
    rows = np.asarray(list(rows), dtype=np.int64)
    keys = np.arange(k.shape[2])
    out = np.empty((len(list(heads)), rows.size, D))
    for hi, g in enumerate(heads):
        b, h = divmod(int(g), H)
        qh, kh, vh = to_f64(q[b, h]), to_f64(k[b, h]), to_f64(v[b, h])
        ok = token_allowed(np.asarray(fmask[b, h]), rows, keys, text_len, frame_len)
        logits = (qh[rows] @ kh.T) * sm_scale
        logits = np.where(ok, logits, -np.inf)
        logits -= logits.max(axis=1, keepdims=True)
        p = np.exp(logits)
        p /= p.sum(axis=1, keepdims=True)
        out[hi] = p @ vh
    return out


def frame_bits(fmask: np.ndarray) -> np.ndarray:
    """uint32 [B*H, F]: bit f2 of word f1 set when mask[f1, f2]."""
    B, H, F, _ = fmask.shape
    w = (fmask.astype(np.uint64) << np.arange(F, dtype=np.uint64)[None, None, None, :]).sum(-1)
    return w.astype(np.uint32).reshape(B * H, F)


def margin(fmap: np.ndarray, threshold: float = 0.9) -> float:
    """Smallest relative distance of a head's cumulative sums from its
    threshold: masks computed with a different rounding agree when this is
    well above the rounding error."""
    B, H, F, _ = fmap.shape
    flat = fmap.reshape(B * H, F * F)
    best = math.inf
    for row in flat:
        cum = np.cumsum(np.sort(row)[::-1])
        best = min(best, float(np.min(np.abs(cum - threshold * cum[-1])) / cum[-1]))
    return best
