"""LocalGlobalAttention oracle (test infrastructure; see ``oracle/__init__.py``).

Restates special_attentions/LocalGlobalAttention.py (module constants :11-19,
``get_mask`` :114-179, ``probe_solver._probe_num`` :44-56, the processor
:183-259) for the CogVideoX-2B layout (226 text tokens, 13 x 30 x 45 video):

* query rows of the text and of frame 0 (the first 226 + 1350) attend every
  key (:193-205);
* the video rows of frames 1-12 fall into 18 patches of 6 x 10 x 15 tokens
  (2 x 3 x 3 patches; patch p = (nt * 3 + nh) * 3 + nw); a patch sees the
  text, frame 0 and a window around it: frames, rows and columns with
  start = clamp(p_start - pad, [1, 0, 0], [13, 30, 45]),
  end = clamp(start + size + 2 pad, same bounds), start = end - size - 2 pad
  (size 6 x 10 x 15, pad 13 x 0.2, 30 x 0.1, 45 x 0.1; float32 arithmetic as
  the reference's tensors), an index i in [start, end) when start <= i < end
  (:125-170);
* the reference gathers each patch's window keys in the order of a
  descending sort of its mask row and keeps as many as the first patch has
  (``remain_num``, :172-178); the patches of the second frame group have
  384 window keys fewer, so their lists go on with keys outside the window
  in sort order.  ``window_lists`` restates that with a stable sort (the
  window keys ascending, then the first non-window keys ascending), the
  order of a stable descending sort;
* plus, per (patch, batch), the 889 keys (int(0.05 x 17776) + 1) of largest
  probe mass outside the patch's window mask (:50-62, :219-238), ties to
  the lower key (a stable descending sort).  The probe mass of batch b is
  the softmax of 1280 sampled video query rows over all keys, summed over
  rows and heads, with the reference's 16-bit roundings: the logits rounded
  to the input type (matmul output), then scaled by 1/8 (exact), the
  softmax rounded to the input type, the sum rounded once
  (``probe_mass``).  The reference draws the sampled rows with
  torch.randint; here they are passed in.

A key can appear twice in a list (a global key among the fill keys of a
second-group patch); the reference's gather keeps both, and so does
``keys_for``.
"""
from __future__ import annotations

import numpy as np

from .selection import to_f64

VIDEO = (13, 30, 45)
PATCH = (6, 10, 15)
COMP = (2, 3, 3)
PAD_FRAC = (0.2, 0.1, 0.1)
TEXT = 226
FRAME = VIDEO[1] * VIDEO[2]
DENSE_ROWS = TEXT + FRAME
N_GLOBAL = int(0.05 * (TEXT + VIDEO[0] * FRAME)) + 1
N_SAMPLE = 1280


def patch_coords(p: int):
    return (p // (COMP[1] * COMP[2])) % COMP[0], (p // COMP[2]) % COMP[1], p % COMP[2]


def window(p: int):
    """(start, end) float32 triples (t, h, w) of patch p's key window."""
    nt, nh, nw = patch_coords(p)
    pad = np.array([VIDEO[i] * PAD_FRAC[i] for i in range(3)], dtype=np.float32)
    lo = np.array([1, 0, 0], dtype=np.float32)
    hi = np.array(VIDEO, dtype=np.float32)
    gap = np.array(PATCH, dtype=np.float32)
    start = np.array([nt * PATCH[0] + 1, nh * PATCH[1], nw * PATCH[2]], dtype=np.float32) - pad
    start = np.clip(start, lo, hi)
    end = np.clip(start + gap + pad * np.float32(2), lo, hi)
    start = end - gap - pad * np.float32(2)
    return start.astype(np.float32), end.astype(np.float32)


def local_mask(S: int = TEXT + VIDEO[0] * FRAME) -> np.ndarray:
    """bool [18, S]: the keys each patch sees besides its global keys."""
    kv = np.arange(S)
    sh = kv - TEXT
    t = np.floor_divide(sh, FRAME)
    h = np.remainder(np.floor_divide(sh, VIDEO[2]), VIDEO[1]).astype(np.float32)
    w = np.remainder(sh, VIDEO[2]).astype(np.float32)
    tf = t.astype(np.float32)
    out = np.zeros((COMP[0] * COMP[1] * COMP[2], S), dtype=bool)
    for p in range(out.shape[0]):
        st, en = window(p)
        inside = ((w >= st[2]) & (w < en[2]) & (h >= st[1]) & (h < en[1]) & (tf >= st[0]) & (tf < en[0]))
        out[p] = (kv < TEXT) | (t == 0) | inside
    return out


def patch_rows(p: int) -> np.ndarray:
    """Token indices of patch p's query rows in the reference's (tp hp wp)
    order (frames 1-12)."""
    nt, nh, nw = patch_coords(p)
    tp, hp, wp = np.meshgrid(np.arange(PATCH[0]), np.arange(PATCH[1]), np.arange(PATCH[2]), indexing="ij")
    t = 1 + nt * PATCH[0] + tp
    h = nh * PATCH[1] + hp
    w = nw * PATCH[2] + wp
    return (TEXT + t * FRAME + h * VIDEO[2] + w).reshape(-1)


def round16(x, kind: str = "bf16") -> np.ndarray:
    """Rounds fp64 values to fp32 and then to bf16 / f16 (round to nearest
    even), returned as fp64 -- a 16-bit result of an fp32 computation."""
    f = np.asarray(x, dtype=np.float64).astype(np.float32)
    if kind == "f16":
        return f.astype(np.float16).astype(np.float64)
    u = f.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return u.view(np.float32).astype(np.float64)


def probe_mass(q, k, samples, scale: float = 0.125, kind: str = "bf16",
               row_offset: int = DENSE_ROWS) -> np.ndarray:
    """fp64 [B, S] holding 16-bit values: per batch, round16 of the sum over
    heads and sampled rows of round16(softmax(round16(q_r . k) * scale)),
    the sampled rows ``samples [B, n]`` indexing the video rows (token
    ``row_offset + s``).  LocalGlobalAttention.py:50-57."""
    q, k = to_f64(q), to_f64(k)
    B, H, S, D = q.shape[0], q.shape[1], k.shape[2], q.shape[3]
    out = np.zeros((B, k.shape[2]))
    for b in range(B):
        rows = row_offset + np.asarray(samples[b])
        for h in range(H):
            lg = round16(q[b, h, rows] @ k[b, h].T, kind) * scale
            lg -= lg.max(axis=1, keepdims=True)
            e = np.exp(lg)
            out[b] += round16(e / e.sum(axis=1, keepdims=True), kind).sum(axis=0)
    return round16(out, kind)


def window_lists(lmask: np.ndarray) -> np.ndarray:
    """int [18, remain]: per patch the window keys ascending, then (second
    frame group) the first non-window keys ascending, remain = the first
    patch's window size -- the first ``remain`` entries of a stable
    descending sort of the mask row (LocalGlobalAttention.py:172-178)."""
    remain = int(lmask[0].sum())
    out = np.empty((lmask.shape[0], remain), dtype=np.int64)
    for p in range(lmask.shape[0]):
        w = np.nonzero(lmask[p])[0]
        nw = np.nonzero(~lmask[p])[0]
        out[p] = np.concatenate([w, nw[:remain - w.size]])[:remain]
    return out


def global_keys(mass: np.ndarray, lmask: np.ndarray, n: int = N_GLOBAL) -> np.ndarray:
    """int [18 * B, n]: per row r = p * B + b the n keys of largest mass
    outside patch p's local mask (ties to the lower key), ascending."""
    B = mass.shape[0]
    P = lmask.shape[0]
    out = np.empty((P * B, n), dtype=np.int64)
    for r in range(P * B):
        p, b = divmod(r, B)
        v = np.where(lmask[p], -np.inf, mass[b])
        order = np.lexsort((np.arange(v.size), -v))
        out[r] = np.sort(order[:n])
    return out


def margin(mass: np.ndarray, lmask: np.ndarray, n: int = N_GLOBAL) -> float:
    """Smallest relative gap between the n-th and (n+1)-th largest masses
    of any row: selections computed with other rounding agree when it is
    well above that rounding."""
    B = mass.shape[0]
    best = np.inf
    for r in range(lmask.shape[0] * B):
        p, b = divmod(r, B)
        v = np.sort(mass[b][~lmask[p]])[::-1]
        best = min(best, (v[n - 1] - v[n]) / v[n - 1])
    return float(best)


def attention_rows(q, k, v, rows, keys_of, scale: float = 0.125) -> np.ndarray:
    """fp64 [len(rows), H, D]: attention of query ``rows`` of batch b over
    ``keys_of(row)`` for every head; rows are (b, token) pairs."""
    q64, k64, v64 = to_f64(q), to_f64(k), to_f64(v)
    H, D = q64.shape[1], q64.shape[3]
    out = np.empty((len(rows), H, D))
    for i, (b, tok) in enumerate(rows):
        keys = np.asarray(keys_of(b, tok))
        for h in range(H):
            lg = (k64[b, h, keys] @ q64[b, h, tok]) * scale
            e = np.exp(lg - lg.max())
            out[i, h] = (e / e.sum()) @ v64[b, h, keys]
    return out


def patch_of(tok: int) -> int:
    """Patch index of a video token of frames 1-12."""
    sh = tok - TEXT
    t, h, w = sh // FRAME, (sh // VIDEO[2]) % VIDEO[1], sh % VIDEO[2]
    nt, nh, nw = (t - 1) // PATCH[0], h // PATCH[1], w // PATCH[2]
    return (nt * COMP[1] + nh) * COMP[2] + nw


def keys_for(b: int, tok: int, wlists: np.ndarray, gkeys, B: int, S: int) -> np.ndarray:
    """The keys (a multiset) query token ``tok`` of batch b attends to:
    every key for the text and frame-0 rows, else its patch's window list
    and global keys (``gkeys`` [18 * B, n], or None when the probe is off)."""
    if tok < DENSE_ROWS:
        return np.arange(S)
    p = patch_of(tok)
    if gkeys is None:
        return wlists[p]
    return np.concatenate([wlists[p], gkeys[p * B + b]])
