"""ToMe bipartite soft matching oracle (test infrastructure; see
``oracle/__init__.py``).

Restates ``bipartite_soft_matching_video`` with its ``merge`` / ``unmerge``
closures (special_attentions/utils/merge_unmerge.py:34-154) in numpy:

* split (:62-97): per (st, sy, sx) cell of frames 1..t-1 one token -- the
  ``rand_idx``-th of the cell, 0 (top-left) with ``no_rand`` -- goes to dst;
  the whole first frame is dst too (:83, :91).  ``a_idx`` (src) and
  ``b_idx`` (dst) are video-token indices.  The reference orders them with an
  unstable ``argsort`` (:82); here the order is the stable one (ascending
  index within dst and within src), and callers may pass the reference's
  order in instead.  ``alternate_split`` is the BASELINE config-3 split
  (src = even tokens, dst = odd tokens).
* match (:99-116): cosine similarity of src x dst, per src the best dst
  (``node_max``, ``node_idx``), src sorted by ``node_max`` descending; the
  first r are merged (``src_idx``, ``dst_idx``), the rest stay
  (``unm_idx``); ``counter`` = 1 + number of src merged into each dst.
  Contract of this build (the reference's bf16 scores are tie-dominated):
  cos(a, b) = dot(a, b) / (sqrt(|a|^2) * sqrt(|b|^2)) in fp64 on the input
  values, every dot product summed in the kernels' fixed order (``lane_dot``:
  exact products, per-lane ascending sums, xor butterfly), correctly rounded
  sqrt / mul / div; arg-max ties -> lower dst position; sort ties -> lower
  src position.
* merge (:119-135): ``[unm, scatter_reduce(dst, dst_idx, src, "mean")]``
  with ``include_self`` (so dst_j = (dst_j + sum of its src) / counter_j);
  the 4-D form prepends the text tokens (:120-128).
* unmerge (:137-154): dst back to ``b_idx``, unm back to ``a_idx[unm_idx]``,
  merged src copy their dst; the 4-D form strips / re-prepends the text.
"""
from __future__ import annotations

import numpy as np

from .selection import to_f64


def video_split(w: int, h: int, t: int, sx: int, sy: int, st: int, rand_idx=None,
                stable: bool = True):
    """(a_idx, b_idx) int64 video-token indices of src and dst.

    ``rand_idx``: int array [(t-1)//st, h//sy, w//sx] of dst positions inside
    each cell (``None`` = 0, the reference's ``no_rand``)."""
    tt = t - 1
    hsy, wsx, tst = h // sy, w // sx, tt // st
    if rand_idx is None:
        rand_idx = np.zeros((tst, hsy, wsx), dtype=np.int64)
    rand_idx = np.asarray(rand_idx, dtype=np.int64).reshape(tst, hsy, wsx)
    buf = np.zeros((tst, hsy, wsx, st * sy * sx), dtype=np.int64)
    np.put_along_axis(buf, rand_idx[..., None], -1, axis=3)
    # "tst hsy wsx st sy sx -> (tst st) (hsy sy) (wsx sx)"
    buf = buf.reshape(tst, hsy, wsx, st, sy, sx).transpose(0, 3, 1, 4, 2, 5)
    buf = buf.reshape(tst * st, hsy * sy, wsx * sx)
    if tst * st < tt or hsy * sy < h or wsx * sx < w:
        full = np.zeros((tt, h, w), dtype=np.int64)
        full[:tst * st, :hsy * sy, :wsx * sx] = buf
        buf = full
    order = np.argsort(buf.reshape(-1), kind="stable" if stable else "quicksort") + w * h
    num_dst = tst * hsy * wsx
    a_idx = order[num_dst:]
    b_idx = np.concatenate([np.arange(w * h), order[:num_dst]])
    return a_idx, b_idx


def alternate_split(n: int):
    """src = even tokens, dst = odd tokens."""
    idx = np.arange(n)
    return idx[0::2].copy(), idx[1::2].copy()


def lane_dot(x, y) -> np.ndarray:
    """fp64 dot products over the last axis in the summation order of the
    CUDA kernels: 32 lanes each add the exact products of columns
    c = lane, lane + 32, ... in ascending order, then the lane sums are
    combined by an xor butterfly (offsets 16, 8, 4, 2, 1).  Products of
    16-bit values are exact in fp64, so this order fixes every rounding."""
    prod = np.asarray(x, np.float64) * np.asarray(y, np.float64)
    C = prod.shape[-1]
    Cp = -(-C // 32) * 32
    if Cp != C:
        prod = np.concatenate([prod, np.zeros(prod.shape[:-1] + (Cp - C,))], axis=-1)
    prod = prod.reshape(prod.shape[:-1] + (Cp // 32, 32))
    p = np.zeros(prod.shape[:-2] + (32,))
    for k in range(Cp // 32):
        p = p + prod[..., k, :]
    lanes = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        p = p + p[..., lanes ^ off]
    return p[..., 0]


def cosine_scores(metric, a_idx, b_idx) -> np.ndarray:
    """[B, Ns, Nd] fp64 cosine similarities evaluated with BLAS (for the
    arg-max search; exact values come from ``exact_cosine``)."""
    x = to_f64(metric)
    a, b = x[:, a_idx], x[:, b_idx]
    na = np.sqrt(np.einsum("bnc,bnc->bn", a, a))
    nb = np.sqrt(np.einsum("bnc,bnc->bn", b, b))
    dots = np.einsum("bic,bjc->bij", a, b)
    return dots / (na[:, :, None] * nb[:, None, :])


def exact_cosine(x, bb, i, j, a_idx, b_idx) -> np.ndarray:
    """The contract's cosine of src i and dst j of batch row bb (arrays):
    lane_dot(a, b) / (sqrt(lane_dot(a, a)) * sqrt(lane_dot(b, b)))."""
    a = x[bb, a_idx[i]]
    b = x[bb, b_idx[j]]
    return lane_dot(a, b) / (np.sqrt(lane_dot(a, a)) * np.sqrt(lane_dot(b, b)))


def match(metric, a_idx, b_idx, r: int, scores=None):
    """Returns dict(unm_idx, src_idx, dst_idx, counter, node_max, node_idx);
    indices are positions within a_idx / b_idx (int64).  The arg-max is over
    the contract's exact cosines: every candidate within 1e-12 of the BLAS
    row maximum (BLAS error is ~1e-15) is re-evaluated with ``exact_cosine``;
    ties go to the lower dst position."""
    x = to_f64(metric)
    a_idx = np.asarray(a_idx)
    b_idx = np.asarray(b_idx)
    if scores is None:
        scores = cosine_scores(x, a_idx, b_idx)
    B, Ns, Nd = scores.shape
    r = min(Ns, r)
    rowmax = scores.max(axis=-1)
    bb, ii, jj = np.nonzero(scores >= rowmax[..., None] - 1e-12)
    ex = exact_cosine(x, bb, ii, jj, a_idx, b_idx)
    node_max = np.full((B, Ns), -np.inf)
    node_idx = np.full((B, Ns), np.iinfo(np.int64).max, dtype=np.int64)
    # visit candidates by (row, exact value desc, column asc): the first wins
    order = np.lexsort((jj, -ex, ii, bb))
    first = np.ones(order.size, dtype=bool)
    key = bb[order] * Ns + ii[order]
    first[1:] = key[1:] != key[:-1]
    sel = order[first]
    node_max[bb[sel], ii[sel]] = ex[sel]
    node_idx[bb[sel], ii[sel]] = jj[sel]
    edge = np.argsort(-node_max, axis=-1, kind="stable")
    unm_idx, src_idx = edge[:, r:], edge[:, :r]
    dst_idx = np.take_along_axis(node_idx, src_idx, axis=-1)
    counter = np.ones((B, Nd), dtype=np.int64)
    for bb in range(B):
        np.add.at(counter[bb], dst_idx[bb], 1)
    return dict(unm_idx=unm_idx, src_idx=src_idx, dst_idx=dst_idx, counter=counter,
                node_max=node_max, node_idx=node_idx, r=r)


def merge(x, a_idx, b_idx, m) -> np.ndarray:
    """3-D merge: x [B, N, C] -> [B, Ns - r + Nd, C] (fp64)."""
    x = to_f64(x)
    src, dst = x[:, a_idx], x[:, b_idx].copy()
    B = x.shape[0]
    out_dst = dst.copy()
    for bb in range(B):
        np.add.at(out_dst[bb], m["dst_idx"][bb], src[bb, m["src_idx"][bb]])
    out_dst /= m["counter"][..., None].astype(np.float64)
    unm = np.take_along_axis(src, m["unm_idx"][..., None], axis=1)
    return np.concatenate([unm, out_dst], axis=1)


def unmerge(y, a_idx, b_idx, m, n: int) -> np.ndarray:
    """3-D unmerge: y [B, Ns - r + Nd, C] -> [B, n, C] (fp64)."""
    y = to_f64(y)
    B, _, C = y.shape
    unm_len = m["unm_idx"].shape[1]
    unm, dst = y[:, :unm_len], y[:, unm_len:]
    out = np.zeros((B, n, C), dtype=np.float64)
    out[:, b_idx] = dst
    for bb in range(B):
        out[bb, a_idx[m["unm_idx"][bb]]] = unm[bb]
        out[bb, a_idx[m["src_idx"][bb]]] = dst[bb, m["dst_idx"][bb]]
    return out


def token_map(a_idx, b_idx, m, n: int, offset: int = 0) -> np.ndarray:
    """[B, n] row of the merged sequence that each original token reads on
    unmerge (``offset`` = rows before the video part, e.g. the text)."""
    B = m["unm_idx"].shape[0]
    unm_len = m["unm_idx"].shape[1]
    out = np.empty((B, n), dtype=np.int64)
    out[:, b_idx] = offset + unm_len + np.arange(len(b_idx))[None, :]
    for bb in range(B):
        out[bb, a_idx[m["unm_idx"][bb]]] = offset + np.arange(unm_len)
        out[bb, a_idx[m["src_idx"][bb]]] = offset + unm_len + m["dst_idx"][bb]
    return out


def proportional_bias(counter, text_len: int, unm_len: int) -> np.ndarray:
    """MergeAttention's attention bias (MergeAttention.py:33-38): log(size)
    on the dst columns of the merged key sequence [text | unm | dst], 0 elsewhere."""
    B, Nd = counter.shape
    bias = np.zeros((B, text_len + unm_len + Nd), dtype=np.float64)
    bias[:, text_len + unm_len:] = np.log(counter.astype(np.float64))
    return bias


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """fp64 -> nearest bf16 value (ties to even), rounded once from fp64
    (as __double2bfloat16), returned as fp64."""
    x = np.asarray(x, dtype=np.float64)
    m, e = np.frexp(x)                      # x = m * 2**e, 0.5 <= |m| < 1
    return np.ldexp(np.rint(m * 256.0) / 256.0, e)


def kv_metric(k, v, text_len: int):
    """MergeAttention's metric [k, |k|, v, |v|] of the video tokens
    (MergeAttention.py:26-31) as [B*H, S - text_len, 2D + 2] in the input's
    16-bit type.  Each norm follows the saf_tome_kv_metric summation order:
    lane l of 32 sums (x[2w]^2 + x[2w+1]^2) over its words w = l, l + 32
    (ascending), the lane sums combine by the xor butterfly 16, 8, 4, 2, 1
    (all in fp64), then the fp64 sqrt is rounded once to the 16-bit type."""
    import torch

    B, H, S, D = k.shape
    parts = []
    for x in (k, v):
        xv = x[:, :, text_len:].reshape(B * H, S - text_len, D)
        f = xv.double().cpu().numpy()
        sq = f * f
        pair = sq[..., 0::2] + sq[..., 1::2]            # word w: x[2w]^2 + x[2w+1]^2
        W = pair.shape[-1]
        lanes = np.zeros(f.shape[:2] + (32,))
        for w0 in range(0, W, 32):                       # words l, l + 32, ... ascending
            chunk = np.zeros(f.shape[:2] + (32,))
            chunk[..., :min(32, W - w0)] = pair[..., w0:w0 + 32]
            lanes = lanes + chunk
        lane = np.arange(32)
        for m in (16, 8, 4, 2, 1):
            lanes = lanes + lanes[..., lane ^ m]
        nrm = np.sqrt(lanes[..., 0])
        if x.dtype == torch.bfloat16:
            n16 = torch.from_numpy(round_to_bf16(nrm)).to(torch.bfloat16)
        else:
            n16 = torch.from_numpy(nrm.astype(np.float16))
        parts += [xv.cpu(), n16.unsqueeze(-1)]
    return torch.cat(parts, dim=-1)
