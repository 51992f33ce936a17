"""Block selection oracle (test infrastructure; see ``oracle/__init__.py``).

Restates the block-selection contract of the CUDA kernels in
``sparseattnfunctions_b200/csrc/select.cu``:

* ``block_means``: per block of rows, the fp64 sum of the (bf16/f16/f32)
  values divided by the number of valid rows.  Replaces the random 8-of-64
  token sample of ``calc_attn_block_sum_efficient``
  (special_attentions/utils/mask_related.py:14-37, :40-81) with a
  deterministic mean, as the build's target asks.
* ``pooled_scores``: ``sum_d qbar[i,d] * kbar[j,d]`` in fp64 with d ascending
  and each product / sum rounded separately -- exactly what the kernel does
  with ``__dmul_rn`` / ``__dadd_rn``.
* ``topk_select``: per row keep the ``topk`` highest scores (ties -> lower
  column) as ``get_sparse_attn_mask_from_topk`` does
  (special_attentions/utils/block_sparse_attn_kernel.py:31-39), then force
  text rows / columns as ``transfer_attn_to_mask`` does
  (special_attentions/SparseGen_Plus.py:81-82) and the diagonal for the
  square CPU configuration.
"""
from __future__ import annotations

import numpy as np


def to_f64(x) -> np.ndarray:
    """bf16/f16/f32 torch tensor or numpy array -> float64 numpy array."""
    try:
        import torch

        if isinstance(x, torch.Tensor):
            return x.detach().to("cpu", torch.float64).numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x, dtype=np.float64)


def block_means(x, block: int) -> np.ndarray:
    """[B, H, S, D] -> [B, H, ceil(S/block), D] fp64 block means."""
    x = to_f64(x)
    B, H, S, D = x.shape
    nb = -(-S // block)
    out = np.empty((B, H, nb, D), dtype=np.float64)
    for i in range(nb):
        r0, r1 = i * block, min(S, (i + 1) * block)
        out[:, :, i, :] = x[:, :, r0:r1, :].sum(axis=2) / float(r1 - r0)
    return out


def pooled_scores(qbar: np.ndarray, kbar: np.ndarray) -> np.ndarray:
    """[B,H,nbq,D] x [B,H,nbk,D] -> [B,H,nbq,nbk], d ascending, no FMA."""
    s = np.zeros(qbar.shape[:3] + (kbar.shape[2],), dtype=np.float64)
    for d in range(qbar.shape[-1]):
        s = s + qbar[..., :, d, None] * kbar[..., None, :, d]
    return s


def topk_select(scores: np.ndarray, topk: int, text_blocks_q: int = 0, text_blocks_k: int = 0,
                force_diag: bool = False, forced_inside_topk: bool = False) -> np.ndarray:
    """Dense bool block mask [B,H,nbq,nbk] from pooled scores.

    Rows ``i < text_blocks_q`` are dense.  Other rows keep their top-k columns
    (NaN first, as torch.topk ranks it, then higher score first; equal scores
    and NaNs -> lower column) united with the forced
    columns (``j < text_blocks_k``; ``j == i`` with ``force_diag``).  With
    ``forced_inside_topk`` the forced columns count toward ``topk`` and the
    remaining ``topk - |forced|`` are chosen among the other columns.
    """
    B, H, nbq, nbk = scores.shape
    mask = np.zeros(scores.shape, dtype=bool)
    cols = np.arange(nbk)
    for i in range(nbq):
        if i < text_blocks_q:
            mask[:, :, i, :] = True
            continue
        forced = cols < text_blocks_k
        if force_diag and i < nbk:
            forced = forced | (cols == i)
        nforced = int(forced.sum())
        if forced_inside_topk:
            k = max(0, topk - nforced)
            elig = ~forced
        else:
            k = topk
            elig = np.ones(nbk, dtype=bool)
        ecols = cols[elig]
        row = scores[:, :, i, :][..., elig]  # [B,H,n_elig]
        k = min(k, ecols.size)
        if k > 0:
            # NaN first (torch.topk ranks NaN highest), then higher scores; the
            # stable sort keeps lower columns first among equal scores and NaNs
            nan = np.isnan(row)
            order = np.lexsort((np.where(nan, 0.0, -row), ~nan), axis=-1)[..., :k]
            sel = ecols[order]
            np.put_along_axis(mask[:, :, i, :], sel, True, axis=-1)
        mask[:, :, i, forced] = True
    return mask


def select_blocks(q, k, block_m: int, block_n: int, topk: int, text_blocks_q: int = 0,
                  text_blocks_k: int = 0, force_diag: bool = False,
                  forced_inside_topk: bool = False):
    """Full oracle of ``saf_pool_topk``: returns (mask, scores)."""
    scores = pooled_scores(block_means(q, block_m), block_means(k, block_n))
    mask = topk_select(scores, topk, text_blocks_q, text_blocks_k, force_diag, forced_inside_topk)
    return mask, scores


def reference_topk_mask(x: np.ndarray, topk: int) -> np.ndarray:
    """Restatement of get_sparse_attn_mask_from_topk
    (special_attentions/utils/block_sparse_attn_kernel.py:31-39) for distinct
    scores: the top-k indices of each row set to True."""
    idx = np.argsort(-x, axis=-1, kind="stable")[..., :topk]
    m = np.zeros(x.shape, dtype=bool)
    np.put_along_axis(m, idx, True, axis=-1)
    return m


def energy_select(attn: np.ndarray, energy_threshold: float, min_retain_ratio: float,
                  max_retain_ratio: float, text_blocks: int = 4) -> np.ndarray:
    """Restatement of transfer_attn_to_mask(mode="energy")
    (special_attentions/SparseGen_Plus.py:52-82): per row, keep the smallest
    prefix of columns in descending score order whose cumulative sum reaches
    ``energy_threshold`` of the row total, clamped to
    [max(1, int(n*min_ratio)), max(1, int(n*max_ratio))]; then force the first
    ``text_blocks`` rows and columns."""
    B, H, n, _ = attn.shape
    min_retain = max(1, int(n * min_retain_ratio))
    max_retain = max(1, int(n * max_retain_ratio))
    order = np.argsort(-attn, axis=-1, kind="stable")
    srt = np.take_along_axis(attn, order, axis=-1)
    cum = np.cumsum(srt, axis=-1)
    total = cum[..., -1:]
    reach = cum >= energy_threshold * total
    kidx = np.argmax(reach, axis=-1)
    unsatisfied = ~reach.any(axis=-1)
    kidx = np.where(unsatisfied, n, kidx)
    kidx = np.clip(kidx, min_retain, max_retain)
    keep_sorted = np.arange(n)[None, None, None, :] < kidx[..., None]
    mask = np.zeros(attn.shape, dtype=bool)
    np.put_along_axis(mask, order, keep_sorted, axis=-1)
    mask[:, :, :text_blocks, :] = True
    mask[:, :, :, :text_blocks] = True
    return mask


def topk_adaptive_select(attn: np.ndarray, init_k, text_blocks: int = 4) -> np.ndarray:
    """Restatement of transfer_attn_to_mask(mode="topk")
    (special_attentions/SparseGen_Plus.py:28-50) on a square map: k0 =
    int(n * init_k) for a fraction, else int(init_k); E = cumulative sum of
    the first k0 sorted values; rows with E < 0.6 total go to min(3 k0, n),
    then rows with E < 0.9 total to min(k // 3 * 2, n); the first k sorted
    blocks are kept; text rows / columns forced."""
    B, H, n, _ = attn.shape
    k0 = int(n * init_k) if init_k < 1 else int(init_k)
    order = np.argsort(-attn, axis=-1, kind="stable")
    srt = np.take_along_axis(attn, order, axis=-1)
    cum = np.cumsum(srt, axis=-1)
    total = cum[..., -1]
    e = cum[..., k0 - 1]
    k = np.full(attn.shape[:-1], k0, dtype=np.int64)
    grow = ~(e >= 0.6 * total) & (k < n)
    cut = ~(e >= 0.9 * total) & (k < n)
    k = np.where(grow, np.minimum(3 * k, n), k)
    k = np.where(cut, np.minimum(k // 3 * 2, n), k)
    keep_sorted = np.arange(n)[None, None, None, :] < k[..., None]
    mask = np.zeros(attn.shape, dtype=bool)
    np.put_along_axis(mask, order, keep_sorted, axis=-1)
    mask[:, :, :text_blocks, :] = True
    mask[:, :, :, :text_blocks] = True
    return mask


def dense_to_csr(mask: np.ndarray):
    """Dense bool [B,H,nbq,nbk] -> (row_ptr [B*H, nbq+1], col_idx) in the
    library's segmented layout (head g's entries start at g*nbq*nbk)."""
    B, H, nbq, nbk = mask.shape
    m = mask.reshape(B * H, nbq, nbk)
    row_ptr = np.zeros((B * H, nbq + 1), dtype=np.int64)
    col_idx = np.full(B * H * nbq * nbk, -1, dtype=np.int64)
    for g in range(B * H):
        off = g * nbq * nbk
        row_ptr[g, 0] = off
        for i in range(nbq):
            cols = np.nonzero(m[g, i])[0]
            col_idx[off:off + cols.size] = cols
            off += cols.size
            row_ptr[g, i + 1] = off
    return row_ptr, col_idx
