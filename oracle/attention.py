"""Block-sparse attention oracle (test infrastructure; see ``oracle/__init__.py``).

The reference defines block-sparse attention by its test oracle
(special_attentions/utils/block_sparse_attn_kernel.py:326-334): expand the
block mask with ``kron(mask, ones(BLOCK, BLOCK))``, crop to the sequence,
``masked_fill(~mask, -inf)`` the scaled logits, softmax, multiply by V.  A row
whose mask is all False therefore yields NaN (softmax of all -inf), which is
also what the Triton kernel produces (0/0 at :201-203).

``block_sparse_attention`` evaluates exactly that, block by block, in fp64
(inputs are converted from their stored precision, so bf16 inputs are used
at their exact bf16 values).  ``masked_sdpa_cpu`` is the same math through
PyTorch's CPU ``scaled_dot_product_attention`` with a boolean mask, query
chunked -- the reference's PyTorch masked path used as the timed CPU
baseline.
"""
from __future__ import annotations

import math
from typing import Iterable, Optional

import numpy as np

from .selection import to_f64


def block_sparse_attention(q, k, v, block_mask, sm_scale: float, block_m: int, block_n: int,
                           kv_bias=None, heads: Optional[Iterable[int]] = None,
                           row_blocks: Optional[Iterable[int]] = None) -> np.ndarray:
    """fp64 block-sparse attention.

    q [B,H,Sq,D], k/v [B,H,Sk,D], block_mask bool [B,H,ceil(Sq/bm),ceil(Sk/bn)],
    kv_bias optional [B*H, Sk] / [Sk] additive logit bias.  ``heads`` (flat
    b*H+h) and ``row_blocks`` restrict the work; rows not computed are NaN.
    Returns float64 [B,H,Sq,D].
    """
    q, k, v = to_f64(q), to_f64(k), to_f64(v)
    mask = np.asarray(to_f64(block_mask) != 0)
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    nbq = math.ceil(Sq / block_m)
    bias = None
    if kv_bias is not None:
        bias = to_f64(kv_bias).reshape(-1, Sk)
    out = np.full((B, H, Sq, D), np.nan, dtype=np.float64)
    heads = range(B * H) if heads is None else heads
    for g in heads:
        b, h = divmod(g, H)
        brow = None if bias is None else bias[0 if bias.shape[0] == 1 else g]
        for i in (range(nbq) if row_blocks is None else row_blocks):
            r0, r1 = i * block_m, min(Sq, (i + 1) * block_m)
            cols = np.nonzero(mask[b, h, i])[0]
            if cols.size == 0:
                continue  # stays NaN: softmax over an empty set
            kv_idx = np.concatenate([np.arange(c * block_n, min(Sk, (c + 1) * block_n)) for c in cols])
            logits = (q[b, h, r0:r1] @ k[b, h, kv_idx].T) * sm_scale
            if brow is not None:
                logits = logits + brow[kv_idx][None, :]
            logits -= logits.max(axis=1, keepdims=True)
            p = np.exp(logits)
            p /= p.sum(axis=1, keepdims=True)
            out[b, h, r0:r1] = p @ v[b, h, kv_idx]
    return out


def block_sparse_attention_rows(q, k, v, block_mask, sm_scale: float, block_m: int, block_n: int,
                                heads: Iterable[int], rows: Iterable[int]) -> np.ndarray:
    """The same fp64 definition as ``block_sparse_attention`` evaluated only
    for the query ``rows`` of the flat heads ``heads`` (b*H + h), for
    sampled parity checks at full sequence lengths.  Returns float64
    ``[len(heads), len(rows), D]`` (NaN for a row with no live block)."""
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    rows = np.asarray(list(rows), dtype=np.int64)
    heads = list(heads)
    mask = block_mask
    out = np.full((len(heads), rows.size, D), np.nan, dtype=np.float64)
    for hi, g in enumerate(heads):
        b, h = divmod(int(g), H)
        qh = to_f64(q[b, h])
        kh = to_f64(k[b, h])
        vh = to_f64(v[b, h])
        mh = np.asarray(to_f64(mask[b, h]) != 0)
        for i in np.unique(rows // block_m):
            sel = np.nonzero(rows // block_m == i)[0]
            cols = np.nonzero(mh[i])[0]
            if cols.size == 0:
                continue
            kv_idx = np.concatenate([np.arange(c * block_n, min(Sk, (c + 1) * block_n)) for c in cols])
            logits = (qh[rows[sel]] @ kh[kv_idx].T) * sm_scale
            logits -= logits.max(axis=1, keepdims=True)
            p = np.exp(logits)
            p /= p.sum(axis=1, keepdims=True)
            out[hi, sel] = p @ vh[kv_idx]
    return out


def attention_with_pooling(q, k, v, sm_scale: float, block_size: int, block_mask=None):
    """fp64 attention with the pooled attention map of
    special_attentions/utils/attn_pooling_kernel.py (non-causal path).

    Per query row r and key block j: R[r, j] = max logit of r in block j
    (:43-47), p[r, j] = exp(R[r, j] - m_r) / l_r with the row's softmax max
    and sum (:81-97, written there in log2 units), pool[i, j] = max of p over
    the rows of query block i (block_size rows), then every pool row divided
    by its sum (:254-255).  ``block_mask`` (optional, [B,H,nbq,nbk] over
    block_size x block_size blocks) restricts the keys a row sees; blocks it
    does not see contribute 0.  Returns (out [B,H,Sq,D], pool [B,H,nbq,nbk]).
    """
    q, k, v = to_f64(q), to_f64(k), to_f64(v)
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    nbq, nbk = math.ceil(Sq / block_size), math.ceil(Sk / block_size)
    mask = np.ones((B, H, nbq, nbk), dtype=bool) if block_mask is None else np.asarray(to_f64(block_mask) != 0)
    out = np.full((B, H, Sq, D), np.nan, dtype=np.float64)
    pool = np.zeros((B, H, nbq, nbk), dtype=np.float64)
    for b in range(B):
        for h in range(H):
            tok = np.repeat(np.repeat(mask[b, h], block_size, axis=0), block_size, axis=1)[:Sq, :Sk]
            logits = (q[b, h] @ k[b, h].T) * sm_scale
            logits = np.where(tok, logits, -np.inf)
            m = logits.max(axis=1, keepdims=True)
            e = np.exp(logits - m)
            l = e.sum(axis=1, keepdims=True)
            out[b, h] = (e / l) @ v[b, h]
            pad = nbk * block_size - Sk
            lp = np.pad(logits, ((0, 0), (0, pad)), constant_values=-np.inf)
            rmax = lp.reshape(Sq, nbk, block_size).max(axis=2)        # R[r, j]
            p = np.exp(rmax - m) / l                                  # 0 where R = -inf
            for i in range(nbq):
                pool[b, h, i] = p[i * block_size:(i + 1) * block_size].max(axis=0)
    pool = pool / pool.sum(axis=-1, keepdims=True)
    return out, pool


def expand_block_mask(block_mask, Sq: int, Sk: int, block_m: int, block_n: int):
    """Token-level mask from a block mask, like ``torch.kron(mask, ones)``
    cropped to ``[:Sq, :Sk]`` (block_sparse_attn_kernel.py:326-328)."""
    import torch

    m = torch.as_tensor(block_mask).bool()
    m = m.repeat_interleave(block_m, dim=-2).repeat_interleave(block_n, dim=-1)
    return m[..., :Sq, :Sk]


def masked_sdpa_cpu(q, k, v, block_mask, sm_scale: float, block_m: int, block_n: int,
                    q_chunk: int = 2048, heads: Optional[Iterable[int]] = None, kv_bias=None):
    """The reference's PyTorch masked-attention path on the host CPU:
    ``F.scaled_dot_product_attention(q, k, v, attn_mask=bool_mask)`` per head,
    in query chunks of ``q_chunk`` rows, in the inputs' dtype.  Returns a torch
    tensor [B,H,Sq,D] (rows of heads not computed are zero)."""
    import torch
    import torch.nn.functional as F

    q, k, v = (torch.as_tensor(t).cpu() for t in (q, k, v))
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    bm = torch.as_tensor(block_mask).bool().cpu()
    out = torch.zeros_like(q)
    heads = range(B * H) if heads is None else heads
    bias = None
    if kv_bias is not None:
        bias = torch.as_tensor(kv_bias).cpu().reshape(-1, Sk)
    for g in heads:
        b, h = divmod(g, H)
        for r0 in range(0, Sq, q_chunk):
            r1 = min(Sq, r0 + q_chunk)
            rb0, rb1 = r0 // block_m, (r1 - 1) // block_m + 1
            m = bm[b, h, rb0:rb1].repeat_interleave(block_m, 0).repeat_interleave(block_n, 1)
            m = m[r0 - rb0 * block_m: r1 - rb0 * block_m, :Sk]
            attn_mask = m
            if bias is not None:
                brow = bias[0 if bias.shape[0] == 1 else g].to(q.dtype)
                attn_mask = torch.where(m, brow[None, :], torch.tensor(float("-inf"), dtype=q.dtype))
            out[b, h, r0:r1] = F.scaled_dot_product_attention(
                q[b, h, r0:r1][None], k[b, h][None], v[b, h][None], attn_mask=attn_mask[None],
                scale=sm_scale)[0]
    return out
