"""Drop-in for special_attentions/utils/block_sparse_attn_kernel.py.

Same public names and call signatures as the reference module; the Triton
kernel is replaced by the sm_100a library (``libsaf.so``):

* ``block_sparse_triton_fn(q, k, v, block_mask, sm_scale)`` -- reference
  :293.  ``block_mask`` is a dense boolean ``[B, H, >=ceil(Sq/64),
  >=ceil(Sk/64)]`` mask over 64 x 64 blocks (the reference kernel's
  BLOCK_M = BLOCK_N = 64, :218-219); extra rows / columns are ignored, as the
  reference kernel never reads them.  The mask is converted to a CSR block
  list on the device and only live blocks are computed.
* ``sparse_attention_factory(BLOCK_M, BLOCK_N)`` -- reference :283-291, for
  other block sizes (64 or 128 on the tensor-core path).
* ``get_sparse_attn_mask_from_topk`` / ``get_sparse_attn_mask_from_threshold``
  -- reference :31-47 (torch ops on the mask's device).

Backward raises ``NotImplementedError`` as the reference does (:278-281).
Asserts mirror :226-231 (``AssertionError`` on mismatched head dims /
sequence lengths; D must be 64 or 128).
"""
from __future__ import annotations

import math

import torch

from ... import kernels


def get_sparse_attn_mask_from_topk(x, topk, use_dense_for_last_block=False):
    bsz, num_head, downsample_len, _ = x.shape
    sparse_index = torch.topk(x, topk, dim=-1).indices
    dense_mask = torch.zeros([bsz, num_head, downsample_len, downsample_len], dtype=torch.bool,
                             device=x.device)
    dense_mask.scatter_(-1, sparse_index, True)
    if use_dense_for_last_block:
        dense_mask[:, :, -2:, :] = True
    return dense_mask


def get_sparse_attn_mask_from_threshold(x, threshold, use_dense_for_last_block=False):
    dense_mask = x > threshold
    if use_dense_for_last_block:
        dense_mask[:, :, -2:, :] = True
    dense_mask.tril_()
    return dense_mask


def _forward(q, k, v, block_sparse_mask, sm_scale, BLOCK_M=64, BLOCK_N=64, out=None):
    assert q.shape[-1] == k.shape[-1] == v.shape[-1]
    assert k.shape[2] == v.shape[2]
    assert q.shape[-1] in [64, 128]
    nbq, nbk = math.ceil(q.shape[2] / BLOCK_M), math.ceil(k.shape[2] / BLOCK_N)
    m = block_sparse_mask
    if m.shape[-2] < nbq or m.shape[-1] < nbk:
        raise ValueError(f"block mask {tuple(m.shape)} is smaller than [{nbq}, {nbk}] blocks")
    m = m[..., :nbq, :nbk]
    if m.shape[0] != q.shape[0] or m.shape[1] != q.shape[1]:
        m = m.expand(q.shape[0], q.shape[1], nbq, nbk)
    csr = kernels.mask_to_csr(m.to(q.device), BLOCK_M, BLOCK_N)
    return kernels.bsa_fwd(q, k, v, csr, sm_scale, out=out)


class _sparse_attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, block_sparse_dense, sm_scale):
        return _forward(q, k, v, block_sparse_dense, sm_scale)

    @staticmethod
    def backward(ctx, do):
        raise NotImplementedError("It does not support gradient propagation yet")


def sparse_attention_factory(BLOCK_M=64, BLOCK_N=64, **kwargs):
    class _sparse_attention_config(_sparse_attention):
        @staticmethod
        def forward(ctx, q, k, v, block_sparse_dense, sm_scale):
            return _forward(q, k, v, block_sparse_dense, sm_scale, BLOCK_M, BLOCK_N)

    return _sparse_attention_config.apply


block_sparse_triton_fn = _sparse_attention.apply
