"""The reference-facing entry points, called the way the reference's callers
call them, against the CPU oracle.

* ``block_sparse_triton_fn(q, k, v, block_mask, sm_scale)``
  (special_attentions/utils/block_sparse_attn_kernel.py:293): dense 64-block
  boolean mask, bf16; also through ``install_alias()`` and the reference's
  import path.
* ``sparse_attention_factory(128, 128)`` (:283-291).
* ``block_mask_attn.BlockSparseAttention.__call__`` (block_mask_attn.py:26).
* backward raises ``NotImplementedError`` (:278-281).
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import selection as osel
from sparseattnfunctions_b200 import workloads
from sparseattnfunctions_b200.geometry import VideoGeometry

pytestmark = pytest.mark.gpu


def _err(out, ref):
    out = out.float().cpu().numpy().astype(np.float64)
    assert np.array_equal(np.isnan(out), np.isnan(ref))
    ok = ~np.isnan(ref)
    return float(np.abs(out[ok] - ref[ok]).max())


def _inputs(S, seed, B=2, H=3):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S, 64, generator=g).to(torch.bfloat16)
    k = torch.randn(B, H, S, 64, generator=g).to(torch.bfloat16)
    v = torch.randn(B, H, S, 64, generator=g).to(torch.bfloat16)
    return q, k, v


def test_block_sparse_triton_fn_through_alias(cuda_device):
    import sparseattnfunctions_b200

    sparseattnfunctions_b200.install_alias()
    from special_attentions.utils.block_sparse_attn_kernel import (block_sparse_triton_fn,
                                                                   get_sparse_attn_mask_from_topk)

    S = 1000  # 16 blocks of 64, the last one ragged (40 rows)
    q, k, v = _inputs(S, 11)
    nb = math.ceil(S / 64)
    g = torch.Generator().manual_seed(12)
    x = torch.randn(2, 3, nb, nb, generator=g)
    x[..., 0] = 100.0  # the reference KAT's forced first column
    mask = get_sparse_attn_mask_from_topk(x, 4)
    dev = cuda_device
    out = block_sparse_triton_fn(q.to(dev), k.to(dev), v.to(dev), mask.to(dev), 0.125)
    torch.cuda.synchronize()
    ref = oatt.block_sparse_attention(q, k, v, mask.numpy(), 0.125, 64, 64)
    assert _err(out, ref) <= 2e-2


def test_sparse_attention_factory_128(cuda_device):
    from sparseattnfunctions_b200.special_attentions.utils.block_sparse_attn_kernel import \
        sparse_attention_factory

    fn = sparse_attention_factory(128, 128)
    S = 1500
    q, k, v = _inputs(S, 21, B=1, H=4)
    nb = math.ceil(S / 128)
    g = torch.Generator().manual_seed(22)
    mask = torch.rand(1, 4, nb, nb, generator=g) < 0.4
    mask[..., 0] = True
    dev = cuda_device
    out = fn(q.to(dev), k.to(dev), v.to(dev), mask.to(dev), 0.125)
    torch.cuda.synchronize()
    ref = oatt.block_sparse_attention(q, k, v, mask.numpy(), 0.125, 128, 128)
    assert _err(out, ref) <= 2e-2


def test_backward_raises(cuda_device):
    from sparseattnfunctions_b200.special_attentions.utils.block_sparse_attn_kernel import \
        block_sparse_triton_fn

    q, k, v = (t.to(cuda_device).requires_grad_() for t in _inputs(128, 31, B=1, H=1))
    mask = torch.ones(1, 1, 2, 2, dtype=torch.bool, device=cuda_device)
    out = block_sparse_triton_fn(q, k, v, mask, 0.125)
    with pytest.raises(NotImplementedError):
        out.float().sum().backward()


def test_block_mask_attn_processor_call(cuda_device):
    """BlockSparseAttention(q, k, v) on a small CogVideoX-shaped geometry:
    the processor's own block selection equals the oracle's, and its output
    is the oracle's attention over that selection."""
    from sparseattnfunctions_b200.special_attentions.block_mask_attn import BlockSparseAttention

    geo = VideoGeometry(226, 3, 12, 20)  # 226 text + 3 frames of 240 tokens = 946
    q, k, v = workloads.video_qkv(geo, B=2, H=2, seed=41)
    dev = cuda_device
    proc = BlockSparseAttention(block_size=128, density=0.25, geometry=geo)
    out = proc(q.to(dev), k.to(dev), v.to(dev))
    torch.cuda.synchronize()
    nb = geo.num_blocks(128)
    tb = geo.text_blocks(128)
    mask_ref, _ = osel.select_blocks(q, k, 128, 128, math.ceil(0.25 * nb), tb, tb)
    assert np.array_equal(proc.last_csr.to_dense().cpu().numpy(), mask_ref)
    ref = oatt.block_sparse_attention(q, k, v, mask_ref, 0.125, 128, 128)
    assert _err(out, ref) <= 2e-2
