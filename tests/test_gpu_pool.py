"""Attention with a pooled attention map (attn_pooling_kernel.py) against the
fp64 oracle (oracle/attention.py: attention_with_pooling): the output within
the bf16 / fp16 attention tolerance, the normalised pooled map within 2e-3
(its entries are block-level probabilities; the scores come from 16-bit
inputs with fp32 accumulation, as the reference's bf16 path casts to fp32
before a TF32-capable dot)."""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from sparseattnfunctions_b200 import kernels
from sparseattnfunctions_b200.special_attentions.utils.attn_pooling_kernel import attn_with_pooling

pytestmark = pytest.mark.gpu


def _inputs(B, H, S, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(B, H, S, D, generator=g).to(dtype) for _ in range(3))


@pytest.mark.parametrize("S,bs,dtype", [(1000, 128, torch.bfloat16), (777, 64, torch.bfloat16),
                                        (640, 64, torch.float16)])
def test_attn_with_pooling_dense(cuda_device, S, bs, dtype):
    q, k, v = _inputs(1, 2, S, 64, dtype, seed=S + bs)
    o, po = attn_with_pooling(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), False, 0.125, bs)
    torch.cuda.synchronize()
    ref_o, ref_po = oatt.attention_with_pooling(q, k, v, 0.125, bs)
    nb = math.ceil(S / bs)
    assert o.dtype == dtype and tuple(po.shape) == (1, 2, nb, nb)
    assert po.dtype == (torch.float32 if dtype == torch.bfloat16 else torch.float16)
    assert np.abs(o.double().cpu().numpy() - ref_o).max() <= 2e-2
    got = po.double().cpu().numpy()
    assert np.abs(got - ref_po).max() <= 2e-3
    np.testing.assert_allclose(got.sum(-1), 1.0, atol=1e-3)


def test_pool_map_sparse_blocks(cuda_device):
    """With a block list, blocks a row does not visit pool to 0 and the
    visited ones follow the restricted softmax."""
    B, H, S, bs = 1, 2, 900, 128
    q, k, v = _inputs(B, H, S, 64, torch.bfloat16, seed=5)
    nb = math.ceil(S / bs)
    g = torch.Generator().manual_seed(6)
    mask = torch.rand(B, H, nb, nb, generator=g) < 0.5
    mask[..., 0] = True  # every row sees at least one block
    csr = kernels.mask_to_csr(mask.to(cuda_device), bs, bs)
    o, po = kernels.bsa_fwd_pool(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), csr, 0.125)
    torch.cuda.synchronize()
    ref_o, ref_po = oatt.attention_with_pooling(q, k, v, 0.125, bs, block_mask=mask)
    got = po.double().cpu().numpy()
    assert np.all(got[~mask.numpy()] == 0.0)
    assert np.abs(got - ref_po).max() <= 2e-3
    assert np.abs(o.double().cpu().numpy() - ref_o).max() <= 2e-2


def test_pooling_rejects_what_it_does_not_provide(cuda_device):
    q = torch.zeros(1, 1, 128, 64, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        attn_with_pooling(q, q, q, True, 0.125, 128)
    with pytest.raises(NotImplementedError):
        attn_with_pooling(q.float(), q.float(), q.float(), False, 0.125, 128)
    with pytest.raises(AssertionError):
        attn_with_pooling(q, q, q, False, 0.125, 96)
