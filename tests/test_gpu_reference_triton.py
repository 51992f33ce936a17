"""This package's kernels against the reference's own Triton kernels, run on
the same GPU and the same inputs (the reference installed unmodified in
baseline/_ref; see baseline/reference_kernels.py).

* block_sparse_triton_fn (block_sparse_attn_kernel.py:293) against
  saf_bsa_fwd: bf16 within 2e-2 of each other (both round P to bf16 before
  the PV product), on a ragged length with a 64-block top-k mask; and the
  config-1 fp32 case, where the reference's tl.dot runs in TF32, so each is
  compared with the fp64 oracle at its own precision.
* attn_with_pooling (attn_pooling_kernel.py:289) against saf_bsa_fwd_pool:
  output within 2e-2, pooled map within 1e-2 (the reference computes in
  fp32 with TF32 dots and stores the map in bf16).

Skipped when the reference is not installed in baseline/_ref.
"""
import math
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from baseline import reference_kernels as rk  # noqa: E402
from oracle import attention as oatt  # noqa: E402
from sparseattnfunctions_b200 import kernels, workloads  # noqa: E402

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not rk.available(), reason="reference not installed in baseline/_ref")]


def test_block_sparse_kernel_matches_reference_triton(cuda_device):
    bsk = rk.load("block_sparse_attn_kernel")
    dev = cuda_device
    g = torch.Generator().manual_seed(7)
    B, H, S = 2, 4, 1000
    q, k, v = (torch.randn(B, H, S, 64, generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
    nb = math.ceil(S / 64)
    x = torch.randn(B, H, nb, nb, generator=g)
    x[..., 0] = 100.0
    mask = bsk.get_sparse_attn_mask_from_topk(x, 5).to(dev)
    ref = bsk.block_sparse_triton_fn(q, k, v, mask, 0.125)
    ours = kernels.bsa_fwd(q, k, v, kernels.mask_to_csr(mask, 64, 64), 0.125)
    torch.cuda.synchronize()
    assert float((ref.float() - ours.float()).abs().max()) <= 2e-2


def test_config1_fp32_against_reference_triton(cuda_device):
    bsk = rk.load("block_sparse_attn_kernel")
    dev = cuda_device
    q, k, v = workloads.config1_qkv()
    csr = kernels.pool_topk(q.to(dev), k.to(dev), block_m=64, block_n=64, topk=8, force_diag=True,
                            forced_inside_topk=True)
    mask = csr.to_dense()
    ours = kernels.bsa_fwd(q.to(dev), k.to(dev), v.to(dev), csr, 0.125)
    ref = bsk.block_sparse_triton_fn(q.to(dev), k.to(dev), v.to(dev), mask.contiguous(), 0.125)
    torch.cuda.synchronize()
    exact = oatt.block_sparse_attention(q, k, v, mask.cpu().numpy(), 0.125, 64, 64)
    err_ours = np.abs(ours.double().cpu().numpy() - exact).max()
    err_ref = np.abs(ref.double().cpu().numpy() - exact).max()
    assert err_ours <= 1e-4
    assert err_ref <= 1e-2  # TF32 dots in the reference kernel
    assert float((ref - ours).abs().max()) <= 1e-2


def test_pooled_attention_matches_reference_triton(cuda_device):
    pk = rk.load("attn_pooling_kernel")
    dev = cuda_device
    g = torch.Generator().manual_seed(8)
    B, H, S = 1, 3, 1024  # whole 64-blocks: the reference's block pointers are not bounds-checked
    q, k, v = (torch.randn(B, H, S, 64, generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
    o_ref, p_ref = pk.attn_with_pooling(q, k, v, False, 0.125, 64)
    dense = kernels.mask_to_csr(torch.ones(B, H, S // 64, S // 64, dtype=torch.bool, device=dev), 64, 64)
    o, p = kernels.bsa_fwd_pool(q, k, v, dense, 0.125, pool_block=64)
    torch.cuda.synchronize()
    assert float((o_ref.float() - o.float()).abs().max()) <= 2e-2
    assert float((p_ref.float() - p).abs().max()) <= 1e-2
