"""GPU block selection (mean-pool -> fp64 score -> top-k -> CSR) must be
bit-exact against the oracle: same block sets, same fp64 scores, same CSR."""
import math

import numpy as np
import pytest
import torch

from oracle import selection as osel
from sparseattnfunctions_b200 import kernels, workloads
from sparseattnfunctions_b200.geometry import VideoGeometry

pytestmark = pytest.mark.gpu


def _check(dev, q, k, bm, bn, topk, tq=0, tk=0, diag=False, inside=False):
    csr = kernels.pool_topk(q.to(dev), k.to(dev), block_m=bm, block_n=bn, topk=topk,
                            text_blocks_q=tq, text_blocks_k=tk, force_diag=diag,
                            forced_inside_topk=inside, return_mask=True, return_scores=True)
    torch.cuda.synchronize()
    mask_ref, score_ref = osel.select_blocks(q, k, bm, bn, topk, tq, tk, diag, inside)
    scores = csr.scores.cpu().numpy()
    assert np.array_equal(scores.view(np.uint64), score_ref.view(np.uint64)), \
        f"scores differ (max abs {np.abs(scores - score_ref).max():.3e})"
    mask = csr.mask.cpu().numpy().astype(bool)
    assert np.array_equal(mask, mask_ref), f"{(mask != mask_ref).sum()} mask bits differ"
    rp_ref, ci_ref = osel.dense_to_csr(mask_ref)
    rp = csr.row_ptr.cpu().numpy()
    ci = csr.col_idx.cpu().numpy()
    assert np.array_equal(rp, rp_ref)
    for g in range(rp.shape[0]):
        s, e = rp[g, 0], rp[g, -1]
        assert np.array_equal(ci[s:e], ci_ref[s:e])
    return csr


def test_config1_selection(cuda_device):
    """fp32, 64x64 blocks, k = ceil(0.25*32) = 8 per row,
    diagonal forced inside the 8."""
    q, k, _ = workloads.config1_qkv()
    csr = _check(cuda_device, q, k, 64, 64, 8, diag=True, inside=True)
    counts = (csr.row_ptr[:, 1:] - csr.row_ptr[:, :-1]).cpu()
    assert torch.all(counts == 8)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_small_video_selection(cuda_device, dtype):
    geo = VideoGeometry(26, 3, 6, 10)  # 206 tokens
    q, k, _ = workloads.video_qkv(geo, B=2, H=3, dtype=dtype, seed=2)
    _check(cuda_device, q, k, 64, 64, 2, tq=1, tk=1)


def test_ragged_rectangular_selection(cuda_device):
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, 4, 1000, 64, generator=g).to(torch.bfloat16)
    k = torch.randn(1, 4, 1500, 64, generator=g).to(torch.bfloat16)
    _check(cuda_device, q, k, 128, 128, 3, tq=1, tk=2)


def test_ties_prefer_lower_column(cuda_device):
    """Identical key blocks give identical scores; lower columns must win."""
    k = torch.ones(1, 1, 1024, 64, dtype=torch.bfloat16)
    q = torch.ones(1, 1, 1024, 64, dtype=torch.bfloat16)
    csr = _check(cuda_device, q, k, 128, 128, 3)
    dense = csr.to_dense()[0, 0].cpu()
    assert torch.equal(dense[:, :3], torch.ones(8, 3, dtype=torch.bool))
    assert not dense[:, 3:].any()


def test_topk_at_least_nbk(cuda_device):
    g = torch.Generator().manual_seed(4)
    q = torch.randn(1, 2, 500, 64, generator=g).to(torch.bfloat16)
    _check(cuda_device, q, q, 128, 128, 10)


@pytest.mark.parametrize("d", [64, 128])
def test_head_dims(cuda_device, d):
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, 2, 640, d, generator=g).to(torch.bfloat16)
    k = torch.randn(1, 2, 640, d, generator=g).to(torch.bfloat16)
    _check(cuda_device, q, k, 64, 64, 3, tq=1, tk=1)


def test_cogvideox_config2_selection(cuda_device):
    """BASELINE config 2 at full size: S = 17776, 128-blocks, 10% -> k = 14,
    text rows / columns (2 blocks) dense.  Bit-exact against the oracle."""
    from sparseattnfunctions_b200.geometry import COGVIDEOX_2B as geo

    q, k, _ = workloads.video_qkv(geo, B=2, H=30)
    nb = geo.num_blocks(128)
    topk = math.ceil(0.10 * nb)
    csr = _check(cuda_device, q, k, 128, 128, topk, tq=geo.text_blocks(128),
                 tk=geo.text_blocks(128))
    nnz = csr.nnz_per_head().cpu()
    assert int(nnz.max()) <= 2 * nb + (nb - 2) * (topk + 2)


@pytest.mark.parametrize("S,block,topk,tq,tk,diag,inside,d", [
    (4096, 128, 8, 1, 1, False, False, 64),       # 32 key blocks, one row block a warp
    (4096, 128, 8, 1, 2, True, True, 64),         # forced columns counted inside the k
    (260 * 128, 128, 20, 2, 2, False, False, 64),  # 9 columns a lane
    (400 * 64, 64, 30, 0, 0, True, False, 64),    # 16 columns a lane
    (17776, 128, 14, 2, 2, False, False, 128),    # key means staged in two passes of 64 dims
])
def test_integer_inputs_many_ties(cuda_device, S, block, topk, tq, tk, diag, inside, d):
    """Small-integer q / k make many block scores exactly equal (the means
    are exact), so the top-k order among equal scores (lower column first)
    decides most rows; bit-exact against the oracle."""
    g = torch.Generator().manual_seed(S + d)
    q = torch.randint(-2, 3, (1, 2, S, d), generator=g).to(torch.bfloat16)
    k = torch.randint(-2, 3, (1, 2, S, d), generator=g).to(torch.bfloat16)
    _check(cuda_device, q, k, block, block, topk, tq=tq, tk=tk, diag=diag, inside=inside)


def test_nan_and_inf_blocks_rank_like_torch_topk(cuda_device):
    """A NaN in a query block makes that row's scores NaN; infinities make
    +-inf or NaN scores.  NaN ranks above every number (torch.topk's rule,
    which the reference selects with) and NaNs tie to the lower column, so
    such rows keep their first k eligible columns.  Masks and CSR must equal
    the oracle's; scores must agree bit for bit where they are numbers."""
    g = torch.Generator().manual_seed(12)
    q = torch.randn(2, 2, 4096, 64, generator=g).to(torch.bfloat16)
    k = torch.randn(2, 2, 4096, 64, generator=g).to(torch.bfloat16)
    q[0, 0, 300, 5] = float("nan")
    q[1, 1, 700, 3] = float("inf")
    q[0, 1, 1000:1100] = 0
    k[0, 1, 2000:2200] = 0
    k[1, 0, 129, 0] = float("-inf")
    csr = kernels.pool_topk(q.to(cuda_device), k.to(cuda_device), block_m=128, block_n=128, topk=6,
                            text_blocks_q=1, text_blocks_k=1, return_mask=True, return_scores=True)
    torch.cuda.synchronize()
    mask_ref, score_ref = osel.select_blocks(q, k, 128, 128, 6, 1, 1)
    scores = csr.scores.cpu().numpy()
    nan = np.isnan(score_ref)
    assert nan.any() and np.array_equal(np.isnan(scores), nan)
    assert np.array_equal(scores[~nan].view(np.uint64), score_ref[~nan].view(np.uint64))
    mask = csr.mask.cpu().numpy().astype(bool)
    assert np.array_equal(mask, mask_ref), f"{(mask != mask_ref).sum()} mask bits differ"
    rp_ref, ci_ref = osel.dense_to_csr(mask_ref)
    rp, ci = csr.row_ptr.cpu().numpy(), csr.col_idx.cpu().numpy()
    assert np.array_equal(rp, rp_ref)
    for h in range(rp.shape[0]):
        assert np.array_equal(ci[rp[h, 0]:rp[h, -1]], ci_ref[rp[h, 0]:rp[h, -1]])
    # the NaN row (head 0, row block 2): its 6 picks are the lowest columns,
    # text column 0 among them
    assert np.array_equal(np.flatnonzero(mask_ref[0, 0, 2]), np.arange(6))
