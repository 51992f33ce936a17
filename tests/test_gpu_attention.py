"""GPU parity of the block-sparse attention kernels against the CPU oracle.

Tolerances (from the build target): 2e-2 max-abs for bf16 / f16 outputs,
1e-4 for fp32.  The oracle evaluates the reference's kron-mask definition
(special_attentions/utils/block_sparse_attn_kernel.py:326-334) in fp64 on
the same (rounded) inputs.
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import selection as osel
from sparseattnfunctions_b200 import kernels

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 2e-2, torch.float16: 2e-2, torch.float32: 1e-4}


def _inputs(B, H, Sq, Sk, D, dtype, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, H, Sq, D, generator=g) * scale).to(dtype)
    k = (torch.randn(B, H, Sk, D, generator=g) * scale).to(dtype)
    v = torch.randn(B, H, Sk, D, generator=g).to(dtype)
    return q, k, v


def _random_mask(B, H, nbq, nbk, density, seed, empty_rows=0):
    g = torch.Generator().manual_seed(seed + 7)
    m = torch.rand(B, H, nbq, nbk, generator=g) < density
    m[..., 0] = True  # keep most rows non-empty
    if empty_rows:
        rows = torch.randint(0, nbq, (empty_rows,), generator=g)
        m[0, 0, rows, :] = False
    return m


def _compare(out, ref, tol):
    out = out.float().cpu().numpy().astype(np.float64)
    nan_o, nan_r = np.isnan(out), np.isnan(ref)
    assert np.array_equal(nan_o, nan_r), "NaN rows differ from the oracle"
    err = np.abs(out[~nan_r] - ref[~nan_r]).max() if (~nan_r).any() else 0.0
    assert err <= tol, f"max abs error {err:.3e} > {tol:.1e}"
    return err


def _run(dev, B, H, Sq, Sk, D, dtype, bm, bn, density, seed, bias=False, empty_rows=0):
    q, k, v = _inputs(B, H, Sq, Sk, D, dtype, seed)
    nbq, nbk = math.ceil(Sq / bm), math.ceil(Sk / bn)
    mask = _random_mask(B, H, nbq, nbk, density, seed, empty_rows)
    kv_bias = None
    if bias:
        g = torch.Generator().manual_seed(seed + 99)
        kv_bias = torch.rand(B * H, Sk, generator=g) * 3.0
    csr = kernels.mask_to_csr(mask.to(dev), bm, bn)
    scale = 1.0 / math.sqrt(D)
    out = kernels.bsa_fwd(q.to(dev), k.to(dev), v.to(dev), csr, scale,
                          kv_bias=None if kv_bias is None else kv_bias.to(dev))
    torch.cuda.synchronize()
    ref = oatt.block_sparse_attention(q, k, v, mask, scale, bm, bn, kv_bias=kv_bias)
    return _compare(out, ref, TOL[dtype])


def test_reference_kat_ragged_dense(cuda_device):
    """block_sparse_attn_kernel.py:296-339: B1 H3 S257 D64 bf16, 64-blocks,
    mask overridden to all ones; ragged last block (257 = 4*64 + 1)."""
    B, H, S, D = 1, 3, 257, 64
    q, k, v = _inputs(B, H, S, S, D, torch.bfloat16, seed=0)
    mask = torch.ones(B, H, 5, 5, dtype=torch.bool)
    csr = kernels.mask_to_csr(mask.to(cuda_device), 64, 64)
    out = kernels.bsa_fwd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), csr, 1 / 8)
    ref = oatt.block_sparse_attention(q, k, v, mask, 1 / 8, 64, 64)
    _compare(out, ref, 2e-2)


def test_reference_kat_qlen_lt_klen(cuda_device):
    """block_sparse_attn_kernel.py:343-390: q 128 < k 256, top-1 block with
    column 0 forced to the top, so only kv block 0 is live."""
    B, H, Sq, Sk, D = 2, 4, 128, 256, 64
    q, k, v = _inputs(B, H, Sq, Sk, D, torch.bfloat16, seed=0)
    g = torch.Generator().manual_seed(0)
    x_ds = torch.randn(B, H, 4, 4, generator=g)
    x_ds[:, :, :, 0] = 100
    mask = torch.from_numpy(osel.reference_topk_mask(x_ds.numpy(), 1))[:, :, :2, :]
    csr = kernels.mask_to_csr(mask.to(cuda_device), 64, 64)
    out = kernels.bsa_fwd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), csr, 1 / 8)
    ref = oatt.block_sparse_attention(q, k, v, mask, 1 / 8, 64, 64)
    _compare(out, ref, 2e-2)


@pytest.mark.parametrize("bm,bn", [(128, 128), (64, 64), (64, 128), (128, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_block_sizes(cuda_device, bm, bn, dtype):
    _run(cuda_device, 2, 3, 1000, 1000, 64, dtype, bm, bn, 0.35, seed=bm + bn)


@pytest.mark.parametrize("Sq,Sk", [(129, 129), (300, 700), (1500, 640), (64, 64), (1, 200)])
def test_ragged_lengths(cuda_device, Sq, Sk):
    _run(cuda_device, 1, 2, Sq, Sk, 64, torch.bfloat16, 128, 128, 0.5, seed=Sq * 7 + Sk)


def test_empty_rows_give_nan(cuda_device):
    _run(cuda_device, 1, 2, 900, 900, 64, torch.bfloat16, 128, 128, 0.3, seed=5, empty_rows=3)


def test_empty_rows_block64(cuda_device):
    _run(cuda_device, 1, 2, 900, 900, 64, torch.bfloat16, 64, 64, 0.3, seed=6, empty_rows=4)


@pytest.mark.parametrize("bn", [128, 64])
def test_kv_bias(cuda_device, bn):
    _run(cuda_device, 2, 2, 777, 1111, 64, torch.bfloat16, 128, bn, 0.4, seed=11, bias=True)


@pytest.mark.parametrize("dtype,bn", [(torch.float16, 128), (torch.float16, 64), (torch.bfloat16, 128)])
def test_kv_bias_masking_values(cuda_device, dtype, bn):
    """The bias enters S through the tensor cores in the input's 16-bit type:
    -inf keys must vanish, large negative biases must act as masks, and a
    head whose keys are all -inf in one block must still see its other
    blocks (the bias is per head)."""
    B, H, Sq, Sk, D = 1, 2, 600, 700, 64
    q, k, v = _inputs(B, H, Sq, Sk, D, dtype, seed=41)
    mask = torch.ones(B, H, math.ceil(Sq / 128), math.ceil(Sk / bn), dtype=torch.bool)
    g = torch.Generator().manual_seed(42)
    bias = torch.log(torch.randint(1, 14, (B * H, Sk), generator=g).float())
    bias[:, 5:40] = float("-inf")
    bias[:, 100:130] = -1.0e4
    bias[1, bn:2 * bn] = float("-inf")  # a whole key block of head 1
    csr = kernels.mask_to_csr(mask.to(cuda_device), 128, bn)
    out = kernels.bsa_fwd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), csr, 1 / 8,
                          kv_bias=bias.to(cuda_device))
    torch.cuda.synchronize()
    ref = oatt.block_sparse_attention(q, k, v, mask, 1 / 8, 128, bn, kv_bias=bias)
    _compare(out, ref, TOL[dtype])


def test_dense_long_rows(cuda_device):
    """Every block live (the dense path of MergeAttention) at S = 4000."""
    _run(cuda_device, 1, 2, 4000, 4000, 64, torch.bfloat16, 128, 128, 1.01, seed=3)


def test_large_logits_rescale(cuda_device):
    """Logit scale large enough that the running max jumps by far more than
    the lazy-rescale threshold between blocks."""
    B, H, S, D = 1, 2, 1024, 64
    q, k, v = _inputs(B, H, S, S, D, torch.bfloat16, seed=21, scale=3.0)
    mask = _random_mask(B, H, 8, 8, 0.6, seed=21)
    csr = kernels.mask_to_csr(mask.to(cuda_device), 128, 128)
    out = kernels.bsa_fwd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), csr, 0.125)
    ref = oatt.block_sparse_attention(q, k, v, mask, 0.125, 128, 128)
    _compare(out, ref, 2e-2)


def test_strided_views(cuda_device):
    """q/k/v as [B, S, H, D] storage viewed as [B, H, S, D] (non-contiguous)."""
    B, H, S, D = 2, 3, 600, 64
    g = torch.Generator().manual_seed(8)
    base = [torch.randn(B, S, H, D, generator=g).to(torch.bfloat16) for _ in range(3)]
    q, k, v = (t.transpose(1, 2) for t in base)
    mask = _random_mask(B, H, 5, 5, 0.5, seed=8)
    csr = kernels.mask_to_csr(mask.to(cuda_device), 128, 128)
    out = kernels.bsa_fwd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), csr, 0.125)
    ref = oatt.block_sparse_attention(q, k, v, mask, 0.125, 128, 128)
    _compare(out, ref, 2e-2)


@pytest.mark.parametrize("bm,bn", [(64, 64), (128, 128), (64, 128)])
def test_fp32_path(cuda_device, bm, bn):
    _run(cuda_device, 1, 2, 700, 900, 64, torch.float32, bm, bn, 0.4, seed=31)


def test_fp32_d128_bias(cuda_device):
    _run(cuda_device, 1, 2, 300, 300, 128, torch.float32, 64, 64, 0.5, seed=32, bias=True)


def test_mask_to_csr_matches_oracle(cuda_device):
    mask = _random_mask(2, 3, 17, 23, 0.3, seed=4, empty_rows=2)
    csr = kernels.mask_to_csr(mask.to(cuda_device), 64, 64)
    rp_ref, ci_ref = osel.dense_to_csr(mask.numpy())
    rp = csr.row_ptr.cpu().numpy()
    ci = csr.col_idx.cpu().numpy()
    assert np.array_equal(rp, rp_ref)
    for g in range(rp.shape[0]):
        s, e = rp[g, 0], rp[g, -1]
        assert np.array_equal(ci[s:e], ci_ref[s:e])
    assert torch.equal(csr.to_dense().cpu(), mask)


def test_rejects_cpu_tensors():
    q = torch.zeros(1, 1, 64, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        kernels.bsa_fwd(q, q, q, None, 0.125)


@pytest.mark.parametrize("bm", [128, 64])
def test_lead_rows_schedule_does_not_change_results(cuda_device, bm):
    """The dense-row hint reorders the work and, with few heads per GPU,
    splits the lead tiles' key blocks over several work items merged per row
    (fp32 partials): outputs stay within the oracle's tolerance and within
    one output rounding of the unsplit launch; the rows outside the lead
    tiles are bitwise identical."""
    B, H, S, D = 2, 3, 1500, 64
    q, k, v = (t.to(cuda_device) for t in _inputs(B, H, S, S, D, torch.bfloat16, seed=41))
    nb = math.ceil(S / bm)
    mask = _random_mask(B, H, nb, nb, 0.3, seed=41).to(cuda_device)
    mask[:, :, :3, :] = True
    outs = []
    for lead in (0, 3, 100):
        csr = kernels.mask_to_csr(mask, bm, bm, dense_rows=lead)
        outs.append(kernels.bsa_fwd(q, k, v, csr, 0.125))
    torch.cuda.synchronize()
    ref = oatt.block_sparse_attention(q.cpu(), k.cpu(), v.cpu(), mask.cpu().numpy(), 0.125, bm, bm)
    for o in outs:
        _compare(o, ref, 2e-2)
    # lead = 3 mask rows: the split covers the first ceil(3 * bm / 128) tiles
    split_rows = math.ceil(3 * bm / 128) * 128
    assert torch.equal(outs[0][:, :, split_rows:], outs[1][:, :, split_rows:])
    for o in outs[1:]:
        assert float((o.float() - outs[0].float()).abs().max()) <= 2e-2
