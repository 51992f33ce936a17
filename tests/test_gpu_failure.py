"""Failure detection on the GPU without a fault.

* A wait that runs out: saf_selftest_timeout waits on an mbarrier that
  nothing arrives on, with the library's bounded wait; after the budget it
  gives up and SAF_DEV_TIMEOUT appears in the sticky status word.  The
  context stays usable: the next attention launch matches the oracle.
* Out-of-range indices are skipped by the kernels' own bounds checks and
  reported as SAF_DEV_BADINDEX.
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from sparseattnfunctions_b200 import _lib, kernels

pytestmark = [pytest.mark.gpu, pytest.mark.expects_device_status]


def test_wait_that_runs_out_sets_timeout_and_context_survives(cuda_device):
    assert _lib.read_device_status(0, clear=True) == 0
    lib = _lib.load()
    _lib.check("saf_selftest_timeout", lib.saf_selftest_timeout(2_000_000, torch.cuda.current_stream().cuda_stream))
    flags = _lib.read_device_status(0, clear=True)
    assert flags & _lib.SAF_DEV_TIMEOUT
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(2, 2, 1000, 64, generator=g).to(torch.bfloat16) for _ in range(3))
    mask = torch.ones(2, 2, 8, 8, dtype=torch.bool)
    csr = kernels.mask_to_csr(mask.to(cuda_device), 128, 128)
    out = kernels.bsa_fwd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), csr, 0.125)
    torch.cuda.synchronize()
    ref = oatt.block_sparse_attention(q, k, v, mask, 0.125, 128, 128)
    assert np.abs(out.double().cpu().numpy() - ref).max() <= 2e-2
    assert _lib.read_device_status(0, clear=True) == 0


def test_out_of_range_indices_are_flagged_not_followed(cuda_device):
    """A permutation entry outside [0, S) and a CSR column outside [0, nbk)
    are skipped by the kernels' own bounds checks and reported as
    SAF_DEV_BADINDEX."""
    assert _lib.read_device_status(0, clear=True) == 0
    x = torch.randn(1, 2, 100, 64, device=cuda_device).to(torch.bfloat16)
    perm = torch.arange(100, dtype=torch.int32, device=cuda_device)
    perm[7] = 100  # one past the end
    out = torch.zeros_like(x)
    kernels.permute_tokens(x, perm, out=out)
    torch.cuda.synchronize()
    assert _lib.read_device_status(0, clear=True) & _lib.SAF_DEV_BADINDEX
    assert int(torch.count_nonzero(out[:, :, 7])) == 0
    assert torch.equal(out[:, :, 8:], x[:, :, 8:])
    # a CSR column past nbk in one row
    q = torch.randn(1, 1, 256, 64, device=cuda_device).to(torch.bfloat16)
    csr = kernels.mask_to_csr(torch.ones(1, 1, 2, 2, dtype=torch.bool, device=cuda_device), 128, 128)
    csr.col_idx[1] = 5  # row 0 lists columns (0, 5)
    kernels.bsa_fwd(q, q, q, csr, 0.125)
    torch.cuda.synchronize()
    assert _lib.read_device_status(0, clear=True) & _lib.SAF_DEV_BADINDEX


def test_attention_kernel_wait_budget_runs_out_then_recovers(cuda_device):
    """The attention kernel's own abort path: with a 1 ns wait budget its
    first mbarrier wait that does not complete at once gives up, raises the
    CTA's abort flag and SAF_DEV_TIMEOUT, drains its copies and MMAs, frees
    TMEM and returns (no fault, no hang).  With the default budget restored
    and the flag cleared, the next launches -- more than 64, so every
    tile-counter slot is taken again -- give the same result as before."""
    assert _lib.read_device_status(0, clear=True) == 0
    dev = cuda_device
    g = torch.Generator().manual_seed(2)
    B, H, S = 2, 8, 4096
    q, k, v = (torch.randn(B, H, S, 64, generator=g).to(torch.bfloat16) for _ in range(3))
    nb = S // 128
    mask = torch.rand(B, H, nb, nb, generator=g) < 0.25
    mask[..., 0] = True
    csr = kernels.mask_to_csr(mask.to(dev), 128, 128)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    good = kernels.bsa_fwd(qd, kd, vd, csr, 0.125)
    torch.cuda.synchronize()
    assert _lib.read_device_status(0, clear=True) == 0
    ref = oatt.block_sparse_attention(q, k, v, mask, 0.125, 128, 128, heads=[0, 13])
    got = good.double().cpu().numpy()
    for gh in (0, 13):
        b, h = divmod(gh, H)
        assert np.abs(got[b, h] - ref[b, h]).max() <= 2e-2

    old = _lib.get_wait_budget_ns()
    out = torch.zeros_like(qd)
    try:
        _lib.set_wait_budget_ns(1)
        kernels.bsa_fwd(qd, kd, vd, csr, 0.125, out=out)
        torch.cuda.synchronize()
    finally:
        _lib.set_wait_budget_ns(old)
    flags = _lib.read_device_status(0, clear=True)
    assert flags & _lib.SAF_DEV_TIMEOUT
    again = torch.empty_like(qd)
    for _ in range(70):
        kernels.bsa_fwd(qd, kd, vd, csr, 0.125, out=again)
    torch.cuda.synchronize()
    assert _lib.read_device_status(0, clear=True) == 0
    assert torch.equal(again, good)


def test_processor_status_check_raises_on_timeout(cuda_device):
    """BlockSparseAttention(check_status=True) turns a wait that ran out into
    SafTimeoutError on the host; the next call with the default budget is
    clean."""
    from sparseattnfunctions_b200.geometry import VideoGeometry
    from sparseattnfunctions_b200.special_attentions.block_mask_attn import BlockSparseAttention
    from sparseattnfunctions_b200 import workloads

    assert _lib.read_device_status(0, clear=True) == 0
    # large enough that every CTA takes several tiles and some wait does not
    # complete at its first poll
    geo = VideoGeometry(226, 8, 30, 45)
    q, k, v = (t.to(cuda_device) for t in workloads.video_qkv(geo, B=2, H=8, seed=5))
    proc = BlockSparseAttention(block_size=128, density=0.3, geometry=geo, check_status=True)
    good = proc(q, k, v)
    old = _lib.get_wait_budget_ns()
    try:
        _lib.set_wait_budget_ns(1)
        with pytest.raises(_lib.SafTimeoutError):
            proc(q, k, v)
    finally:
        _lib.set_wait_budget_ns(old)
    assert _lib.read_device_status(0, clear=True) == 0  # the raise cleared it
    assert torch.equal(proc(q, k, v), good)
