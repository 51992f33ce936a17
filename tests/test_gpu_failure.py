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
