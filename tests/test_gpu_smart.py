"""GPU parity of the frame-band attention path (SmartAttention) against the
CPU oracle (oracle/smart.py, pinned to the reference's SmartAttention
functions by tests/golden/smart_layout.npz).

* saf_bsa_fwd_ranges: per-row key intervals on top of the block list,
  bf16 / f16 (tcgen05 kernel) and fp32 (CUDA-core kernel) -- 2e-2 / 1e-4.
* saf_permute_tokens: exact gathers.
* SmartAttention with a given strategy and with its own probe.
"""
import math

import numpy as np
import pytest
import torch

from oracle import smart as osm
from sparseattnfunctions_b200 import kernels
from sparseattnfunctions_b200.geometry import VideoGeometry, video_token_perm
from sparseattnfunctions_b200.special_attentions.SmartAttention import SmartAttention

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 2e-2, torch.float16: 2e-2, torch.float32: 1e-4}
GEOM = VideoGeometry(26, 5, 10, 15)  # S = 776


def _qkv(B, H, Sq, Sk, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, H, Sq, D, generator=g).to(dtype), torch.randn(B, H, Sk, D, generator=g).to(dtype),
            torch.randn(B, H, Sk, D, generator=g).to(dtype))


def _random_ranges(Sq, Sk, seed):
    g = np.random.RandomState(seed)
    r = np.zeros((Sq, 4), dtype=np.int32)
    for i in range(Sq):
        a = g.randint(0, Sk)
        r[i, 0], r[i, 1] = a, min(Sk, a + g.randint(1, 300))
        if g.rand() < 0.6:
            c = g.randint(0, Sk)
            r[i, 2], r[i, 3] = c, min(Sk, c + g.randint(0, 200))
    r[:5] = [0, Sk, 0, 0]      # full rows
    r[5:9] = [10, 10, 40, 40]  # rows with no key at all -> NaN
    return r


@pytest.mark.parametrize("dtype,bm,bn", [(torch.bfloat16, 128, 128), (torch.bfloat16, 64, 64),
                                         (torch.float16, 64, 128), (torch.float32, 64, 64)])
def test_row_ranges_against_oracle(cuda_device, dtype, bm, bn):
    B, H, Sq, Sk, D = 1, 2, 700, 900, 64
    q, k, v = _qkv(B, H, Sq, Sk, D, dtype, seed=bm + bn)
    r = _random_ranges(Sq, Sk, seed=bn)
    g = torch.Generator().manual_seed(4)
    nbq, nbk = math.ceil(Sq / bm), math.ceil(Sk / bn)
    block = torch.rand(B, H, nbq, nbk, generator=g) < 0.7
    csr = kernels.mask_to_csr(block.to(cuda_device), bm, bn)
    out = kernels.bsa_fwd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), csr, 1 / 8,
                          row_ranges=torch.from_numpy(r).to(cuda_device))
    allowed = osm.ranges_mask(r, Sk)[None, None] & \
        np.repeat(np.repeat(block.numpy(), bm, axis=2), bn, axis=3)[:, :, :Sq, :Sk]
    ref = osm.masked_attention(q, k, v, allowed, 1 / 8)
    got = out.double().cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.abs(got[ok] - ref[ok]).max() <= TOL[dtype]


def test_row_ranges_rejects_bias(cuda_device):
    q = torch.zeros(1, 1, 128, 64, dtype=torch.bfloat16, device=cuda_device)
    csr = kernels.mask_to_csr(torch.ones(1, 1, 1, 1, dtype=torch.bool, device=cuda_device), 128, 128)
    r = torch.tensor([[0, 128, 0, 0]] * 128, dtype=torch.int32, device=cuda_device)
    with pytest.raises(Exception):
        kernels.bsa_fwd(q, q, q, csr, 0.125, kv_bias=torch.zeros(128, device=cuda_device), row_ranges=r)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_permute_tokens(cuda_device, dtype):
    g = torch.Generator().manual_seed(1)
    base = torch.randn(2, GEOM.seq_len, 3, 64, generator=g).to(dtype).to(cuda_device)
    x = base.transpose(1, 2)  # strided [B, H, S, D]
    perm, inv = video_token_perm(GEOM, cuda_device)
    y = kernels.permute_tokens(x, perm)
    assert torch.equal(y, x[:, :, perm.long()])
    heads = torch.tensor([1, 5], dtype=torch.int32, device=cuda_device)  # flat b*H + h
    out = torch.zeros_like(x)
    kernels.permute_tokens(y, inv, heads, out=out)
    assert torch.equal(out[0, 1], x[0, 1]) and torch.equal(out[1, 2], x[1, 2])
    assert int(torch.count_nonzero(out[0, 0])) == 0 and int(torch.count_nonzero(out[1, 0])) == 0


def test_smart_attention_given_strategy(cuda_device):
    B, H, D = 2, 3, 64
    q, k, v = _qkv(B, H, GEOM.seq_len, GEOM.seq_len, D, torch.bfloat16, seed=7)
    strategy = torch.tensor([[True, False, True], [False, False, True]])
    sa = SmartAttention(geometry=GEOM, block_size=64)
    out = sa(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), strategy=strategy)
    ref = osm.smart_attention(q, k, v, strategy.numpy(), GEOM.text_len, GEOM.frames, GEOM.height, GEOM.width)
    assert np.abs(out.double().cpu().numpy() - ref).max() <= 2e-2


@pytest.mark.parametrize("block", [64, 128])
def test_smart_attention_probe(cuda_device, block):
    """The probe's three outputs match the oracle on the same sampled rows;
    the chosen strategy matches wherever the two distances differ by more
    than the outputs' error can move them."""
    B, H, D = 1, 4, 64
    q, k, v = _qkv(B, H, GEOM.seq_len, GEOM.seq_len, D, torch.bfloat16, seed=block)
    sa = SmartAttention(geometry=GEOM, block_size=block, generator=torch.Generator().manual_seed(3))
    out = sa(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    pr = sa.last_probe
    sd, td, full, sp, tp = osm.probe(q, k, v, pr["idx"].numpy(), GEOM.text_len, GEOM.frames, GEOM.height,
                                     GEOM.width)
    for got, ref in ((pr["full"], full), (pr["spatial"], sp), (pr["temporal"], tp)):
        assert np.abs(got.double().cpu().numpy() - ref).max() <= 2e-2
    strat = sa.last_strategy.cpu().numpy()
    n = pr["idx"].numel() * D
    d = 2e-2  # per-element error bound of each output
    clear = np.abs(sd - td) > 4 * d * (np.sqrt(n * sd) + np.sqrt(n * td)) + 8 * n * d * d
    assert np.array_equal(strat[clear], (sd < td)[clear])
    ref = osm.smart_attention(q, k, v, strat, GEOM.text_len, GEOM.frames, GEOM.height, GEOM.width)
    assert np.abs(out.double().cpu().numpy() - ref).max() <= 2e-2
