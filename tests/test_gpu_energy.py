"""GPU energy-threshold block selection (saf_energy_select) and the
SparseGen_Plus processor.

* Block masks from the reference's own transfer_attn_to_mask outputs
  (tests/golden/energy_masks.npz, made by running the reference) are
  reproduced bit for bit from the same inputs.
* Pooled-score mode: the mask equals the oracle rule applied to the mass the
  kernel reports, bit for bit.
* The processor's output is within 2e-2 of the fp64 oracle on its own mask.
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import selection as osel
from sparseattnfunctions_b200 import kernels
from sparseattnfunctions_b200.special_attentions import SparseGen_Plus as sgp
import importlib.util
from pathlib import Path

GOLDEN = Path(__file__).resolve().parent / "golden"
_spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
mg = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(mg)

pytestmark = pytest.mark.gpu


def test_energy_masks_match_reference_outputs(cuda_device):
    data = np.load(GOLDEN / "energy_masks.npz")
    for seed, B, H, n, thr, mn, mx in data["cases"]:
        a = torch.from_numpy(mg.energy_input(int(seed), int(B), int(H), int(n))).to(cuda_device)
        got = sgp.transfer_attn_to_mask(a, mode="energy", max_retain_ratio=float(mx),
                                        min_retain_ratio=float(mn), energy_threshold=float(thr))
        assert np.array_equal(got.cpu().numpy(), data[f"case_{int(seed)}"])


@pytest.mark.parametrize("S,bs,thr", [(1000, 64, 0.9), (2300, 64, 0.98), (1777, 128, 0.95)])
def test_pooled_mode_matches_oracle_rule(cuda_device, S, bs, thr):
    g = torch.Generator().manual_seed(S)
    q = torch.randn(2, 3, S, 64, generator=g).to(torch.bfloat16).to(cuda_device)
    k = torch.randn(2, 3, S, 64, generator=g).to(torch.bfloat16).to(cuda_device)
    pooled = kernels.pool_topk(q, k, block_m=bs, block_n=bs, topk=1, return_scores=True)
    nbk = pooled.nbk
    mn, mx = max(1, int(nbk * 0.1)), max(1, int(nbk * 0.8))
    mask, mass = kernels.energy_select(pooled.scores, threshold=thr, min_retain=mn, max_retain=mx,
                                       text_blocks=2, is_mass=False, scale=0.125, block_n=bs, Sk=S,
                                       return_mass=True)
    ref = osel.energy_select(mass.cpu().numpy(), thr, 0.1, 0.8, text_blocks=2)
    assert np.array_equal(mask.cpu().numpy().astype(bool), ref)
    # the mass follows its definition (block-size-weighted softmax numerator)
    s = pooled.scores.cpu().numpy() * 0.125
    cols = np.full(nbk, float(bs))
    cols[-1] = S - (nbk - 1) * bs
    want = cols * np.exp(s - s.max(axis=-1, keepdims=True))
    np.testing.assert_allclose(mass.cpu().numpy(), want, rtol=1e-12, atol=0)


def test_sparsegen_plus_processor(cuda_device):
    B, H, S, D = 1, 2, 1500, 64
    g = torch.Generator().manual_seed(4)
    q, k, v = (torch.randn(B, H, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    attn = sgp.BlockSparseAttention(layernum=1, timestep=10, warmup_epoch=1)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    dense = attn(qd, kd, vd)  # warm-up step: every block live
    nb = math.ceil(S / 64)
    ref_dense = oatt.block_sparse_attention(q, k, v, np.ones((B, H, nb, nb), bool), 1 / 8, 64, 64)
    assert np.abs(dense.double().cpu().numpy() - ref_dense).max() <= 2e-2
    out = attn(qd, kd, vd)    # step 1: energy-selected blocks
    csr = attn.mask[0]
    mask = csr.to_dense().cpu().numpy()
    max_r, min_r, thr = attn.schedule(1)
    ref_mask = osel.energy_select(attn.last_mass.cpu().numpy(), thr, min_r, max_r, text_blocks=4)
    assert np.array_equal(mask, ref_mask)
    assert mask.mean() < 1.0
    ref = oatt.block_sparse_attention(q, k, v, mask, 1 / 8, 64, 64)
    assert np.abs(out.double().cpu().numpy() - ref).max() <= 2e-2
    assert attn.sparsity_records[0]["records"][-1]["layer"] == 0


def test_sparsegen_plus_warmup_pooling(cuda_device):
    """warmup_pooling: the warm-up step returns the dense attention and keeps
    its pooled map; the first sparse step of the layer selects its blocks by
    the energy rule on that map (checked against the oracle's pooled map)."""
    B, H, S, D = 1, 2, 1100, 64
    g = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(B, H, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    attn = sgp.BlockSparseAttention(layernum=1, timestep=10, warmup_epoch=1, warmup_pooling=True)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    dense = attn(qd, kd, vd)
    ref_o, ref_pool = oatt.attention_with_pooling(q, k, v, 1 / 8, 64)
    assert np.abs(dense.double().cpu().numpy() - ref_o).max() <= 2e-2
    wmap = attn.warmup_map[0].double().cpu().numpy()
    assert np.abs(wmap - ref_pool).max() <= 2e-3
    out = attn(qd, kd, vd)  # step 1: blocks from the warm-up map
    assert attn.warmup_map[0] is None
    mask = attn.mask[0].to_dense().cpu().numpy()
    max_r, min_r, thr = attn.schedule(1)
    ref_mask = osel.energy_select(wmap, thr, min_r, max_r, text_blocks=4)
    assert np.array_equal(mask, ref_mask)
    ref = oatt.block_sparse_attention(q, k, v, mask, 1 / 8, 64, 64)
    assert np.abs(out.double().cpu().numpy() - ref).max() <= 2e-2


def test_topk_mode_matches_reference_outputs(cuda_device):
    """transfer_attn_to_mask(mode="topk") on the GPU against the reference's
    own masks (tests/golden/topk_adaptive_masks.npz): bit-exact."""
    import importlib.util
    from pathlib import Path

    from sparseattnfunctions_b200.special_attentions.SparseGen_Plus import transfer_attn_to_mask

    golden = Path(__file__).resolve().parent / "golden"
    spec = importlib.util.spec_from_file_location("make_golden", golden / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    data = np.load(golden / "topk_adaptive_masks.npz")
    for seed, B, H, n, init_k, power in data["cases"]:
        a = torch.from_numpy(mg.topk_adaptive_input(int(seed), int(B), int(H), int(n), float(power)))
        init = float(init_k) if init_k < 1 else int(init_k)
        got = transfer_attn_to_mask(a.to(cuda_device), mode="topk", init_k=init)
        assert np.array_equal(got.cpu().numpy(), data[f"case_{int(seed)}"]), f"case {int(seed)}"
