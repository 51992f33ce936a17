"""Frame-scope masks on the GPU (BlockSparseAttention.forward_backup's path,
special_attentions/utils/mask_related.py:194-245 and block_mask_attn.py:11-20)
against the CPU oracle (oracle/frame_scope.py, itself pinned to the
reference's generate_attention_mask_frame_scope by tests/golden/frame_scope.npz).

* saf_frame_mask: the frame map within 1e-6 (relative) of the fp64 oracle on
  the same values and the mask bit-exact, on the golden cases (whose
  cumulative sums stay >= 1.4e-3 of the total away from the threshold, far
  above the kernel's fp32-logit error); the golden mask itself is matched.
* saf_frame_csr: the listed blocks equal the oracle's block expansion of the
  token-level frame mask, for 128- and 64-blocks.
* saf_bsa_fwd_frames: within 2e-2 of the fp64 oracle that masks token by
  token, for 128- and 64-blocks, bf16 and f16.
* forward_backup at the CogVideoX-2B shape (B=1, H=2): mask equal to the
  oracle's, sampled attention rows within 2e-2.
"""
import importlib.util
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import frame_scope as ofs
from oracle import selection as osel
from sparseattnfunctions_b200 import kernels, workloads
from sparseattnfunctions_b200.geometry import COGVIDEOX_2B, VideoGeometry

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
_spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
mg = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(mg)


@pytest.mark.parametrize("case", [c[0] for c in mg.FRAME_CASES])
def test_frame_mask_matches_golden_and_oracle(cuda_device, case):
    d = np.load(GOLDEN / "frame_scope.npz")
    name, seed, B, H, text, frames, height, width, n, thr = next(c for c in mg.FRAME_CASES if c[0] == case)
    q64, k64 = mg.frame_inputs(seed, B, H, text, frames, height, width)
    q, k = torch.from_numpy(q64).float(), torch.from_numpy(k64).float()
    spatial = torch.from_numpy(d[f"{name}_spatial"].astype(np.int64))
    fm = kernels.frame_mask(q.to(cuda_device), k.to(cuda_device), spatial, text_len=text, frames=frames,
                            frame_len=height * width, threshold=thr, return_map=True)
    torch.cuda.synchronize()
    ref_map = ofs.frame_map(q, k, spatial.numpy(), text, frames, height * width)
    got_map = fm.map.cpu().numpy()
    assert np.abs(got_map - ref_map).max() <= 1e-6 * ref_map.max()
    assert ofs.margin(ref_map, thr) > 1e-4
    ref_mask = ofs.frame_select(ref_map, thr)
    assert np.array_equal(fm.mask.cpu().numpy().astype(bool), ref_mask)
    assert np.array_equal(ref_mask, d[f"{name}_mask"])
    assert np.array_equal(fm.bits.cpu().numpy().view(np.uint32), ofs.frame_bits(ref_mask))


def _random_frame_mask(B, H, F, seed, p=0.4):
    g = torch.Generator().manual_seed(seed)
    m = torch.rand(B, H, F, F, generator=g) < p
    m |= torch.eye(F, dtype=torch.bool)
    return m.numpy()


@pytest.mark.parametrize("bs", [128, 64])
def test_frame_csr_matches_oracle(cuda_device, bs):
    geo = VideoGeometry(226, 5, 12, 20)  # frames of 240 tokens, not block aligned
    B, H = 2, 3
    fmask = _random_frame_mask(B, H, geo.frames, seed=bs)
    bits = torch.from_numpy(ofs.frame_bits(fmask).view(np.int32)).to(cuda_device)
    fm = kernels.FrameMask(bits, None, None, geo.text_len, geo.frames, geo.frame_len)
    csr = kernels.frame_csr(fm, B, H, bs, bs)
    torch.cuda.synchronize()
    ref = ofs.frame_block_mask(fmask, geo.text_len, geo.frame_len, geo.seq_len, bs, bs)
    assert np.array_equal(csr.to_dense().cpu().numpy(), ref)
    rp_ref, ci_ref = osel.dense_to_csr(ref)
    rp = csr.row_ptr.cpu().numpy()
    assert np.array_equal(rp, rp_ref)
    ci = csr.col_idx.cpu().numpy()
    for g in range(B * H):
        assert np.array_equal(ci[rp[g, 0]:rp[g, -1]], ci_ref[rp_ref[g, 0]:rp_ref[g, -1]])


@pytest.mark.parametrize("bs,dtype", [(128, torch.bfloat16), (64, torch.bfloat16), (128, torch.float16)])
def test_attention_under_frame_masks(cuda_device, bs, dtype):
    geo = VideoGeometry(226, 5, 12, 20)
    B, H = 1, 3
    q, k, v = workloads.video_qkv(geo, B=B, H=H, dtype=dtype, seed=17)
    fmask = _random_frame_mask(B, H, geo.frames, seed=5)
    bits = torch.from_numpy(ofs.frame_bits(fmask).view(np.int32)).to(cuda_device)
    fm = kernels.FrameMask(bits, None, None, geo.text_len, geo.frames, geo.frame_len)
    csr = kernels.frame_csr(fm, B, H, bs, bs)
    out = kernels.bsa_fwd_frames(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), csr, fm, 0.125)
    torch.cuda.synchronize()
    ref = ofs.frame_attention_rows(q, k, v, fmask, geo.text_len, geo.frame_len, 0.125, range(B * H),
                                   range(geo.seq_len))
    got = out.float().cpu().numpy().reshape(B * H, geo.seq_len, 64)
    assert np.abs(got - ref).max() <= 2e-2


def test_forward_backup_cogvideox_shape(cuda_device):
    from sparseattnfunctions_b200.special_attentions.block_mask_attn import BlockSparseAttention

    geo = COGVIDEOX_2B
    q, k, v = workloads.video_qkv(geo, B=1, H=2, seed=23)
    spatial = torch.randint(0, geo.frame_len, (60,), generator=torch.Generator().manual_seed(3))
    proc = BlockSparseAttention(block_size=128, geometry=geo)
    out = proc.forward_backup(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), spatial=spatial)
    torch.cuda.synchronize()
    ref_map = ofs.frame_map(q, k, spatial.numpy(), geo.text_len, geo.frames, geo.frame_len)
    assert ofs.margin(ref_map) > 1e-4
    fmask = ofs.frame_select(ref_map)
    assert np.array_equal(proc.last_frame_mask.mask.cpu().numpy().astype(bool), fmask)
    rows = np.arange(0, geo.seq_len, 61)
    ref = ofs.frame_attention_rows(q, k, v, fmask, geo.text_len, geo.frame_len, 0.125, range(2), rows)
    got = out.float().cpu().numpy().reshape(2, geo.seq_len, 64)[:, rows]
    assert np.abs(got - ref).max() <= 2e-2


def test_mask_related_mirror_on_gpu(cuda_device):
    """special_attentions.utils.mask_related: the frame-scope mask through
    the mirror's reference-named function (golden case, injected sample), and
    calc_attn_block_sum_efficient = the block-size-weighted softmax numerator
    of the mean-pooled logits, rows normalised to 1 (fp64, 1e-12)."""
    from sparseattnfunctions_b200.special_attentions.utils import mask_related as mr

    d = np.load(GOLDEN / "frame_scope.npz")
    name, seed, B, H, text, frames, height, width, n, thr = mg.FRAME_CASES[0]
    q64, k64 = mg.frame_inputs(seed, B, H, text, frames, height, width)
    q, k = torch.from_numpy(q64).float().to(cuda_device), torch.from_numpy(k64).float().to(cuda_device)
    spatial = torch.from_numpy(d[f"{name}_spatial"].astype(np.int64))
    m = mr.generate_attention_mask_frame_scope(q, k, text_length=text, f=frames, width=width, height=height,
                                               sample_num=n, base_threshold=thr, spatial=spatial)
    assert np.array_equal(m.cpu().numpy(), d[f"{name}_mask"])

    g = torch.Generator().manual_seed(9)
    qq = torch.randn(1, 2, 1000, 64, generator=g).to(torch.bfloat16)
    kk = torch.randn(1, 2, 1000, 64, generator=g).to(torch.bfloat16)
    est = mr.calc_attn_block_sum_efficient(qq.to(cuda_device), kk.to(cuda_device), block_size=64).cpu().numpy()
    s = osel.pooled_scores(osel.block_means(qq, 64), osel.block_means(kk, 64)) / 8.0
    cols = np.full(16, 64.0)
    cols[-1] = 1000 - 15 * 64
    mass = cols * np.exp(s - s.max(-1, keepdims=True))
    np.testing.assert_allclose(est, mass / mass.sum(-1, keepdims=True), rtol=1e-12, atol=1e-15)
