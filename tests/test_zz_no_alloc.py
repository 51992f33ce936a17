"""Scratch-free block selection (saf_pool_topk_noalloc) against the regular
entry point.

saf_pool_topk_noalloc serves callers that cannot allocate device memory when
they call in -- for example a process whose GPU memory is planned once and
then frozen, or a plugin slot that only receives its input and output
buffers.  It takes its scratch from a static device array instead of a
caller workspace.  These tests call it through the C ABI and require the
same block lists, masks and scores as saf_pool_topk (which the rest of the
suite checks against the CPU oracle) on two calls in a row, the second
running over the scratch the first one left behind.

This file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from sparseattnfunctions_b200 import _lib, kernels, workloads
from sparseattnfunctions_b200.geometry import VideoGeometry


def _t4(x):
    t = _lib.Tensor4()
    t.data = x.data_ptr()
    t.dtype = {torch.bfloat16: _lib.SAF_BF16, torch.float16: _lib.SAF_F16,
               torch.float32: _lib.SAF_F32}[x.dtype]
    t.B, t.H, t.S, t.D = x.shape
    t.stride_b, t.stride_h, t.stride_s = x.stride(0), x.stride(1), x.stride(2)
    return t


def _noalloc(q, k, bm, bn, topk, tq, tk):
    B, H, Sq, _ = q.shape
    nbq, nbk = -(-Sq // bm), -(-k.shape[2] // bn)
    row_ptr = torch.full((B * H, nbq + 1), -1, dtype=torch.int32, device=q.device)
    col_idx = torch.full((B * H * nbq * nbk,), -1, dtype=torch.int32, device=q.device)
    mask = torch.full((B, H, nbq, nbk), 7, dtype=torch.uint8, device=q.device)
    scores = torch.full((B, H, nbq, nbk), float("nan"), dtype=torch.float64, device=q.device)
    cfg = _lib.SelectCfg(bm, bn, topk, tq, tk, 0, 0, 0)
    tq4, tk4 = _t4(q), _t4(k)
    rc = _lib.load().saf_pool_topk_noalloc(
        ctypes.byref(tq4), ctypes.byref(tk4), ctypes.byref(cfg), row_ptr.data_ptr(),
        col_idx.data_ptr(), mask.data_ptr(), scores.data_ptr(),
        torch.cuda.current_stream(q.device).cuda_stream)
    _lib.check("saf_pool_topk_noalloc", rc)
    return row_ptr, col_idx, mask, scores


def _same(dev, q, k, bm, bn, topk, tq, tk):
    q, k = q.to(dev), k.to(dev)
    ref = kernels.pool_topk(q, k, block_m=bm, block_n=bn, topk=topk, text_blocks_q=tq,
                            text_blocks_k=tk, return_mask=True, return_scores=True)
    rp, ci, mask, scores = _noalloc(q, k, bm, bn, topk, tq, tk)
    torch.cuda.synchronize()
    assert torch.equal(rp, ref.row_ptr)
    assert torch.equal(mask, ref.mask)
    assert np.array_equal(scores.cpu().numpy().view(np.uint64), ref.scores.cpu().numpy().view(np.uint64))
    rp_h, ci_h, ci_ref = rp.cpu().numpy(), ci.cpu().numpy(), ref.col_idx.cpu().numpy()
    for g in range(rp_h.shape[0]):
        s, e = rp_h[g, 0], rp_h[g, -1]
        assert np.array_equal(ci_h[s:e], ci_ref[s:e])


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    # call 1: a video-shaped problem with dense text blocks
    geo = VideoGeometry(226, 5, 30, 45)  # 6976 tokens
    q, k, _ = workloads.video_qkv(geo, B=2, H=4, seed=91)
    _same(cuda_device, q, k, 128, 128, 6, 2, 2)
    # call 2, right after, on different sizes: the static scratch still holds
    # call 1's data and must not leak into the result
    g = torch.Generator().manual_seed(92)
    q2 = torch.randn(1, 3, 1500, 64, generator=g).to(torch.bfloat16)
    k2 = torch.randn(1, 3, 2100, 64, generator=g).to(torch.bfloat16)
    _same(cuda_device, q2, k2, 64, 64, 5, 1, 1)
    assert _lib.read_device_status(0, clear=True) == 0


@pytest.mark.gpu
def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    # config-5 sized selection needs ~33 MB of scratch, above the 16 MiB array
    q = torch.empty(2, 30, 33976, 64, dtype=torch.bfloat16, device=cuda_device)
    cfg = _lib.SelectCfg(128, 128, 27, 2, 2, 0, 0, 0)
    t = _t4(q)
    need = _lib.load().saf_pool_topk_workspace_bytes(ctypes.byref(t), ctypes.byref(t), ctypes.byref(cfg))
    assert need > (16 << 20)
    rc = _lib.load().saf_pool_topk_noalloc(ctypes.byref(t), ctypes.byref(t), ctypes.byref(cfg),
                                           q.data_ptr(), q.data_ptr(), None, None, None)
    assert rc == _lib.SAF_ERR_WORKSPACE
