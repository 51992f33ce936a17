"""Parity at the BASELINE configurations' own shapes (GPU against the CPU
oracle).

* Config 1: B1 H2 S2048 D64 fp32, 64-blocks, k = 8 with the diagonal forced
  inside the 8: selection bit-exact, attention within 1e-4 of the fp64
  oracle (every row), through both the library call and the drop-in
  ``block_sparse_triton_fn``.
* Config 2: B2 H30 S17776 D64 bf16, 128-blocks, top-14 + text dense:
  selection bit-exact, attention within 2e-2 on two whole heads (0 and 37)
  plus every 97th query row of all 60 heads.
* Config 5: B2 H30 S33976 (25 frames) bf16, 128-blocks (nb = 266), top-27 +
  text dense: selection bit-exact on all heads (oracle in head chunks),
  attention within 2e-2 on every 331st query row of all 60 heads.
* Config 3: ToMe on [2, 17550, 1920] bf16 hidden states, alternate split,
  r = 4000: pairings, node_max bits, counters and token maps bit-exact.
* Config 4 (per-head matching of MergeAttention / CombinedAttn): metric
  [60, 17550, 130] from ``tome_kv_metric`` (bit-exact against the oracle's
  metric), the reference split, r = 4000: bit-exact plan, checked in chunks
  of three rows.

The oracle's arg-max search takes fp64 BLAS scores; they are computed here
with fp64 matmuls on the GPU (every candidate within 1e-12 of a row's BLAS
maximum is then re-scored by the oracle's exact summation order).
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import selection as osel
from oracle import tome as otome
from sparseattnfunctions_b200 import kernels, workloads
from sparseattnfunctions_b200.geometry import COGVIDEOX_2B, COGVIDEOX_2B_LONG

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
FP32_TOL = 1e-4


def _max_err(out, ref):
    out = np.asarray(out, dtype=np.float64)
    nan_o, nan_r = np.isnan(out), np.isnan(ref)
    assert np.array_equal(nan_o, nan_r), "NaN rows differ from the oracle"
    return float(np.abs(out[~nan_r] - ref[~nan_r]).max()) if (~nan_r).any() else 0.0


def _check_selection(csr, mask_ref):
    mask = csr.mask.cpu().numpy().astype(bool)
    assert np.array_equal(mask, mask_ref), f"{(mask != mask_ref).sum()} mask bits differ"


# --------------------------------------------------------------------------- config 1

def test_config1_selection_and_attention(cuda_device):
    q, k, v = workloads.config1_qkv()
    dev = cuda_device
    csr = kernels.pool_topk(q.to(dev), k.to(dev), block_m=64, block_n=64, topk=8, force_diag=True,
                            forced_inside_topk=True, return_mask=True)
    mask_ref, _ = osel.select_blocks(q, k, 64, 64, 8, 0, 0, True, True)
    torch.cuda.synchronize()
    _check_selection(csr, mask_ref)
    assert mask_ref.sum(-1).min() == 8 and mask_ref.sum(-1).max() == 8
    assert all(mask_ref[0, h, i, i] for h in range(2) for i in range(32))
    scale = 1.0 / 8
    out = kernels.bsa_fwd(q.to(dev), k.to(dev), v.to(dev), csr, scale)
    torch.cuda.synchronize()
    ref = oatt.block_sparse_attention(q, k, v, mask_ref, scale, 64, 64)
    err = _max_err(out.cpu().numpy(), ref)
    assert err <= FP32_TOL, f"config 1 max abs error {err:.3e} > {FP32_TOL:.0e}"

    # the drop-in entry point with the dense 64-block mask (reference :293)
    from sparseattnfunctions_b200.special_attentions.utils.block_sparse_attn_kernel import \
        block_sparse_triton_fn

    out2 = block_sparse_triton_fn(q.to(dev), k.to(dev), v.to(dev), torch.from_numpy(mask_ref).to(dev), scale)
    torch.cuda.synchronize()
    err2 = _max_err(out2.cpu().numpy(), ref)
    assert err2 <= FP32_TOL, f"drop-in config 1 max abs error {err2:.3e}"


# --------------------------------------------------------------------------- config 2

def test_config2_selection_then_attention(cuda_device):
    geo = COGVIDEOX_2B
    dev = cuda_device
    q, k, v = workloads.video_qkv(geo, B=2, H=30)
    nb = geo.num_blocks(128)
    topk = math.ceil(0.10 * nb)
    tb = geo.text_blocks(128)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    csr = kernels.pool_topk(qd, kd, block_m=128, block_n=128, topk=topk, text_blocks_q=tb,
                            text_blocks_k=tb, return_mask=True)
    out = kernels.bsa_fwd(qd, kd, vd, csr, 0.125)
    torch.cuda.synchronize()
    mask_ref, _ = osel.select_blocks(q, k, 128, 128, topk, tb, tb)
    _check_selection(csr, mask_ref)
    out_np = out.float().cpu().numpy()
    # two whole heads
    for g in (0, 37):
        b, h = divmod(g, 30)
        ref = oatt.block_sparse_attention(q, k, v, mask_ref, 0.125, 128, 128, heads=[g])[b, h]
        err = _max_err(out_np[b, h], ref)
        assert err <= BF16_TOL, f"head {g}: max abs error {err:.3e}"
    # every 97th query row of every head
    rows = np.arange(0, geo.seq_len, 97)
    ref = oatt.block_sparse_attention_rows(q, k, v, mask_ref, 0.125, 128, 128, range(60), rows)
    got = out_np.reshape(60, geo.seq_len, 64)[:, rows]
    err = _max_err(got, ref)
    assert err <= BF16_TOL, f"sampled rows: max abs error {err:.3e}"


# --------------------------------------------------------------------------- config 5

def test_config5_selection_then_sampled_attention(cuda_device):
    geo = COGVIDEOX_2B_LONG
    dev = cuda_device
    q, k, v = workloads.video_qkv(geo, B=2, H=30, seed=777)
    nb = geo.num_blocks(128)
    assert nb == 266
    topk = math.ceil(0.10 * nb)
    tb = geo.text_blocks(128)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    csr = kernels.pool_topk(qd, kd, block_m=128, block_n=128, topk=topk, text_blocks_q=tb,
                            text_blocks_k=tb, return_mask=True)
    out = kernels.bsa_fwd(qd, kd, vd, csr, 0.125)
    torch.cuda.synchronize()
    mask = csr.mask.cpu().numpy().astype(bool)
    for b in range(2):
        for h0 in range(0, 30, 10):
            sl = (slice(b, b + 1), slice(h0, h0 + 10))
            ref, _ = osel.select_blocks(q[sl], k[sl], 128, 128, topk, tb, tb)
            assert np.array_equal(mask[sl], ref), f"batch {b} heads {h0}..{h0 + 9}: mask bits differ"
    rows = np.arange(0, geo.seq_len, 331)
    ref = oatt.block_sparse_attention_rows(q, k, v, mask, 0.125, 128, 128, range(60), rows)
    got = out.float().cpu().numpy().reshape(60, geo.seq_len, 64)[:, rows]
    err = _max_err(got, ref)
    assert err <= BF16_TOL, f"config 5 sampled rows: max abs error {err:.3e}"


# --------------------------------------------------------------------------- ToMe configs 3 and 4

def _gpu_scores(metric_dev, a_idx, b_idx):
    """fp64 cosine scores [B, Ns, Nd] on the GPU (cuBLAS DGEMM), as numpy."""
    x = metric_dev.double()
    a = x[:, a_idx.long()]
    b = x[:, b_idx.long()]
    na = a.square().sum(-1).sqrt()
    nb = b.square().sum(-1).sqrt()
    s = torch.bmm(a, b.transpose(1, 2)) / (na[:, :, None] * nb[:, None, :])
    return s.cpu().numpy()


def _compare_plan_rows(plan, m, rows, a, b, n):
    sl = slice(rows.start, rows.stop)
    assert np.array_equal(plan.node_idx[sl].cpu().numpy(), m["node_idx"])
    assert np.array_equal(plan.node_max[sl].cpu().numpy().view(np.uint64), m["node_max"].view(np.uint64))
    assert np.array_equal(plan.unm_idx[sl].cpu().numpy(), m["unm_idx"])
    assert np.array_equal(plan.src_idx[sl].cpu().numpy(), m["src_idx"])
    assert np.array_equal(plan.dst_idx[sl].cpu().numpy(), m["dst_idx"])
    assert np.array_equal(plan.counter[sl].cpu().numpy(), m["counter"])
    assert np.array_equal(plan.token_map[sl].cpu().numpy(), otome.token_map(a, b, m, n))


def test_config3_tome_match_full_size(cuda_device):
    from sparseattnfunctions_b200.special_attentions.utils import merge_unmerge as mu

    dev = cuda_device
    x = workloads.video_hidden(COGVIDEOX_2B, B=2, C=1920, seed=4321)
    xd = x.to(dev)
    a, b = mu.alternate_split(x.shape[1], dev)
    plan = kernels.tome_match(xd, a, b, 4000, keep_node=True)
    scores = _gpu_scores(xd, a, b)
    an, bn = a.cpu().numpy().astype(np.int64), b.cpu().numpy().astype(np.int64)
    m = otome.match(x, an, bn, 4000, scores=scores)
    torch.cuda.synchronize()
    _compare_plan_rows(plan, m, range(0, 2), an, bn, x.shape[1])
    assert int(plan.counter.sum()) == 2 * (bn.size + 4000)


def test_config4_per_head_metric_and_match(cuda_device):
    from sparseattnfunctions_b200.special_attentions.utils import merge_unmerge as mu

    dev = cuda_device
    geo = COGVIDEOX_2B
    _, k, v = workloads.video_qkv(geo, B=2, H=30, seed=99)
    metric = kernels.tome_kv_metric(k.to(dev), v.to(dev), geo.text_len)
    torch.cuda.synchronize()
    assert tuple(metric.shape) == (60, geo.video_len, 130)
    ref_metric = otome.kv_metric(k, v, geo.text_len)
    assert torch.equal(metric.cpu().view(torch.int16), ref_metric.view(torch.int16)), \
        "tome_kv_metric differs from the oracle's metric"
    a, b = mu.video_split(45, 30, 13, 3, 3, 4, dev)
    plan = kernels.tome_match(metric, a, b, 4000, keep_node=True)
    an, bn = a.cpu().numpy().astype(np.int64), b.cpu().numpy().astype(np.int64)
    assert (an.size, bn.size) == (15750, 1800)
    for r0 in range(0, 60, 3):
        rows = range(r0, r0 + 3)
        md = metric[r0:r0 + 3]
        scores = _gpu_scores(md, a, b)
        m = otome.match(md.cpu(), an, bn, 4000, scores=scores)
        _compare_plan_rows(plan, m, rows, an, bn, geo.video_len)
