"""GPU ToMe matching / merge / unmerge against the CPU oracle (oracle/tome.py,
itself pinned to the reference's merge_unmerge.py by tests/golden).

Matching is bit-exact: the same merged / kept src tokens in the same order,
the same dst for every merged src, the same counters and the same fp64
node_max.  Merge outputs are within 2e-2 (bf16), unmerge is an exact gather.
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import tome as otome
from sparseattnfunctions_b200 import kernels
from sparseattnfunctions_b200.special_attentions.utils import merge_unmerge as mu

pytestmark = pytest.mark.gpu


def _metric(B, N, C, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, N, C, generator=g).to(dtype)


def _check_plan(plan, metric, a_idx, b_idx, r):
    a = a_idx.cpu().numpy().astype(np.int64)
    b = b_idx.cpu().numpy().astype(np.int64)
    m = otome.match(metric, a, b, r)
    torch.cuda.synchronize()
    assert np.array_equal(plan.node_idx.cpu().numpy(), m["node_idx"])
    assert np.array_equal(plan.node_max.cpu().numpy().view(np.uint64), m["node_max"].view(np.uint64))
    assert np.array_equal(plan.unm_idx.cpu().numpy(), m["unm_idx"])
    assert np.array_equal(plan.src_idx.cpu().numpy(), m["src_idx"])
    assert np.array_equal(plan.dst_idx.cpu().numpy(), m["dst_idx"])
    assert np.array_equal(plan.counter.cpu().numpy(), m["counter"])
    assert np.array_equal(plan.token_map.cpu().numpy(), otome.token_map(a, b, m, metric.shape[1]))
    np.testing.assert_allclose(plan.log_count.cpu().numpy(), np.log(m["counter"]), rtol=1e-6)
    return m


@pytest.mark.parametrize("r", [4000, 9000])
def test_match_reference_split(cuda_device, r):
    """The reference's CogVideoX-2B split (first frame + one per 4x3x3 cell)."""
    metric = _metric(2, 17550, 16, seed=r)
    a, b = mu.video_split(45, 30, 13, 3, 3, 4, cuda_device)
    plan = kernels.tome_match(metric.to(cuda_device), a, b, r, keep_node=True)
    _check_plan(plan, metric, a, b, r)


def test_match_alternate_split_wide(cuda_device):
    """BASELINE config-3 split (src even, dst odd) with wide hidden states."""
    metric = _metric(1, 4000, 1920, seed=3)
    a, b = mu.alternate_split(4000, cuda_device)
    plan = kernels.tome_match(metric.to(cuda_device), a, b, 900, keep_node=True)
    _check_plan(plan, metric, a, b, 900)


@pytest.mark.parametrize("N,C,r", [(1000, 130, 200), (777, 72, 10000), (300, 8, 1), (5000, 200, 2400)])
def test_match_ragged_sizes(cuda_device, N, C, r):
    metric = _metric(3, N, C, seed=N + C)
    a, b = mu.alternate_split(N, cuda_device)
    plan = kernels.tome_match(metric.to(cuda_device), a, b, r, keep_node=True)
    _check_plan(plan, metric, a, b, min(r, a.numel()))


def test_match_f16(cuda_device):
    metric = _metric(2, 2000, 64, seed=9, dtype=torch.float16)
    a, b = mu.alternate_split(2000, cuda_device)
    plan = kernels.tome_match(metric.to(cuda_device), a, b, 600, keep_node=True)
    _check_plan(plan, metric, a, b, 600)


def test_match_near_ties_use_exact_scan(cuda_device):
    """Duplicated dst rows give exactly tied best candidates: the lower dst
    position must win, and rows whose 8 candidates are within the error band
    take the exact full scan."""
    g = torch.Generator().manual_seed(5)
    base = torch.randn(1, 100, 32, generator=g)
    metric = torch.empty(1, 2000, 32)
    metric[:, 0::2] = torch.randn(1, 1000, 32, generator=g)
    metric[:, 1::2] = base.repeat(1, 10, 1)  # every dst row appears 10 times
    metric = metric.to(torch.bfloat16)
    a, b = mu.alternate_split(2000, cuda_device)
    plan = kernels.tome_match(metric.to(cuda_device), a, b, 500, keep_node=True)
    _check_plan(plan, metric, a, b, 500)
    assert int(plan.node_idx.max()) < 100  # ties resolved to the first copy


@pytest.mark.parametrize("text", [0, 226])
def test_merge_unmerge(cuda_device, text):
    N, C, r = 17550, 64, 4000
    metric = _metric(2, N, 16, seed=7)
    a, b = mu.video_split(45, 30, 13, 3, 3, 4, cuda_device)
    plan = kernels.tome_match(metric.to(cuda_device), a, b, r)
    m = otome.match(metric, a.cpu().numpy(), b.cpu().numpy(), r)
    g = torch.Generator().manual_seed(8)
    x = torch.randn(2, text + N, C, generator=g).to(torch.bfloat16)
    merged = kernels.tome_merge(x.to(cuda_device), plan, text_len=text)
    ref_video = otome.merge(x[:, text:], a.cpu().numpy(), b.cpu().numpy(), m)
    ref = np.concatenate([x[:, :text].double().numpy(), ref_video], axis=1)
    got = merged.double().cpu().numpy()
    unm = text + (a.numel() - r)
    assert np.array_equal(got[:, :unm], ref[:, :unm])  # copies are exact
    assert np.abs(got - ref).max() <= 2e-2
    y = torch.randn(2, text + plan.merged_len, C, generator=g).to(torch.bfloat16)
    un = kernels.tome_unmerge(y.to(cuda_device), plan, text_len=text).cpu()
    ref_un = otome.unmerge(y[:, text:], a.cpu().numpy(), b.cpu().numpy(), m, N)
    assert torch.equal(un[:, :text], y[:, :text])
    assert np.array_equal(un[:, text:].double().numpy(), ref_un)


def test_bipartite_closures_4d_roundtrip(cuda_device):
    """The reference's 4-D MergeAttention layout: [b, h, text + N, D] with the
    matching per (b, h); merge keeps the text in front, unmerge restores
    the 4-D shape (merge_unmerge.py:119-154)."""
    Bh, H, N, D, text = 1, 2, 17550, 64, 226
    metric = _metric(Bh * H, N, 16, seed=11)
    merge, unmerge = mu.bipartite_soft_matching_video(metric.to(cuda_device), 45, 30, 13, 3, 3, 4,
                                                      4000, no_rand=True)
    g = torch.Generator().manual_seed(12)
    x = torch.randn(Bh, H, text + N, D, generator=g).to(torch.bfloat16).to(cuda_device)
    y = merge(x)
    assert y.shape == (Bh * H, text + N - 4000, D)
    back = unmerge(y)
    assert back.shape == x.shape
    # tokens that were kept or are dst come back unchanged
    plan = merge.plan
    keep = torch.ones(N, dtype=torch.bool)
    src_tok = plan.a_idx.cpu()[plan.src_idx.cpu().long()]
    for h in range(Bh * H):
        kept = keep.clone()
        kept[src_tok[h].long()] = False
        kept[plan.b_idx.cpu().long()] = False
        xb = x.reshape(Bh * H, text + N, D)[h].cpu()
        bb = back.reshape(Bh * H, text + N, D)[h].cpu()
        assert torch.equal(bb[:text], xb[:text])
        assert torch.equal(bb[text:][kept], xb[text:][kept])
    assert mu.counter.shape == (Bh * H, plan.Nd, 1)


@pytest.mark.parametrize("full_merge", [False, True])
def test_merge_attention_against_oracle(cuda_device, full_merge):
    from sparseattnfunctions_b200.special_attentions.MergeAttention import MergeAttention

    cfg = dict(w=15, h=10, t=5, sx=3, sy=2, st=2, r=200)
    B, H, D, text = 1, 2, 64, 26
    N = cfg["w"] * cfg["h"] * cfg["t"]
    g = torch.Generator().manual_seed(21)
    q, k, v = (torch.randn(B, H, text + N, D, generator=g).to(torch.bfloat16) for _ in range(3))
    attn = MergeAttention(merge_config=cfg, full_merge=full_merge)
    attn.generator = torch.Generator(device=cuda_device).manual_seed(3)
    out = attn(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)).float().cpu()
    plan = attn.merge_fn.plan
    # oracle composition on the same metric and split
    metric = otome.kv_metric(k, v, text)
    a, b = plan.a_idx.cpu().numpy(), plan.b_idx.cpu().numpy()
    m = otome.match(metric, a, b, cfg["r"])
    def omerge(x):
        x3 = x.reshape(B * H, text + N, D)
        return np.concatenate([x3[:, :text].double().numpy(), otome.merge(x3[:, text:], a, b, m)], axis=1)
    bias = otome.proportional_bias(m["counter"], text, a.size - cfg["r"])
    mk, mv = omerge(k), omerge(v)
    L = mk.shape[1]
    if full_merge:
        mq = omerge(q)
        ref_m = oatt.block_sparse_attention(mq.reshape(B, H, L, D), mk.reshape(B, H, L, D),
                                            mv.reshape(B, H, L, D),
                                            np.ones((B, H, math.ceil(L / 128), math.ceil(L / 128)), bool),
                                            1 / 8, 128, 128, kv_bias=bias)
        ref_m = ref_m.reshape(B * H, L, D)
        ref = np.concatenate([ref_m[:, :text], otome.unmerge(ref_m[:, text:], a, b, m, N)], axis=1)
        ref = ref.reshape(B, H, text + N, D)
    else:
        ref = oatt.block_sparse_attention(q, mk.reshape(B, H, L, D), mv.reshape(B, H, L, D),
                                          np.ones((B, H, math.ceil((text + N) / 128), math.ceil(L / 128)), bool),
                                          1 / 8, 128, 128, kv_bias=bias)
    err = np.abs(out.numpy() - ref).max()
    assert err <= 2e-2, err


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_kv_metric_bit_exact(cuda_device, dtype):
    g = torch.Generator().manual_seed(31)
    base = torch.randn(2, 300, 3, 64, generator=g).to(dtype)
    k = base.transpose(1, 2)                                            # strided [B, H, S, D]
    v = (torch.randn(2, 3, 300, 64, generator=g) * 3).to(dtype)
    got = kernels.tome_kv_metric(k.to(cuda_device), v.to(cuda_device), 26).cpu()
    want = otome.kv_metric(k, v, 26)
    assert got.shape == (6, 274, 130)
    assert torch.equal(got, want)
