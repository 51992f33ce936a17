"""GPU parity of CombinedAttn (ToMe merge -> block selection on the merged
sequence -> block-sparse attention with the log(size) bias -> unmerge)
against the CPU oracle composition.

Bit-exact: the merge pairing (oracle/tome.py match) and the block list chosen
on the merged q / k (oracle/selection.py).  Output: 2e-2 max-abs (bf16).
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import selection as osel
from oracle import tome as otome
from sparseattnfunctions_b200.geometry import VideoGeometry
from sparseattnfunctions_b200.special_attentions.block_mask_attn import BlockSparseAttention
from sparseattnfunctions_b200.special_attentions.combined_attn import CombinedAttn

pytestmark = pytest.mark.gpu

GEOM = VideoGeometry(26, 5, 10, 15)
CFG = dict(w=15, h=10, t=5, sx=3, sy=2, st=2, r=200)


def _qkv(B, H, S, D, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, S, D, generator=g).to(torch.bfloat16) for _ in range(3)]


def _oracle_combined(q, k, v, plan, csr_mask, block, full_merge, text):
    B, H, S, D = q.shape
    N = S - text
    a, b = plan.a_idx.cpu().numpy(), plan.b_idx.cpu().numpy()
    metric = otome.kv_metric(k, v, text)
    m = otome.match(metric, a, b, CFG["r"])
    assert np.array_equal(plan.src_idx.cpu().numpy(), m["src_idx"])
    assert np.array_equal(plan.dst_idx.cpu().numpy(), m["dst_idx"])
    assert np.array_equal(plan.unm_idx.cpu().numpy(), m["unm_idx"])

    def omerge(x):
        x3 = x.reshape(B * H, S, D)
        return np.concatenate([x3[:, :text].double().numpy(), otome.merge(x3[:, text:], a, b, m)], axis=1)

    bias = otome.proportional_bias(m["counter"], text, a.size - CFG["r"])
    mk, mv = omerge(k), omerge(v)
    L = mk.shape[1]
    if full_merge:
        mq = omerge(q)
        o = oatt.block_sparse_attention(mq.reshape(B, H, L, D), mk.reshape(B, H, L, D), mv.reshape(B, H, L, D),
                                        csr_mask, 1 / math.sqrt(D), block, block, kv_bias=bias)
        o = o.reshape(B * H, L, D)
        o = np.concatenate([o[:, :text], otome.unmerge(o[:, text:], a, b, m, N)], axis=1)
        return o.reshape(B, H, S, D)
    return oatt.block_sparse_attention(q, mk.reshape(B, H, L, D), mv.reshape(B, H, L, D), csr_mask,
                                       1 / math.sqrt(D), block, block, kv_bias=bias)


@pytest.mark.parametrize("block,full_merge", [(64, True), (128, True), (64, False)])
def test_combined_against_oracle(cuda_device, block, full_merge):
    B, H, D = 1, 2, 64
    S = GEOM.seq_len
    q, k, v = _qkv(B, H, S, D, seed=block + full_merge)
    attn = CombinedAttn(layer_num=1, merge_config=CFG, density=0.3, block_size=block,
                        full_merge=full_merge, geometry=GEOM)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    out = attn(qd, kd, vd)
    torch.cuda.synchronize()
    st = attn._layers[0]
    plan = st.merge_fn.plan
    csr = attn.last_csr
    # block list: bit-exact against the oracle's selection on the same merged q / k
    mk = st.merge_fn(kd).view(B, H, -1, D)
    mq = st.merge_fn(qd).view(B, H, -1, D) if full_merge else qd
    nbk = math.ceil(mk.shape[2] / block)
    ref_mask, _ = osel.select_blocks(mq.cpu(), mk.cpu(), block, block, max(1, math.ceil(0.3 * nbk)),
                                     math.ceil(GEOM.text_len / block), math.ceil(GEOM.text_len / block))
    assert np.array_equal(csr.to_dense().cpu().numpy(), ref_mask)
    ref = _oracle_combined(q, k, v, plan, ref_mask, block, full_merge, GEOM.text_len)
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err <= 2e-2, err
    assert out.shape == q.shape


def test_combined_warmup_uses_block_sparse(cuda_device):
    B, H, D = 1, 2, 64
    q, k, v = (t.to(cuda_device) for t in _qkv(B, H, GEOM.seq_len, D, seed=3))
    attn = CombinedAttn(warmup_epoch=1, layer_num=2, merge_config=CFG, density=0.3, block_size=64,
                        geometry=GEOM)
    plain = BlockSparseAttention(block_size=64, density=0.3, geometry=GEOM)
    want = plain(q, k, v)
    for _ in range(2):  # one warm-up pass over both layers
        assert torch.equal(attn(q, k, v), want)
    merged = attn(q, k, v)  # first merged step of layer 0
    assert attn._layers[0].merge_fn is not None and attn._layers[1].merge_fn is None
    assert not torch.equal(merged, want)


def test_combined_rejects_rearranger(cuda_device):
    q = torch.zeros(1, 1, GEOM.seq_len, 64, dtype=torch.bfloat16, device=cuda_device)
    attn = CombinedAttn(layer_num=1, merge_config=CFG, geometry=GEOM)
    with pytest.raises(NotImplementedError):
        attn(q, q, q, use_rearranger=True)
