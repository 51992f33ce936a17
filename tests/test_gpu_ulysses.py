"""GPU checks of the Ulysses layout kernels (saf_ulysses_pack / unpack) against
the host restatement (oracle/ulysses.py), bit-exact, and of the
sequence-parallel attention exchange emulated for P ranks on one GPU."""
import math

import pytest
import torch

from oracle import ulysses as oul
from sparseattnfunctions_b200 import kernels
from sparseattnfunctions_b200.geometry import VideoGeometry
from sparseattnfunctions_b200.special_attentions.block_mask_attn import BlockSparseAttention
from sparseattnfunctions_b200.ulysses import UlyssesAttention

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("P", [1, 2, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_pack_unpack_match_host(cuda_device, P, dtype):
    g = torch.Generator().manual_seed(P)
    B, s, H, D = 2, 37, 30, 64
    proj = torch.randn(B, s, 3, H, D, generator=g).to(dtype)  # a q/k/v projection of a shard
    ts = [proj[:, :, t] for t in range(3)]                    # strided [B, s, H, D] views
    off = kernels.head_split(H, P)
    want = oul.pack(ts, off)
    pd = proj.to(cuda_device)
    got = kernels.ulysses_pack([pd[:, :, i] for i in range(3)], off)
    assert torch.equal(got.cpu(), want)
    outs = [torch.zeros(B, s, H, D, dtype=dtype, device=cuda_device) for _ in range(3)]
    kernels.ulysses_unpack(got, outs, off)
    for o, t in zip(outs, ts):
        assert torch.equal(o.cpu(), t)


def test_pack_rejects_misaligned_rows(cuda_device):
    x = torch.zeros(1, 4, 2, 60, dtype=torch.bfloat16, device=cuda_device)  # 120-byte rows
    with pytest.raises(ValueError):
        kernels.ulysses_pack([x], [0, 2])


GEOM = VideoGeometry(26, 4, 10, 15)  # S = 626


def _full_inputs(dev, H=5, D=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(2, GEOM.seq_len, H, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(3)]


def test_single_rank_matches_plain_processor(cuda_device):
    q, k, v = _full_inputs(cuda_device)
    inner = BlockSparseAttention(block_size=64, density=0.3, geometry=GEOM)
    ua = UlyssesAttention(inner, heads=5)
    out = ua(q, k, v)
    want = inner(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
    assert torch.equal(out, want)


@pytest.mark.parametrize("P", [2, 4])
def test_emulated_ranks_match_plain_processor(cuda_device, P):
    """P ranks emulated on one GPU: pack every shard, route chunk j of every
    sender to rank j (the all-to-all), attention on the strided head views,
    route the output rows back, unpack."""
    H, D = 5, 64
    q, k, v = _full_inputs(cuda_device, H, D, seed=P)
    S = q.shape[1]
    lens = [S // P + (1 if r < S % P else 0) for r in range(P)]
    starts = [sum(lens[:r]) for r in range(P)]
    off = kernels.head_split(H, P)
    hs = [off[j + 1] - off[j] for j in range(P)]
    inner = BlockSparseAttention(block_size=64, density=0.3, geometry=GEOM)
    sends = [kernels.ulysses_pack([t[:, starts[r]:starts[r] + lens[r]] for t in (q, k, v)], off)
             for r in range(P)]

    def chunk(buf, sizes, j):
        a = sum(sizes[:j])
        return buf[a:a + sizes[j]]

    rows = []
    for r in range(P):
        recv = torch.cat([chunk(sends[i], [lens[i] * 2 * 3 * hj * D for hj in hs], r) for i in range(P)])
        grid = recv.view(S, 2, 3, hs[r], D)
        qh, kh, vh = (grid[:, :, t].permute(1, 2, 0, 3) for t in range(3))
        o_rows = torch.empty(S, 2, hs[r], D, dtype=q.dtype, device=cuda_device)
        inner(qh, kh, vh, out=o_rows.permute(1, 2, 0, 3))
        rows.append(o_rows.view(-1))
    want = inner(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
    for r in range(P):
        back = torch.cat([chunk(rows[j], [n * 2 * hs[j] * D for n in lens], r) for j in range(P)])
        out = torch.empty(2, lens[r], H, D, dtype=q.dtype, device=cuda_device)
        kernels.ulysses_unpack(back, [out], off)
        assert torch.equal(out, want[:, starts[r]:starts[r] + lens[r]])


@pytest.mark.parametrize("P,chunks", [(2, 3), (4, 2)])
def test_emulated_chunked_exchange_matches_plain_processor(cuda_device, P, chunks):
    """The head-chunked exchange of UlyssesAttention emulated for P ranks on
    one GPU: per chunk, pack the head-slice views of every shard, route the
    chunks, attention on the strided views, route the rows back and unpack
    into the head-slice view of each rank's output."""
    from sparseattnfunctions_b200.ulysses import chunk_plan

    H, D = 5, 64
    q, k, v = _full_inputs(cuda_device, H, D, seed=10 + P)
    S = q.shape[1]
    lens = [S // P + (1 if r < S % P else 0) for r in range(P)]
    starts = [sum(lens[:r]) for r in range(P)]
    inner = BlockSparseAttention(block_size=64, density=0.3, geometry=GEOM)
    want = inner(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
    outs = [torch.empty(2, lens[r], H, D, dtype=q.dtype, device=cuda_device) for r in range(P)]

    def chunk(buf, sizes, j):
        a = sum(sizes[:j])
        return buf[a:a + sizes[j]]

    for c0, offs in chunk_plan(H, P, chunks):
        hc = offs[-1]
        hs = [offs[j + 1] - offs[j] for j in range(P)]
        sends = [kernels.ulysses_pack([t[:, starts[r]:starts[r] + lens[r], c0:c0 + hc] for t in (q, k, v)], offs)
                 for r in range(P)]
        rows = []
        for r in range(P):
            recv = torch.cat([chunk(sends[i], [lens[i] * 2 * 3 * hj * D for hj in hs], r) for i in range(P)])
            o_rows = torch.empty(S, 2, hs[r], D, dtype=q.dtype, device=cuda_device)
            if hs[r] > 0:
                grid = recv.view(S, 2, 3, hs[r], D)
                qh, kh, vh = (grid[:, :, t].permute(1, 2, 0, 3) for t in range(3))
                inner(qh, kh, vh, out=o_rows.permute(1, 2, 0, 3))
            rows.append(o_rows.view(-1))
        for r in range(P):
            back = torch.cat([chunk(rows[j], [n * 2 * hs[j] * D for n in lens], r) for j in range(P)])
            kernels.ulysses_unpack(back, [outs[r][:, :, c0:c0 + hc]], offs)
    for r in range(P):
        ref = want[:, starts[r]:starts[r] + lens[r]]
        assert torch.equal(outs[r].isnan(), ref.isnan())
        assert float((outs[r].float() - ref.float()).nan_to_num().abs().max()) <= 2e-2
