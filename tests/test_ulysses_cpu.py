"""Sequence-parallel (Ulysses) exchange logic on CPU: two gloo ranks, host
pack / unpack (oracle/ulysses.py) and an fp64 dense attention as the inner
processor.  The gathered sequence-sharded outputs must equal single-process
attention over the whole sequence, for equal and uneven shards and an uneven
head split (5 heads -> 3 + 2)."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ulysses as oul

B, H, D = 2, 5, 16


def _inputs(S, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, S, H, D, generator=g, dtype=torch.float64) for _ in range(3)]


def _dense(q, k, v, out):
    """[B, h, S, D] views -> out (fp64 softmax(q k^T / sqrt(D)) v)."""
    s = torch.einsum("bhqd,bhkd->bhqk", q, k) / math.sqrt(q.shape[-1])
    out.copy_(torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, dim=-1), v))
    return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, lens, chunks, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from sparseattnfunctions_b200.ulysses import UlyssesAttention

        q, k, v = _inputs(sum(lens))
        at = sum(lens[:rank])
        shard = [t[:, at:at + lens[rank]].contiguous() for t in (q, k, v)]
        ua = UlyssesAttention(_dense, heads=H, seq_lens=lens, pack=oul.pack, unpack=oul.unpack, chunks=chunks)
        out = ua(*shard)
        result_q.put((rank, out.numpy(), ua.local_heads))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("lens,chunks", [([24, 24], 1), ([17, 31], 2), ([24, 24], 3)])
def test_ulysses_two_gloo_ranks(lens, chunks):
    """Single exchange (chunks = 1) and the head-chunked pipeline."""
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, lens, chunks, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        rank, out, h = result_q.get(timeout=120)
        got[rank] = (out, h)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0][1] == 3 and got[1][1] == 2
    q, k, v = _inputs(sum(lens))
    full = torch.empty(B, H, sum(lens), D, dtype=torch.float64)
    _dense(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), full)
    want = full.transpose(1, 2).numpy()
    have = np.concatenate([got[0][0], got[1][0]], axis=1)
    np.testing.assert_allclose(have, want, rtol=0, atol=1e-12)


def test_pack_unpack_roundtrip_and_layout():
    from sparseattnfunctions_b200.kernels import head_split

    g = torch.Generator().manual_seed(3)
    ts = [torch.randn(2, 7, 30, 8, generator=g) for _ in range(3)]
    off = head_split(30, 8)
    assert off == [0, 4, 8, 12, 16, 20, 24, 27, 30]
    assert head_split(30, 4) == [0, 8, 16, 23, 30] and head_split(30, 2) == [0, 15, 30]
    buf = oul.pack(ts, off)
    # chunk 6 (heads 24..26) of tensor 1, row s=5, batch 1, head 25
    at = sum(7 * 2 * 3 * (off[j + 1] - off[j]) * 8 for j in range(6))
    chunk = buf[at:at + 7 * 2 * 3 * 3 * 8].view(7, 2, 3, 3, 8)
    assert torch.equal(chunk[5, 1, 1, 1], ts[1][1, 5, 25])
    outs = [torch.zeros_like(t) for t in ts]
    oul.unpack(buf, outs, off)
    assert all(torch.equal(a, b) for a, b in zip(outs, ts))


def test_chunk_plan_keeps_each_ranks_head_count():
    from sparseattnfunctions_b200.kernels import head_split
    from sparseattnfunctions_b200.ulysses import chunk_plan

    for H, P, C in ((30, 8, 2), (30, 2, 2), (5, 2, 3), (30, 4, 4), (3, 8, 2)):
        plan = chunk_plan(H, P, C)
        off = head_split(H, P)
        per_rank = [0] * P
        c_prev = 0
        for c0, offs in plan:
            assert c0 == c_prev and offs[0] == 0 and offs[-1] > 0
            c_prev = c0 + offs[-1]
            for j in range(P):
                per_rank[j] += offs[j + 1] - offs[j]
        assert c_prev == H
        assert per_rank == [off[j + 1] - off[j] for j in range(P)]
    assert chunk_plan(30, 2, 2) == [(0, [0, 8, 16]), (16, [0, 7, 14])]
