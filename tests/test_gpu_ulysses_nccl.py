"""Sequence-parallel attention across two GPUs with NCCL: every rank's output
shard of ``UlyssesAttention`` (single exchange and the head-chunked pipeline)
equals the single-GPU processor's rows -- within the fp32 merge rounding of
the dense text rows, whose key blocks the attention kernel splits over more
work items when a GPU holds fewer heads, and bit for bit below them.  Needs
two GPUs; skipped otherwise (the exchange logic itself is covered on CPU with
gloo ranks)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

H, D = 6, 64


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from sparseattnfunctions_b200 import workloads
        from sparseattnfunctions_b200.geometry import VideoGeometry
        from sparseattnfunctions_b200.special_attentions.block_mask_attn import BlockSparseAttention
        from sparseattnfunctions_b200.ulysses import UlyssesAttention

        geo = VideoGeometry(frames=3, height=16, width=24, text_len=40)
        dev = torch.device("cuda", rank)
        q, k, v = (t.transpose(1, 2).contiguous().to(dev) for t in
                   workloads.video_qkv(geo, B=2, H=H, D=D, dtype=torch.bfloat16, seed=9))
        S = q.shape[1]
        lens = [S // world + (1 if r < S % world else 0) for r in range(world)]
        at = sum(lens[:rank])
        shard = [t[:, at:at + lens[rank]].contiguous() for t in (q, k, v)]
        inner = BlockSparseAttention(block_size=128, density=0.3, geometry=geo)
        outs = {}
        for chunks in (1, 3):
            ua = UlyssesAttention(inner, heads=H, seq_lens=lens, chunks=chunks)
            outs[chunks] = ua(*shard).cpu()
        torch.cuda.synchronize()
        dist.barrier()
        want = None
        if rank == 0:  # the single-GPU processor over the whole sequence
            want = inner(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2).cpu()
        result_q.put((rank, at, outs, want))
    finally:
        dist.destroy_process_group()


def test_two_ranks_match_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        rank, at, outs, want = result_q.get(timeout=300)
        got[rank] = (at, outs, want)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    want = got[0][2]
    text_tiles = 128  # the lead (dense text) tile of 128 query rows
    for rank in (0, 1):
        at, outs, _ = got[rank]
        for chunks, out in outs.items():
            ref = want[:, at:at + out.shape[1]]
            assert torch.equal(out.isnan(), ref.isnan()), (rank, chunks)
            diff = (out.float() - ref.float()).nan_to_num().abs().max().item()
            assert diff <= 2e-2, (rank, chunks, diff)
            below = max(0, text_tiles - at)
            assert torch.equal(out[:, below:], ref[:, below:]), (rank, chunks)
