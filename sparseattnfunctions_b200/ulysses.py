"""Sequence-parallel attention across GPUs (Ulysses all-to-all).

For the long-video configuration (S = 33976) the transformer blocks around
attention run sequence-sharded: every rank holds ``[B, s, H, D]`` rows of
q / k / v.  Attention needs whole sequences, so ``UlyssesAttention``

1. packs the rank's q, k, v into one send buffer, chunk j = the heads of rank
   j as ``[s, B, 3, h_j, D]`` (``saf_ulysses_pack``);
2. exchanges the chunks with one NCCL all-to-all (``all_to_all_single`` with
   uneven splits; heads split contiguously, 4,4,4,4,4,4,3,3 for 30 heads on 8
   ranks) -- the receive buffer is ``[S, B, 3, h, D]``, and q, k, v of the
   rank's heads are strided ``[B, h, S, D]`` views of it that the selection
   and attention kernels read in place;
3. runs the inner processor (block selection + block-sparse attention) on the
   rank's heads, writing the output straight into the ``[S, B, h, D]``
   return buffer;
4. exchanges the output rows back (second all-to-all) and unpacks them into
   ``[B, s, H, D]`` (``saf_ulysses_unpack``).

Every (b, h) is independent in selection and attention, so the only data
movement is the two all-to-alls; when the input is not sequence-sharded,
heads are simply partitioned with no collective.  On one rank there is no
exchange and no pack: the kernels read ``[B, S, H, D]`` in place as strided
``[B, H, S, D]`` views and write the output rows in place.  The reference
itself is single-GPU.

With ``chunks`` > 1 the heads go in chunks that pipeline: chunk c holds
heads [C_c, C_c+1) split over the ranks (every rank keeps its head count of
the contiguous split), and while the selection and attention of chunk c run,
the all-to-alls of chunk c + 1's inputs and of chunk c - 1's outputs are in
flight (asynchronous NCCL collectives on their own stream, waited for on the
compute stream only where their data is used).

``pack`` / ``unpack`` / ``all_to_all`` default to the library kernels and
``torch.distributed``; tests inject host versions to check the exchange
logic with the gloo backend on CPU.
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch
import torch.distributed as dist

from . import kernels


def _default_all_to_all(out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, group):
    """Asynchronous all-to-all; the returned work's ``wait()`` orders the
    current stream after it."""
    return dist.all_to_all_single(out, inp, output_split_sizes=list(out_splits),
                                  input_split_sizes=list(in_splits), group=group, async_op=True)


def chunk_plan(H: int, P: int, chunks: int) -> list:
    """Head chunks of the pipelined exchange: a list of ``(c0, offs)`` with
    chunk c = heads [c0, c0 + offs[-1]) and rank j's share of it
    [c0 + offs[j], c0 + offs[j + 1]).  Rank j's shares add up to its count in
    the contiguous split ``head_split(H, P)``."""
    per_rank = kernels.head_split(H, P)
    counts = [per_rank[j + 1] - per_rank[j] for j in range(P)]
    plan, c0 = [], 0
    for c in range(max(1, chunks)):
        offs = [0]
        for n in counts:
            base, extra = divmod(n, max(1, chunks))
            offs.append(offs[-1] + base + (1 if c < extra else 0))
        if offs[-1] > 0:
            plan.append((c0, offs))
        c0 += offs[-1]
    return plan


class UlyssesAttention:
    def __init__(self, inner: Callable, heads: int, group=None, seq_lens: Optional[Sequence[int]] = None,
                 pack: Optional[Callable] = None, unpack: Optional[Callable] = None,
                 all_to_all: Optional[Callable] = None, chunks: int = 3):
        """``inner(q, k, v, out=o)`` computes attention of ``[B, h, S, D]``
        (strided) views into ``o``; ``heads`` is the total head count H;
        ``seq_lens`` the per-rank shard lengths (default: equal shards);
        ``chunks`` the head chunks of the pipelined exchange.  An injected
        ``all_to_all`` may run synchronously (return None) or return a work
        with ``wait()``."""
        self.inner = inner
        self.heads = heads
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        self.seq_lens = list(seq_lens) if seq_lens is not None else None
        self.head_off = kernels.head_split(heads, self.world)
        self.plan = chunk_plan(heads, self.world, chunks)
        self.pack = pack or (lambda ts, off: kernels.ulysses_pack(ts, off))
        self.unpack = unpack or kernels.ulysses_unpack
        self.all_to_all = all_to_all or _default_all_to_all
        self.last = {}

    @property
    def local_heads(self) -> int:
        return self.head_off[self.rank + 1] - self.head_off[self.rank]

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        B, s, H, D = q.shape
        if H != self.heads or k.shape != q.shape or v.shape != q.shape:
            raise ValueError(f"expected q, k, v [B, s, {self.heads}, D] sequence shards")
        P, r = self.world, self.rank
        lens = self.seq_lens or [s] * P
        if len(lens) != P or lens[r] != s:
            raise ValueError(f"shard length {s} does not match seq_lens {lens}")
        S = sum(lens)
        off = self.head_off
        h = off[r + 1] - off[r]
        if P == 1:
            # one rank holds every head and the whole sequence: the kernels
            # read the [B, S, H, D] inputs as strided [B, H, S, D] views and
            # write the output rows in place, no pack / unpack
            out = torch.empty(B, s, H, D, dtype=q.dtype, device=q.device)
            self.inner(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), out=out.transpose(1, 2))
            self.last = {"S": S, "local_heads": H, "send_elems": 0, "recv_elems": 0}
            return out
        # inputs of every chunk packed and sent up front (the collectives
        # run in order on the communication stream)
        sends = []
        for c0, offs in self.plan:
            hc = offs[-1]  # the chunk's heads; this rank's share h_c
            h_c = offs[r + 1] - offs[r]
            hs_c = [offs[j + 1] - offs[j] for j in range(P)]
            send = self.pack([t[:, :, c0:c0 + hc] for t in (q, k, v)], offs)
            recv = torch.empty(S * B * 3 * h_c * D, dtype=q.dtype, device=q.device)
            work = self.all_to_all(recv, send, [n * B * 3 * h_c * D for n in lens],
                                   [s * B * 3 * hj * D for hj in hs_c], self.group)
            sends.append((c0, hc, offs, h_c, hs_c, send, recv, work))
        backs = []
        send_elems = recv_elems = 0
        for c0, hc, offs, h_c, hs_c, send, recv, work in sends:
            if work is not None:
                work.wait()
            send_elems += send.numel()
            recv_elems += recv.numel()
            grid = recv.view(S, B, 3, h_c, D)
            qh, kh, vh = (grid[:, :, t].permute(1, 2, 0, 3) for t in range(3))
            o_rows = torch.empty(S, B, h_c, D, dtype=q.dtype, device=q.device)
            if h_c > 0:
                self.inner(qh, kh, vh, out=o_rows.permute(1, 2, 0, 3))
            back = torch.empty(s * B * hc * D, dtype=q.dtype, device=q.device)
            wb = self.all_to_all(back, o_rows.view(-1), [s * B * hj * D for hj in hs_c],
                                 [n * B * h_c * D for n in lens], self.group)
            backs.append((c0, hc, offs, back, o_rows, wb))
        out = torch.empty(B, s, H, D, dtype=q.dtype, device=q.device)
        for c0, hc, offs, back, o_rows, wb in backs:
            if wb is not None:
                wb.wait()
            self.unpack(back, [out[:, :, c0:c0 + hc]], offs)
        self.last = {"S": S, "local_heads": h, "send_elems": send_elems, "recv_elems": recv_elems,
                     "chunks": len(self.plan)}
        return out
