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

``pack`` / ``unpack`` / ``all_to_all`` default to the library kernels and
``torch.distributed``; tests inject host versions to check the exchange
logic with the gloo backend on CPU.
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch
import torch.distributed as dist

from . import kernels


def _default_all_to_all(out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, group) -> None:
    dist.all_to_all_single(out, inp, output_split_sizes=list(out_splits),
                           input_split_sizes=list(in_splits), group=group)


class UlyssesAttention:
    def __init__(self, inner: Callable, heads: int, group=None, seq_lens: Optional[Sequence[int]] = None,
                 pack: Optional[Callable] = None, unpack: Optional[Callable] = None,
                 all_to_all: Optional[Callable] = None):
        """``inner(q, k, v, out=o)`` computes attention of ``[B, h, S, D]``
        (strided) views into ``o``; ``heads`` is the total head count H;
        ``seq_lens`` the per-rank shard lengths (default: equal shards)."""
        self.inner = inner
        self.heads = heads
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        self.seq_lens = list(seq_lens) if seq_lens is not None else None
        self.head_off = kernels.head_split(heads, self.world)
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
        hs = [off[j + 1] - off[j] for j in range(P)]
        if P == 1:
            # one rank holds every head and the whole sequence: the kernels
            # read the [B, S, H, D] inputs as strided [B, H, S, D] views and
            # write the output rows in place, no pack / unpack
            out = torch.empty(B, s, H, D, dtype=q.dtype, device=q.device)
            self.inner(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), out=out.transpose(1, 2))
            self.last = {"S": S, "local_heads": H, "send_elems": 0, "recv_elems": 0}
            return out
        send = self.pack([q, k, v], off)
        recv = torch.empty(S * B * 3 * h * D, dtype=q.dtype, device=q.device)
        self.all_to_all(recv, send, [n * B * 3 * h * D for n in lens], [s * B * 3 * hj * D for hj in hs],
                        self.group)
        grid = recv[:S * B * 3 * h * D].view(S, B, 3, h, D)
        qh, kh, vh = (grid[:, :, t].permute(1, 2, 0, 3) for t in range(3))
        o_rows = torch.empty(S, B, h, D, dtype=q.dtype, device=q.device)
        oh = o_rows.permute(1, 2, 0, 3)
        if h > 0:
            self.inner(qh, kh, vh, out=oh)
        back = torch.empty(s * B * H * D, dtype=q.dtype, device=q.device)
        self.all_to_all(back, o_rows.view(-1), [s * B * hj * D for hj in hs], [n * B * h * D for n in lens],
                        self.group)
        out = torch.empty(B, s, H, D, dtype=q.dtype, device=q.device)
        self.unpack(back, [out], off)
        self.last = {"S": S, "local_heads": h, "send_elems": send.numel(), "recv_elems": recv.numel()}
        return out
