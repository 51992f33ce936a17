"""Host restatement of the Ulysses layout steps -- TEST INFRASTRUCTURE ONLY.

``pack`` / ``unpack`` restate, with torch indexing on the CPU, what
``saf_ulysses_pack`` / ``saf_ulysses_unpack`` compute: P chunks back to
back, chunk j = heads [off[j], off[j+1]) of T sequence-sharded
``[B, s, H, D]`` tensors laid out as ``[s, B, T, h_j, D]``.  The reference
has no sequence-parallel path (it runs on one GPU); these define the layout
contract the multi-GPU exchange is tested against.
"""
from __future__ import annotations

import torch


def pack(tensors, head_off):
    P = len(head_off) - 1
    chunks = []
    for j in range(P):
        part = torch.stack([t[:, :, head_off[j]:head_off[j + 1]] for t in tensors], dim=2)  # [B,s,T,h,D]
        chunks.append(part.permute(1, 0, 2, 3, 4).reshape(-1))
    return torch.cat(chunks)


def unpack(buf, outs, head_off):
    P = len(head_off) - 1
    B, s, H, D = outs[0].shape
    T = len(outs)
    at = 0
    for j in range(P):
        h = head_off[j + 1] - head_off[j]
        n = s * B * T * h * D
        part = buf[at:at + n].view(s, B, T, h, D).permute(1, 0, 2, 3, 4)  # [B,s,T,h,D]
        for t in range(T):
            outs[t][:, :, head_off[j]:head_off[j + 1]] = part[:, :, t]
        at += n
