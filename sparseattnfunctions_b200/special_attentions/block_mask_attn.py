"""Drop-in for special_attentions/block_mask_attn.py.

The reference ``BlockSparseAttention`` (block_mask_attn.py:5-29) keeps a
frame-scope sparse path in ``forward_backup`` (:11-20) and a dense SDPA path
in ``forward`` / ``__call__`` (:21-29; ``__call__`` has no ``return``).  Here
the class is the block-sparse processor the build targets: ``__call__``
selects blocks by mean-pooled scores (top ``density`` of the key blocks of
every row block, text rows / columns dense) and runs the sm_100a sparse
attention kernel over the live blocks only, returning the output.

``forward_backup`` keeps the reference's frame-scope idea (a frame x frame
energy mask of the sampled attention map) but builds the block list directly
on the unpadded sequence, so no token is padded or truncated
(the reference pads Q and randomly truncates K/V: mask_related.py:87-167).
"""
from __future__ import annotations

import math

import torch

from .. import _lib, kernels
from ..geometry import COGVIDEOX_2B, VideoGeometry


class BlockSparseAttention:
    def __init__(self, block_size: int = 128, density: float = 0.10,
                 geometry: VideoGeometry = COGVIDEOX_2B, text_dense: bool = True,
                 sm_scale: float | None = None, check_status: bool = False):
        """``check_status``: after every call, synchronise the device and
        raise ``SafTimeoutError`` (a kernel wait ran out) or ``SafError`` (an
        index was out of range and skipped) if the device status word is
        set.  Off by default: it costs a host synchronisation per call."""
        super().__init__()
        self.check_status = check_status
        self.block_size = block_size
        self.density = density
        self.geometry = geometry
        self.text_dense = text_dense
        self.sm_scale = sm_scale
        self.last_csr = None  # block list of the latest call (for inspection)

    def select(self, q: torch.Tensor, k: torch.Tensor) -> kernels.BlockCSR:
        bs = self.block_size
        nbk = math.ceil(k.shape[2] / bs)
        topk = max(1, math.ceil(self.density * nbk))
        text = self.geometry.text_blocks(bs) if self.text_dense else 0
        return kernels.pool_topk(q, k, block_m=bs, block_n=bs, topk=topk, text_blocks_q=text,
                                 text_blocks_k=text)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """``out``: optional (possibly strided) ``[B, H, S, D]`` destination."""
        scale = self.sm_scale if self.sm_scale is not None else 1.0 / math.sqrt(q.shape[-1])
        csr = self.select(q, k)
        self.last_csr = csr
        out = kernels.bsa_fwd(q, k, v, csr, scale, out=out)
        if self.check_status:
            _lib.raise_on_device_status(q.device.index)
        return out

    def __call__(self, q, k, v, out=None):
        return self.forward(q, k, v, out=out)
