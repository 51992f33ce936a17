"""Drop-in for special_attentions/block_mask_attn.py.

The reference ``BlockSparseAttention`` (block_mask_attn.py:5-29) keeps a
frame-scope sparse path in ``forward_backup`` (:11-20) and a dense SDPA path
in ``forward`` / ``__call__`` (:21-29; ``__call__`` has no ``return``).  Here
the class is the block-sparse processor the build targets: ``__call__``
selects blocks by mean-pooled scores (top ``density`` of the key blocks of
every row block, text rows / columns dense) and runs the sm_100a sparse
attention kernel over the live blocks only, returning the output.

``forward_backup`` is the reference's frame-scope path: a frame x frame
mask from the attention of a sampled token subset (the per-head energy rule
of generate_attention_mask_frame_scope, mask_related.py:194-245), then
sparse attention where a video query of frame f1 sees the text keys and the
keys of the frames f2 its head's mask allows.  The reference pads q to
64-multiples per frame, randomly truncates k / v (mask_related.py:87-167)
and expands the frame mask by an inner per-frame block mask computed with
threshold 1 (which keeps every block in exact arithmetic); here the frame
mask applies token by token on the unpadded sequence (saf_frame_csr lists
the blocks, saf_bsa_fwd_frames masks inside them), so no token is padded,
dropped or assigned to the wrong frame.
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
        self.last_frame_mask = None  # frame masks of the latest forward_backup call

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

    def forward_backup(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                       spatial: torch.Tensor | None = None, sample_num: int = 60,
                       threshold: float = 0.9, scale_factor: float = 1 / 8,
                       generator: torch.Generator | None = None) -> torch.Tensor:
        """Frame-scope sparse attention (block_mask_attn.py:11-20).

        ``spatial``: the ``sample_num`` positions inside a frame sampled in
        every frame; drawn like the reference (``torch.randint`` on the CPU,
        from ``generator`` or the default generator) when not given.
        ``threshold`` / ``scale_factor``: the frame mask's energy fraction and
        logit scale (the reference's base_threshold 0.9 and 1/8)."""
        geo = self.geometry
        B, H, S, D = q.shape
        if S != geo.seq_len:
            raise ValueError(f"sequence length {S} does not match the geometry's {geo.seq_len}")
        if spatial is None:
            spatial = torch.randint(0, geo.frame_len, (sample_num,), generator=generator)
        fm = kernels.frame_mask(q, k, spatial, text_len=geo.text_len, frames=geo.frames,
                                frame_len=geo.frame_len, threshold=threshold, sm_scale=scale_factor)
        csr = kernels.frame_csr(fm, B, H, self.block_size, self.block_size)
        self.last_frame_mask = fm
        self.last_csr = csr
        scale = self.sm_scale if self.sm_scale is not None else 1.0 / math.sqrt(D)
        out = kernels.bsa_fwd_frames(q, k, v, csr, fm, scale)
        if self.check_status:
            _lib.raise_on_device_status(q.device.index)
        return out

    def __call__(self, q, k, v, out=None):
        return self.forward(q, k, v, out=out)
