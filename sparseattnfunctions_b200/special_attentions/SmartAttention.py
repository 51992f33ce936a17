"""Drop-in for special_attentions/SmartAttention.py.

The reference processor (SmartAttention.py:75-168) gives every video frame's
queries the keys of the text, the first frame and the frames next to its own
(a block-tridiagonal frame band, :30-43), and picks per (batch, head)
between two token orders (:97-108): a probe of ``sample_num`` random query
rows compares full attention with the band mask in the natural (t, h, w)
order ("spatial") and in the (h, w, t) order ("temporal"); heads where the
temporal band is closer to full attention get their tokens reordered to
(h, w, t) (:155-160), run the band attention (:130-143), and are reordered
back (:164-166).

Here the band is a per-row key-interval mask served by the block-sparse
sm_100a kernel (``saf_bsa_fwd_ranges``; the static block list holds the
blocks the band touches, ~32% at CogVideoX-2B), the reorderings are one
gather each (``saf_permute_tokens``), and the probe runs the same kernel on
the sampled rows.  The temporal probe reads k / v in (h, w, t) order with
the band of the sampled rows' reordered positions, which equals the
reference's reordered mask (process_mask_back, :44-51) on natural keys.
Heads of the other order get no blocks in each pass, so each head is
computed once.

The probe's rows come from ``generator`` (a CPU ``torch.Generator``; the
global RNG when None, as the reference's ``torch.randint``); ``strategy=``
overrides the probe (bool ``[B, H]``, True = natural order).
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .. import kernels
from ..geometry import COGVIDEOX_2B, VideoGeometry, frame_band_ranges, ranges_block_mask, video_token_perm


class SmartAttention:
    def __init__(self, geometry: VideoGeometry = COGVIDEOX_2B, block_size: int = 128, sample_num: int = 64,
                 diag: int = 1, generator: Optional[torch.Generator] = None):
        self.geometry = geometry
        self.block_size = block_size
        self.sample_num = sample_num
        self.diag = diag
        self.generator = generator
        self._static = {}
        self.last_strategy = None

    def _layout(self, dev):
        if dev not in self._static:
            geo, bs = self.geometry, self.block_size
            ranges = frame_band_ranges(geo, self.diag, dev)
            perm, inv = video_token_perm(geo, dev)
            block = ranges_block_mask(ranges, geo.seq_len, bs, bs)
            self._static[dev] = dict(ranges=ranges, perm=perm, inv=inv, block=block)
        return self._static[dev]

    def _csr(self, block: torch.Tensor, heads_on: torch.Tensor) -> kernels.BlockCSR:
        B, H = heads_on.shape
        mask = block[None, None] & heads_on[:, :, None, None]
        return kernels.mask_to_csr(mask, self.block_size, self.block_size)

    def choose_strategy(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        k_perm: torch.Tensor, v_perm: torch.Tensor) -> torch.Tensor:
        """bool [B, H]: True where the natural-order band is closer to full
        attention on the sampled rows (SmartAttention.py:97-108)."""
        st = self._layout(q.device)
        B, H, S, D = q.shape
        idx = torch.randint(low=0, high=S, size=[self.sample_num], generator=self.generator)
        idx_d = idx.to(q.device)
        qs = q[:, :, idx_d].contiguous()
        scale = 1.0 / math.sqrt(D)
        n = self.sample_num
        nbk = math.ceil(S / self.block_size)
        dense = kernels.mask_to_csr(torch.ones(B, H, math.ceil(n / 64), nbk, dtype=torch.bool, device=q.device),
                                    64, self.block_size)
        full = kernels.bsa_fwd(qs, k, v, dense, scale)
        spatial = kernels.bsa_fwd(qs, k, v, dense, scale, row_ranges=st["ranges"][idx_d].contiguous())
        # the temporal band of a natural row = the band of its (h, w, t) position on reordered keys
        temporal = kernels.bsa_fwd(qs, k_perm, v_perm, dense, scale,
                                   row_ranges=st["ranges"][st["inv"][idx_d].long()].contiguous())
        sd = (spatial.float() - full.float()).pow(2).sum(dim=[-1, -2])
        td = (temporal.float() - full.float()).pow(2).sum(dim=[-1, -2])
        self.last_probe = dict(idx=idx, full=full, spatial=spatial, temporal=temporal)
        return sd < td

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                strategy: Optional[torch.Tensor] = None) -> torch.Tensor:
        st = self._layout(q.device)
        B, H, S, D = q.shape
        if S != self.geometry.seq_len:
            raise ValueError(f"sequence length {S} does not match the geometry ({self.geometry.seq_len})")
        scale = 1.0 / math.sqrt(D)
        k_perm = v_perm = None
        if strategy is None:
            k_perm = kernels.permute_tokens(k, st["perm"])
            v_perm = kernels.permute_tokens(v, st["perm"])
            strategy = self.choose_strategy(q, k, v, k_perm, v_perm)
        strategy = strategy.to(device=q.device, dtype=torch.bool)
        self.last_strategy = strategy
        out = torch.empty_like(q)
        if bool(strategy.any()):
            kernels.bsa_fwd(q, k, v, self._csr(st["block"], strategy), scale, out=out,
                            row_ranges=st["ranges"])
        if not bool(strategy.all()):
            heads = torch.nonzero(~strategy.flatten()).flatten().to(torch.int32)
            if k_perm is None:
                k_perm = kernels.permute_tokens(k, st["perm"], heads)
                v_perm = kernels.permute_tokens(v, st["perm"], heads)
            q_perm = kernels.permute_tokens(q, st["perm"], heads)
            o_perm = kernels.bsa_fwd(q_perm, k_perm, v_perm, self._csr(st["block"], ~strategy), scale,
                                     row_ranges=st["ranges"])
            kernels.permute_tokens(o_perm, st["inv"], heads, out=out)
        return out

    def __call__(self, q, k, v, strategy: Optional[torch.Tensor] = None):
        return self.forward(q, k, v, strategy)
