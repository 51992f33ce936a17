"""Drop-in for special_attentions/SparseGen_Plus.py: the adaptive-density
block-sparse processor.

The reference processor (SparseGen_Plus.py:105-212) runs dense attention for
``warmup_epoch`` denoising steps, then per call estimates the attention mass
of every (row block, key block) pair, keeps per row the smallest set of key
blocks holding ``energy_threshold`` of the mass (clamped to a retain ratio
range; all three follow per-timestep schedules, :117-121) and runs the
block-sparse kernel on 64x64 blocks.

Here the mass estimate is the deterministic mean-pool one (softmax numerator
of the pooled logits, weighted by key block size) instead of the reference's
random 8-of-64 token sample (mask_related.py:14-81); the selection rule is the
reference's, computed on the GPU (``saf_energy_select``), and dense warm-up
steps run the same kernel with every block live (the reference calls
sageattention, which is not part of this path).  With
``warmup_pooling=True`` the warm-up steps run the attention with a pooled
attention map (``utils/attn_pooling_kernel.py``) and the first sparse step of
every layer selects its blocks from the last warm-up map of that layer (an
exact block-level attention estimate obtained in the dense pass) instead of
the mean-pool estimate.  Sparsity records are kept in memory
(``sparsity_records``); nothing is printed or written to files.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

from .. import kernels


def transfer_attn_to_mask(attn: torch.Tensor, mode: str = "energy", init_k=None, max_retain_ratio: float = 0.7,
                          min_retain_ratio: float = 0.1, energy_threshold: float = 0.95,
                          text_blocks: int = 4) -> torch.Tensor:
    """Bool block mask ``[B, H, n, n']`` from a non-negative block attention
    estimate ``attn`` (SparseGen_Plus.py:12-84).  ``mode="energy"``: per row
    the smallest set of blocks holding ``energy_threshold`` of the mass,
    clamped to the retain ratios.  ``mode="topk"``: ``init_k`` blocks per row
    (a fraction of the row when below 1), tripled for rows whose first
    ``init_k`` hold under 60 % of the mass, then cut to 2/3 for rows under
    90 % (the reference's rule, :28-50).  Text rows / columns forced."""
    n = attn.shape[-1]
    if mode == "topk":
        if init_k is None:
            raise ValueError("the topk mode needs an initial k (init_k)")
        if attn.shape[-2] != n:
            raise ValueError("the topk mode takes a square block map (the reference caps k at its row count)")
        k0 = int(n * init_k) if init_k < 1 else int(init_k)
        mask = kernels.topk_adaptive_select(attn, init_k=k0, text_blocks=text_blocks, is_mass=True)
        return mask.bool()
    if mode != "energy":
        raise ValueError(f"Unsupported mode: {mode}")
    min_retain = max(1, int(n * min_retain_ratio))
    max_retain = max(1, int(n * max_retain_ratio))
    mask = kernels.energy_select(attn, threshold=energy_threshold, min_retain=min_retain,
                                 max_retain=max_retain, text_blocks=text_blocks, is_mass=True)
    return mask.bool()


def concentrated_interpolation(min_val, max_val, n_points, concentration=0.2):
    """Schedule values concentrated near both ends (SparseGen_Plus.py:86-103)."""
    concentration = np.clip(concentration, 0.05, 0.95)
    x = np.linspace(-6, 6, n_points)
    scale = 2 * (1 - concentration)
    cdf = 1 / (1 + np.exp(-x / scale))
    return np.clip(max_val - cdf * (max_val - min_val), min_val, max_val)


class BlockSparseAttention:
    def __init__(self, block_size: int = 64, layernum: int = 42, timestep: int = 50, num_samples: int = 1,
                 warmup_epoch: int = 5, text_blocks: int = 4, warmup_pooling: bool = False):
        self.block_size = block_size
        self.sm_scale = 1 / 8
        self.layernum = layernum
        self.timestep = timestep
        self.num_samples = num_samples
        self.counter = 0
        self.warmup_epoch = warmup_epoch
        self.text_blocks = text_blocks
        self.sparsity_records = [{"records": []} for _ in range(num_samples)]
        self.update_list = []
        self.mask = [None] * layernum
        self.k_list = [0.3, 0.2, 0.15, 0.1]
        self.max_retain_ratio_list = concentrated_interpolation(0.8, 1, 50, concentration=0.5)
        self.min_retain_ratio_list = concentrated_interpolation(0.1, 0.12, 50, concentration=0.5)
        self.energy_threshold_list = concentrated_interpolation(0.9, 0.98, 50, concentration=0.5)
        self.last_mass = None
        self.warmup_pooling = warmup_pooling
        self.warmup_map = [None] * layernum  # pooled map of the layer's last warm-up step

    def schedule(self, step: int):
        """(max_retain_ratio, min_retain_ratio, energy_threshold) of a step."""
        i = min(step, len(self.energy_threshold_list) - 1)
        return (float(self.max_retain_ratio_list[i]), float(self.min_retain_ratio_list[i]),
                float(self.energy_threshold_list[i]))

    def select(self, q: torch.Tensor, k: torch.Tensor, step: int, layer: int = 0) -> kernels.BlockCSR:
        bs = self.block_size
        Sk = k.shape[2]
        nbk = math.ceil(Sk / bs)
        max_r, min_r, thr = self.schedule(step)
        keep = dict(threshold=thr, min_retain=max(1, int(nbk * min_r)), max_retain=max(1, int(nbk * max_r)),
                    text_blocks=self.text_blocks, return_mass=True)
        wmap = self.warmup_map[layer] if self.warmup_pooling else None
        if wmap is not None:
            self.warmup_map[layer] = None
            mask, mass = kernels.energy_select(wmap, is_mass=True, **keep)
        else:
            pooled = kernels.pool_topk(q, k, block_m=bs, block_n=bs, topk=1, return_scores=True)
            mask, mass = kernels.energy_select(pooled.scores, is_mass=False, scale=self.sm_scale, block_n=bs,
                                               Sk=Sk, **keep)
        self.last_mass = mass
        return kernels.mask_to_csr(mask, bs, bs, dense_rows=min(self.text_blocks, mask.shape[2]))

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        self.sm_scale = 1 / q.size(-1) ** 0.5
        counter = self.counter % (self.layernum * self.timestep)
        layer, step = counter % self.layernum, counter // self.layernum
        csr = self.select(q, k, step, layer)
        self.mask[layer] = csr
        out = kernels.bsa_fwd(q, k, v, csr, self.sm_scale)
        sparsity = self._calculate_sparsity(csr)
        sample = self.counter // (self.layernum * self.timestep)
        if sample < len(self.sparsity_records):
            self.sparsity_records[sample]["records"].append(
                {"timestep": step, "layer": layer, "sparsity": sparsity})
        return out

    @staticmethod
    def _calculate_sparsity(csr: kernels.BlockCSR) -> float:
        """The reference's record (SparseGen_Plus.py:136-141): the fraction of
        dead blocks; with a batch of one it is blended as if the heads were
        H of 96 with the remaining 96 - H at 0.9."""
        dead = 1.0 - float(csr.nnz_per_head().sum()) / (csr.B * csr.H * csr.nbq * csr.nbk)
        if csr.B == 1:
            return (dead * csr.H + 0.9 * (96 - csr.H)) / 96
        return dead

    def dense(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layer: int = 0) -> torch.Tensor:
        bs = self.block_size
        B, H, Sq, _ = q.shape
        nbq, nbk = math.ceil(Sq / bs), math.ceil(k.shape[2] / bs)
        csr = kernels.mask_to_csr(torch.ones(B, H, nbq, nbk, dtype=torch.bool, device=q.device), bs, bs)
        if self.warmup_pooling:
            out, self.warmup_map[layer] = kernels.bsa_fwd_pool(q, k, v, csr, 1 / q.size(-1) ** 0.5, pool_block=bs)
            return out
        return kernels.bsa_fwd(q, k, v, csr, 1 / q.size(-1) ** 0.5)

    def __call__(self, q, k, v):
        counter = self.counter % (self.layernum * self.timestep)
        if counter // self.layernum < self.warmup_epoch:
            out = self.dense(q, k, v, counter % self.layernum)
        else:
            out = self.forward(q, k, v)
        self.counter += 1
        if (self.counter // self.layernum) in self.update_list:
            self.mask = [None] * self.layernum
        return out
