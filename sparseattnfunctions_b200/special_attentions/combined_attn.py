"""Drop-in for special_attentions/combined_attn.py: token merging fused with
block-sparse attention (combined attention).

The reference ``CombinedAttn`` (combined_attn.py:7-101) runs its
block-sparse processor for ``warmup_epoch`` passes over the ``layer_num``
layers (:43-47) and then splits heads between a pattern attention and the
block-sparse path (:48-100).  The build's combined attention is the
composition the target names, on the sm_100a kernels:

1. ToMe matching per (batch, head) on the metric ``[k, |k|, v, |v|]`` of the
   video tokens (as MergeAttention.py:26-31), refreshed every ``gap`` steps
   of each layer;
2. size-weighted merge of q (with ``full_merge``), k and v, text rows kept in
   front (merge_unmerge.py:119-135);
3. block selection on the merged sequence by mean-pooled scores, top
   ``density`` of the key blocks per row block, text rows / columns dense;
4. block-sparse attention over the live blocks with the proportional
   ``log(size)`` bias on the merged dst columns (MergeAttention.py:33-38);
5. unmerge of the output back to the full sequence (merge_unmerge.py:137-154).

Warm-up passes use the plain block-sparse processor at the same density, as
the reference does.  ``use_rearranger`` (the CogVideoX1.5-5B tile
rearrangement of combined_attn.py:17-41, only reached on the pattern path)
is not provided and raises ``NotImplementedError``.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .. import kernels
from ..geometry import COGVIDEOX_2B, VideoGeometry
from .block_mask_attn import BlockSparseAttention
from .MergeAttention import MergeAttention


class CombinedAttn:
    def __init__(self, warmup_epoch: int = 0, layer_num: int = 30, merge_config: Optional[dict] = None,
                 density: float = 0.15, block_size: int = 128, gap: int = 1, full_merge: bool = True,
                 geometry: VideoGeometry = COGVIDEOX_2B):
        self.layer_num = layer_num
        self.warmup_epoch = warmup_epoch
        self.density = density
        self.block_size = block_size
        self.full_merge = full_merge
        self.geometry = geometry
        cfg = dict(merge_config or {"w": geometry.width, "h": geometry.height, "t": geometry.frames,
                                    "sx": 3, "sy": 3, "st": 4, "r": 4000})
        self.block_sparse_attention = BlockSparseAttention(block_size=block_size, density=density,
                                                           geometry=geometry)
        # one matching state per layer: plans are refreshed per layer every `gap` steps
        self._layers = [MergeAttention(merge_config=cfg, full_merge=full_merge, gap=gap, block=block_size)
                        for _ in range(layer_num)]
        self.ct = 0
        self.last_csr = None

    @property
    def merge_config(self) -> dict:
        return self._layers[0].merge_config

    def _select(self, q: torch.Tensor, k: torch.Tensor, text_len: int) -> kernels.BlockCSR:
        bs = self.block_size
        nbk = math.ceil(k.shape[2] / bs)
        topk = max(1, math.ceil(self.density * nbk))
        text = math.ceil(text_len / bs) if text_len > 0 else 0
        return kernels.pool_topk(q, k, block_m=bs, block_n=bs, topk=topk, text_blocks_q=text,
                                 text_blocks_k=text)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                use_rearranger: bool = False) -> torch.Tensor:
        if use_rearranger:
            raise NotImplementedError("the CogVideoX1.5-5B tile rearranger is not provided")
        layer = self.ct % self.layer_num
        warm = self.ct // self.layer_num < self.warmup_epoch
        self.ct += 1
        if warm:
            return self.block_sparse_attention(q, k, v)
        st = self._layers[layer]
        if st.count % st.gap == 0 or st.merge_fn is None or st.bias is None:
            st._match(k, v)
        st.count += 1
        B, H, S, D = q.shape
        cfg = st.merge_config
        text_len = S - cfg["w"] * cfg["h"] * cfg["t"]
        scale = 1.0 / math.sqrt(D)
        mk = st.merge_fn(k).view(B, H, -1, D)
        mv = st.merge_fn(v).view(B, H, -1, D)
        if self.full_merge:
            mq = st.merge_fn(q).view(B, H, -1, D)
            csr = self._select(mq, mk, text_len)
            out = kernels.bsa_fwd(mq, mk, mv, csr, scale, kv_bias=st.bias)
            out = st.unmerge_fn(out)
        else:
            csr = self._select(q, mk, text_len)
            out = kernels.bsa_fwd(q, mk, mv, csr, scale, kv_bias=st.bias)
        self.last_csr = csr
        return out

    def __call__(self, q, k, v, use_rearranger: bool = False):
        return self.forward(q, k, v, use_rearranger)
