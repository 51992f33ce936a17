"""Drop-in for special_attentions/MergeAttention.py.

The reference processor (MergeAttention.py:14-51) merges the video tokens of
k and v with ToMe every ``gap`` steps -- per (batch, head) row, on the metric
``[k, |k|, v, |v|]`` (:26-31) -- and runs SDPA of the full q against the
merged k / v with a ``log(size)`` bias on the dst columns (proportional
attention, :33-38, :45-49); with ``full_merge`` q is merged too and the output
unmerged (:39-44).

Here the matching, merge and unmerge are the sm_100a ToMe kernels and the
attention is the block-sparse kernel with every block live and the bias as a
per-key-column fp32 bias.  The reference reads the step from an external
``global_vars.count``; this class keeps its own step counter (``count``), or
takes ``step=`` per call.  Shapes come from ``merge_config`` (w, h, t of the
video grid) and the inputs (text rows = S - w*h*t, in front).
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .. import kernels
from .utils.merge_unmerge import bipartite_soft_matching_video, init_generator


class MergeAttention:
    def __init__(self, merge_config: Optional[dict] = None, full_merge: bool = False, gap: int = 1,
                 block: int = 128):
        self.merge_config = dict(merge_config or {"w": 45, "h": 30, "t": 13, "sx": 3, "sy": 3,
                                                  "st": 4, "r": 9000})
        self.full_merge = full_merge
        self.gap = gap
        self.block = block
        self.count = 0
        self.generator = None
        self.merge_fn = self.unmerge_fn = None
        self.bias = None
        self._csr = {}

    def _dense_csr(self, B, H, Sq, Sk, dev):
        key = (B, H, Sq, Sk, dev)
        if key not in self._csr:
            nbq, nbk = math.ceil(Sq / self.block), math.ceil(Sk / self.block)
            mask = torch.ones(B, H, nbq, nbk, dtype=torch.bool, device=dev)
            self._csr[key] = kernels.mask_to_csr(mask, self.block, self.block)
        return self._csr[key]

    def _match(self, k: torch.Tensor, v: torch.Tensor):
        cfg = self.merge_config
        B, H, S, D = k.shape
        n = cfg["w"] * cfg["h"] * cfg["t"]
        text = S - n
        if self.generator is None:
            self.generator = init_generator(k.device)
        metric = kernels.tome_kv_metric(k, v, text)  # [k, |k|, v, |v|] per video token
        self.merge_fn, self.unmerge_fn = bipartite_soft_matching_video(
            metric, **cfg, generator=self.generator)
        plan = self.merge_fn.plan
        L = text + plan.merged_len
        bias = torch.zeros(B * H, L, dtype=torch.float32, device=k.device)
        bias[:, L - plan.Nd:] = plan.log_count
        self.bias = bias

    def forward(self, q, k, v, step: Optional[int] = None):
        step = self.count if step is None else step
        if step % self.gap == 0 or self.merge_fn is None or self.bias is None:
            self._match(k, v)
        B, H, S, D = q.shape
        scale = 1.0 / math.sqrt(D)
        mk = self.merge_fn(k).view(B, H, -1, D)
        mv = self.merge_fn(v).view(B, H, -1, D)
        if self.full_merge:
            mq = self.merge_fn(q).view(B, H, -1, D)
            csr = self._dense_csr(B, H, mq.shape[2], mk.shape[2], q.device)
            out = kernels.bsa_fwd(mq, mk, mv, csr, scale, kv_bias=self.bias)
            out = self.unmerge_fn(out)
        else:
            csr = self._dense_csr(B, H, S, mk.shape[2], q.device)
            out = kernels.bsa_fwd(q, mk, mv, csr, scale, kv_bias=self.bias)
        self.count += 1
        return out

    def __call__(self, *args, **kwds):
        return self.forward(*args, **kwds)
