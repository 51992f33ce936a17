"""Drop-in for special_attentions/utils/attn_pooling_kernel.py: attention
whose output comes with a pooled attention map.

``attn_with_pooling(q, k, v, causal, sm_scale, block_size) -> (o, Po)``
(reference ``_attention_pooling.forward``, :212-264): ``o`` is dense
softmax attention in the input dtype; ``Po [B, H, nb, nb]`` holds, for query
block i and key block j (both ``block_size`` wide), the largest normalised
probability any row of block i gives a key of block j, every row of Po then
divided by its sum -- a block-level attention estimate that costs no extra
pass over q and k.  The reference computes it in a Triton kernel on fp32
copies of bf16 inputs; here the sm_100a block-sparse attention kernel runs
every block and records each row's block maxima and log-sum-exp
(``saf_bsa_fwd_pool``), and two small kernels pool and normalise them.

Supported here: the non-causal case (the video DiT's), 16-bit inputs,
``block_size`` 64 or 128, head dim 64.  ``Po`` is fp32 for bf16 inputs (the
reference casts bf16 to fp32) and fp16 for fp16 inputs.
"""
from __future__ import annotations

import math

import torch

from ... import kernels


def attn_with_pooling(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, sm_scale: float,
                      block_size: int):
    assert block_size in {32, 64, 128}
    if causal:
        raise NotImplementedError("causal attention with pooling is not provided (video DiT attention is "
                                  "non-causal)")
    if block_size == 32:
        raise NotImplementedError("block_size 32: the tensor-core kernel takes 64- or 128-token blocks")
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise NotImplementedError("attention with pooling takes bf16 / fp16 inputs here")
    assert q.shape[-1] == k.shape[-1] == v.shape[-1]
    B, H, Sq, _ = q.shape
    Sk = k.shape[2]
    nbq, nbk = math.ceil(Sq / block_size), math.ceil(Sk / block_size)
    dense = torch.ones(B, H, nbq, nbk, dtype=torch.bool, device=q.device)
    csr = kernels.mask_to_csr(dense, block_size, block_size)
    o, po = kernels.bsa_fwd_pool(q, k, v, csr, sm_scale, pool_block=block_size)
    if q.dtype == torch.float16:
        po = po.to(torch.float16)
    return o, po
