"""Drop-in for special_attentions/utils/mask_related.py: block-mask helpers.

* ``calc_attn_block_sum_efficient(q, k, block_size, num_keep)`` (reference
  :40-81) -- the block attention estimate.  The reference samples
  ``num_keep`` random tokens of every block and sum-pools the softmax of the
  sampled logits; here the estimate is deterministic: the softmax numerator
  of the mean-pooled block logits weighted by the key block's token count
  (saf_pool_topk's fp64 scores turned into mass by saf_energy_select), each
  row normalised to sum to 1.  Row-wise rules (top-k, energy thresholds) do
  not depend on the row's scale.
* ``generate_attention_mask_frame_scope`` (:194-245) -- saf_frame_mask on the
  GPU.  The reference draws its spatial sample with ``torch.randint`` from
  the default CPU generator; the same draw is made here unless ``spatial`` is
  given, so a seeded caller gets the reference's sample.
* ``get_inner_frame_mask`` (:344-393) -- with the reference's default
  threshold 1 every block of the frame holds part of the mass and is kept in
  exact arithmetic, so the mask is all True; other thresholds are not part
  of this build.
* ``get_block_mask`` (:397-404) -- the kron of the frame mask with the inner
  block mask plus four dense text blocks, for any batch and head count (the
  reference fixes them at 2 x 30).
* ``pad_to_multiple``, ``random_sample_tokens`` (:2-37), ``preprocess_qkv``
  and ``reverse_process_out`` (:87-187) -- the reference's layout helpers
  (frame-wise padding of q, random per-frame truncation of k / v), as tensor
  reshapes and gathers.  The block-sparse path of this build does not need
  them: BlockSparseAttention.forward_backup works on the unpadded sequence.

The k-means token rearrangers (ClusterRearrange*) are not part of this build.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from ... import kernels


def pad_to_multiple(x: torch.Tensor, multiple: int) -> torch.Tensor:
    """Pads dim 2 of ``[B, H, L, D]`` to a multiple of ``multiple`` by
    repeating the last token."""
    rem = x.size(2) % multiple
    if rem == 0:
        return x
    return F.pad(x, (0, 0, 0, multiple - rem), mode="replicate")


def random_sample_tokens(x: torch.Tensor, block_size: int = 64, sample_num: int = 8,
                         generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """``sample_num`` distinct random tokens of every block of ``block_size``
    (L a multiple of it): ``[B, H, L / block_size * sample_num, D]``."""
    B, H, L, D = x.shape
    nb = L // block_size
    u = torch.rand(B, H, nb, block_size, device=x.device, generator=generator)
    idx = u.topk(sample_num, dim=3).indices
    blocks = x.view(B, H, nb, block_size, D)
    return blocks.gather(3, idx[..., None].expand(-1, -1, -1, -1, D)).reshape(B, H, nb * sample_num, D)


def calc_attn_block_sum_efficient(q: torch.Tensor, k: torch.Tensor, block_size: int = 64,
                                  num_keep: int = 16) -> torch.Tensor:
    """Block attention estimate ``[B, H, nbq, nbk]`` (fp64, rows summing to 1)
    from mean-pooled q / k blocks.  ``num_keep`` (the reference's sample
    size) has no role in the deterministic estimate."""
    del num_keep
    nbk = math.ceil(k.shape[2] / block_size)
    csr = kernels.pool_topk(q, k, block_m=block_size, block_n=block_size, topk=1, return_scores=True)
    _, mass = kernels.energy_select(csr.scores, threshold=1.0, min_retain=0, max_retain=nbk, is_mass=False,
                                    scale=1.0 / math.sqrt(q.shape[-1]), block_n=block_size, Sk=k.shape[2],
                                    return_mass=True)
    return mass / mass.sum(dim=-1, keepdim=True)


def generate_attention_mask_frame_scope(q: torch.Tensor, k: torch.Tensor, text_length: int = 226, f: int = 13,
                                        width: int = 45, height: int = 30, sample_num: int = 60,
                                        scale_factor: float = 1 / 8, base_threshold: float = 0.9, *,
                                        spatial: Optional[torch.Tensor] = None,
                                        generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """Bool frame x frame mask ``[B, H, f, f]`` of the sampled attention's
    per-head energy (saf_frame_mask)."""
    if spatial is None:
        spatial = torch.randint(0, width * height, (sample_num,), generator=generator)
    fm = kernels.frame_mask(q, k, spatial, text_len=text_length, frames=f, frame_len=width * height,
                            threshold=base_threshold, sm_scale=scale_factor)
    return fm.mask.bool()


def get_inner_frame_mask(q: torch.Tensor, k: torch.Tensor, scope: str = "row", original_length: int = 1350,
                         stride: int = 64, threshold: float = 1) -> torch.Tensor:
    """Per-frame block mask ``[B, H, ceil(L/stride), floor(L/stride)]`` for
    threshold 1 (every block kept)."""
    if not 0 < threshold <= 1:
        raise AssertionError("threshold must be in (0, 1]")
    if threshold != 1:
        raise NotImplementedError("only threshold 1 (keep every block) is part of this build")
    if scope not in ("row", "head"):
        raise ValueError(f"unknown scope {scope!r}")
    rows = math.ceil(original_length / stride)
    cols = original_length // stride
    return torch.ones(q.shape[0], q.shape[1], rows, cols, dtype=torch.bool, device=q.device)


def get_block_mask(inner_frame_mask: torch.Tensor, frame_mask: torch.Tensor, text_blocks: int = 4) -> torch.Tensor:
    """``kron(frame_mask, inner_frame_mask)`` per (batch, head) followed by
    ``text_blocks`` dense rows and columns (float32, as the reference)."""
    B, H, F1, F2 = frame_mask.shape
    r, c = inner_frame_mask.shape[-2:]
    video = frame_mask.float()[:, :, :, None, :, None] * inner_frame_mask.float()[:, :, None, :, None, :]
    video = video.reshape(B, H, F1 * r, F2 * c)
    return F.pad(video, (0, text_blocks, 0, text_blocks), value=1.0)


def preprocess_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, stride: int = 64, text_length: int = 226,
                   frame_length: int = 1350, frame_num: int = 13,
                   generator: Optional[torch.Generator] = None):
    """The reference's frame-aligned layout: q's frames zero-padded to a
    multiple of ``stride``, k / v frames cut to a multiple of ``stride`` at a
    random start per (batch, frame) shared by the heads, text moved to the
    end: returns ``(q', k', v')``."""
    def frames(x):
        return x[:, :, text_length:text_length + frame_num * frame_length].reshape(
            x.shape[0], x.shape[1], frame_num, frame_length, x.shape[3])

    rem = frame_length % stride
    qv = frames(q)
    if rem:
        qv = F.pad(qv, (0, 0, 0, stride - rem))
    kv_parts = [frames(k), frames(v)]
    if rem:
        keep = frame_length - rem
        B = k.shape[0]
        starts = torch.randint(0, rem + 1, (B, frame_num), device=k.device, generator=generator)
        idx = starts[..., None] + torch.arange(keep, device=k.device)
        idx = idx[:, None, :, :, None].expand(-1, k.shape[1], -1, -1, k.shape[3])
        kv_parts = [x.gather(3, idx) for x in kv_parts]
    out_q = torch.cat([qv.reshape(q.shape[0], q.shape[1], -1, q.shape[3]), q[:, :, :text_length]], dim=2)
    out_k, out_v = (torch.cat([x.reshape(x.shape[0], x.shape[1], -1, x.shape[4]), y[:, :, :text_length]], dim=2)
                    for x, y in zip(kv_parts, (k, v)))
    return out_q, out_k, out_v


def reverse_process_out(out: torch.Tensor, text_length: int = 226, original_length: int = 1350,
                        stride: int = 64, frame_num: int = 13) -> torch.Tensor:
    """Inverse of ``preprocess_qkv`` for the query side: text back in front,
    each frame's padding dropped."""
    padded = math.ceil(original_length / stride) * stride
    text = out[:, :, -text_length:]
    video = out[:, :, :-text_length].reshape(out.shape[0], out.shape[1], frame_num, padded, out.shape[3])
    video = video[:, :, :, :original_length].reshape(out.shape[0], out.shape[1], -1, out.shape[3])
    return torch.cat([text, video], dim=2)
