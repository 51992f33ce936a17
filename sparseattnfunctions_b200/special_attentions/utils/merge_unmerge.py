"""Drop-in for special_attentions/utils/merge_unmerge.py.

``bipartite_soft_matching_video(metric, w, h, t, sx, sy, st, r, no_rand=False,
generator=None)`` returns ``(merge, unmerge)`` closures like the reference
(:34-156), with the matching, merge and unmerge done by the sm_100a library
(``saf_tome_match`` / ``saf_tome_merge`` / ``saf_tome_unmerge``).

Split (:62-97): the whole first frame and one token per (st, sy, sx) cell of
frames 1..t-1 go to dst (the ``rand_idx``-th of the cell, drawn from
``generator``; the top-left one with ``no_rand``), every other video token to
src.  The reference orders both lists with an unstable ``argsort`` (:82);
here the order is the stable one (ascending token index), computed with torch
ops on the metric's device.  ``split=(a_idx, b_idx)`` overrides the split
(e.g. the BASELINE config-3 alternate split, or the reference's own order).

Matching contract: exact fp64 cosine similarity of the metric values (the
reference normalises and multiplies in the metric's dtype, which in bf16 is
tie-dominated), arg-max ties to the lower dst position, stable sort.

``merge(x)``: 3-D ``[B, N(+text), C]`` or 4-D ``[b, h, S, D]`` with
``b*h == B`` (the reference's MergeAttention layout, text rows first); the
text rows (``S - N``) are kept in front, as the reference does for 4-D
inputs (:120-128).  ``unmerge(y)`` inverts it, returning the 4-D shape when
the last merge was 4-D.  The module attribute ``counter`` holds the merged
sizes ``[B, Nd, 1]`` (int64) after each matching, as in the reference.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch

from ... import kernels

counter = None


def do_nothing(x: torch.Tensor, mode: str = None):
    return x


def init_generator(device: torch.device, fallback: torch.Generator = None):
    """A generator on ``device`` seeded from the current RNG state
    (merge_unmerge.py:8-22)."""
    if device.type == "cpu":
        return torch.Generator(device="cpu").set_state(torch.get_rng_state())
    if device.type == "cuda":
        return torch.Generator(device=device).set_state(torch.cuda.get_rng_state(device))
    return fallback if fallback is not None else init_generator(torch.device("cpu"))


def video_split(w: int, h: int, t: int, sx: int, sy: int, st: int, device,
                rand_idx: Optional[torch.Tensor] = None):
    """(a_idx, b_idx) int32 video-token indices on ``device`` (stable order)."""
    tt = t - 1
    hsy, wsx, tst = h // sy, w // sx, tt // st
    if rand_idx is None:
        rand_idx = torch.zeros(tst, hsy, wsx, 1, dtype=torch.int64, device=device)
    rand_idx = rand_idx.to(device=device, dtype=torch.int64).reshape(tst, hsy, wsx, 1)
    buf = torch.zeros(tst, hsy, wsx, st * sy * sx, dtype=torch.int64, device=device)
    buf.scatter_(3, rand_idx, -torch.ones_like(rand_idx))
    buf = buf.view(tst, hsy, wsx, st, sy, sx).permute(0, 3, 1, 4, 2, 5).reshape(tst * st, hsy * sy, wsx * sx)
    if tst * st < tt or hsy * sy < h or wsx * sx < w:
        full = torch.zeros(tt, h, w, dtype=torch.int64, device=device)
        full[:tst * st, :hsy * sy, :wsx * sx] = buf
        buf = full
    # the stable argsort of the {-1, 0} buffer is a stable partition (the one
    # dst token of every cell first, in token order, then the src tokens):
    # two prefix counts and a scatter instead of a device radix sort
    flat = buf.reshape(-1)
    n = flat.numel()
    num_dst = tst * hsy * wsx
    is_dst = flat < 0
    c_dst = torch.cumsum(is_dst, 0)
    pos = torch.where(is_dst, c_dst - 1, num_dst + torch.arange(n, device=device) - c_dst)
    order = torch.empty(n, dtype=torch.int64, device=device)
    order.scatter_(0, pos, torch.arange(n, dtype=torch.int64, device=device))
    order += w * h
    a_idx = order[num_dst:]
    b_idx = torch.cat([torch.arange(w * h, device=device), order[:num_dst]])
    return a_idx.to(torch.int32), b_idx.to(torch.int32)


def alternate_split(n: int, device):
    """src = even tokens, dst = odd tokens."""
    idx = torch.arange(n, device=device, dtype=torch.int32)
    return idx[0::2].contiguous(), idx[1::2].contiguous()


def bipartite_soft_matching_video(metric: torch.Tensor, w: int, h: int, t: int, sx: int, sy: int,
                                  st: int, r: int, no_rand: bool = False,
                                  generator: torch.Generator = None,
                                  split: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
                                  ) -> Tuple[Callable, Callable]:
    global counter
    B, N, _ = metric.shape
    if r <= 0:
        return do_nothing, do_nothing
    dev = metric.device
    with torch.no_grad():
        if split is not None:
            a_idx, b_idx = split
        else:
            rand_idx = None
            if not no_rand:
                if generator is None:
                    raise ValueError("a generator is required unless no_rand=True")
                tst, hsy, wsx = (t - 1) // st, h // sy, w // sx
                rand_idx = torch.randint(sy * sx * st, size=(tst, hsy, wsx, 1), device=generator.device,
                                         generator=generator)
            a_idx, b_idx = video_split(w, h, t, sx, sy, st, dev, rand_idx)
        m = metric if metric.dtype in (torch.bfloat16, torch.float16) else metric.to(torch.bfloat16)
        plan = kernels.tome_match(m, a_idx.to(dev), b_idx.to(dev), r)
        counter = plan.counter.to(torch.int64).unsqueeze(-1)
    state = {"shape4": None}

    def merge(x: torch.Tensor, mode: str = "mean") -> torch.Tensor:
        if mode != "mean":
            raise NotImplementedError("only the reference's 'mean' merge is provided")
        if x.dim() == 4:
            state["shape4"] = (x.shape[0], x.shape[1])
            x3 = x.reshape(B, x.shape[2], x.shape[3])
        else:
            x3 = x
        return kernels.tome_merge(x3, plan, text_len=x3.shape[1] - N)

    def unmerge(x: torch.Tensor) -> torch.Tensor:
        x3 = x.reshape(B, -1, x.shape[-1]) if x.dim() == 4 else x
        out = kernels.tome_unmerge(x3, plan, text_len=x3.shape[1] - plan.merged_len)
        if state["shape4"] is not None:
            b, hh = state["shape4"]
            return out.reshape(b, hh, -1, out.shape[-1])
        return out

    merge.plan = plan
    unmerge.plan = plan
    return merge, unmerge
