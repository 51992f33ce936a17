"""Torch-facing wrappers of the libsaf kernels.

Each function takes CUDA tensors, allocates its outputs (and workspace) with
the PyTorch caching allocator, enqueues the kernels on the current CUDA
stream of the tensors' device and returns without synchronising.  There is no
CPU path: CPU tensors raise ``ValueError``.

Block lists use a *segmented CSR* (see ``BlockCSR``): one CSR per head, all
heads in one ``col_idx`` buffer with a fixed per-head segment, so it can be
written without a device-wide prefix sum and read without a host sync.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.SAF_BF16, torch.float16: _lib.SAF_F16, torch.float32: _lib.SAF_F32}


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if not isinstance(t, torch.Tensor):
            raise TypeError("expected torch.Tensor arguments")
        if t.device.type != "cuda":
            raise ValueError("sparseattnfunctions_b200 kernels run on CUDA tensors only")
        if t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


def _stream_ptr(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _t4(x: torch.Tensor) -> _lib.Tensor4:
    if x.dim() != 4:
        raise ValueError(f"expected a [B, H, S, D] tensor, got shape {tuple(x.shape)}")
    if x.dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {x.dtype}")
    if x.stride(-1) != 1:
        raise ValueError("the last (D) dimension must be contiguous")
    t = _lib.Tensor4()
    t.data = x.data_ptr()
    t.dtype = _DTYPES[x.dtype]
    t.B, t.H, t.S, t.D = x.shape
    t.stride_b, t.stride_h, t.stride_s = x.stride(0), x.stride(1), x.stride(2)
    return t


def _d_last(x: torch.Tensor) -> torch.Tensor:
    return x if x.stride(-1) == 1 else x.contiguous()


@dataclass
class BlockCSR:
    """Live key blocks of every query block, per head.

    ``row_ptr``: int32 ``[B*H, nbq + 1]``, absolute offsets into ``col_idx``;
    head ``g``'s entries lie in ``[g*nbq*nbk, (g+1)*nbq*nbk)``.
    ``col_idx``: int32, capacity ``B*H*nbq*nbk``, ascending within a row.
    """

    row_ptr: torch.Tensor
    col_idx: torch.Tensor
    B: int
    H: int
    nbq: int
    nbk: int
    block_m: int
    block_n: int
    mask: Optional[torch.Tensor] = None    # uint8 [B, H, nbq, nbk] when requested
    scores: Optional[torch.Tensor] = None  # fp64 [B, H, nbq, nbk] when requested
    dense_rows: int = 0  # leading row blocks that are dense (scheduled first by bsa_fwd)

    def nnz_per_head(self) -> torch.Tensor:
        """Live blocks per head (device tensor, no sync)."""
        return self.row_ptr[:, -1] - self.row_ptr[:, 0]

    def to_dense(self) -> torch.Tensor:
        """Dense bool mask ``[B, H, nbq, nbk]`` rebuilt from the CSR (torch ops;
        for inspection and tests)."""
        rp = self.row_ptr.long()
        counts = (rp[:, 1:] - rp[:, :-1]).reshape(-1)
        rows = torch.repeat_interleave(torch.arange(counts.numel(), device=rp.device), counts)
        starts = rp[:, :-1].reshape(-1)
        first = torch.repeat_interleave(starts, counts)
        within = torch.arange(rows.numel(), device=rp.device) - torch.repeat_interleave(
            torch.cumsum(counts, 0) - counts, counts)
        cols = self.col_idx.long()[first + within]
        dense = torch.zeros(self.B * self.H * self.nbq, self.nbk, dtype=torch.bool, device=rp.device)
        dense[rows, cols] = True
        return dense.view(self.B, self.H, self.nbq, self.nbk)

    def live_flops(self, Sq: int, Sk: int, D: int) -> torch.Tensor:
        """Algorithmic FLOP of the live blocks: 4*D*sum(rows_i * cols_j) with
        the exact sizes of partial edge blocks (device tensor)."""
        dense = self.to_dense().double()
        rows = torch.full((self.nbq,), float(self.block_m), dtype=torch.float64, device=dense.device)
        rows[-1] = Sq - (self.nbq - 1) * self.block_m
        cols = torch.full((self.nbk,), float(self.block_n), dtype=torch.float64, device=dense.device)
        cols[-1] = Sk - (self.nbk - 1) * self.block_n
        return 4.0 * D * torch.einsum("bhij,i,j->", dense, rows, cols)


def pool_topk(q: torch.Tensor, k: torch.Tensor, *, block_m: int, block_n: int, topk: int,
              text_blocks_q: int = 0, text_blocks_k: int = 0, force_diag: bool = False,
              forced_inside_topk: bool = False, return_mask: bool = False,
              return_scores: bool = False) -> BlockCSR:
    """Block selection by mean-pooled scores (one launch sequence, no sync).

    Keeps, in every row block ``i >= text_blocks_q``, the ``topk`` columns of
    highest ``mean(q_block_i) . mean(k_block_j)`` (fp64; ties -> lower column; NaN
    ranks above every number, as torch.topk ranks it),
    plus the forced columns ``j < text_blocks_k`` (and ``j == i`` with
    ``force_diag``).  With ``forced_inside_topk`` the forced columns count
    toward ``topk``.  Rows ``i < text_blocks_q`` are dense.
    """
    dev = _require_cuda(q, k)
    q, k = _d_last(q), _d_last(k)
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    nbq, nbk = math.ceil(Sq / block_m), math.ceil(Sk / block_n)
    cfg = _lib.SelectCfg(block_m, block_n, topk, text_blocks_q, text_blocks_k, int(force_diag),
                         int(forced_inside_topk), 0)
    tq, tk = _t4(q), _t4(k)
    lib = _lib.load()
    ws_bytes = lib.saf_pool_topk_workspace_bytes(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(cfg))
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    row_ptr = torch.empty(B * H, nbq + 1, dtype=torch.int32, device=dev)
    col_idx = torch.empty(B * H * nbq * nbk, dtype=torch.int32, device=dev)
    mask = torch.empty(B, H, nbq, nbk, dtype=torch.uint8, device=dev) if return_mask else None
    scores = torch.empty(B, H, nbq, nbk, dtype=torch.float64, device=dev) if return_scores else None
    with torch.cuda.device(dev):
        rc = lib.saf_pool_topk(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(cfg),
                               row_ptr.data_ptr(), col_idx.data_ptr(),
                               mask.data_ptr() if mask is not None else None,
                               scores.data_ptr() if scores is not None else None,
                               ws.data_ptr(), ws.numel(), _stream_ptr(dev))
    _lib.check("saf_pool_topk", rc)
    return BlockCSR(row_ptr, col_idx, B, H, nbq, nbk, block_m, block_n, mask, scores,
                    dense_rows=min(text_blocks_q, nbq))


def energy_select(x: torch.Tensor, *, threshold: float, min_retain: int, max_retain: int,
                  text_blocks: int = 0, is_mass: bool = True, scale: float = 1.0, block_n: int = 0,
                  Sk: int = 0, return_mass: bool = False):
    """Energy-threshold block mask from ``x [B, H, nbq, nbk]`` (fp64 block
    mass when ``is_mass``, else mean-pooled scores turned into mass with
    ``scale``, ``block_n`` and ``Sk``).  Returns the uint8 mask
    ``[B, H, nbq, nbk]`` (and the fp64 mass used when ``return_mass``)."""
    dev = _require_cuda(x)
    if x.dim() != 4:
        raise ValueError("expected a [B, H, nbq, nbk] tensor")
    x = x.to(torch.float64).contiguous()
    B, H, nbq, nbk = x.shape
    mask = torch.empty(B, H, nbq, nbk, dtype=torch.uint8, device=dev)
    mass = torch.empty_like(x) if return_mass else None
    with torch.cuda.device(dev):
        rc = _lib.load().saf_energy_select(x.data_ptr(), int(is_mass), B * H, nbq, nbk, int(block_n), int(Sk),
                                           float(scale), float(threshold), int(min_retain), int(max_retain),
                                           int(text_blocks), mass.data_ptr() if mass is not None else None,
                                           mask.data_ptr(), _stream_ptr(dev))
    _lib.check("saf_energy_select", rc)
    return (mask, mass) if return_mass else mask


def topk_adaptive_select(x: torch.Tensor, *, init_k: int, text_blocks: int = 0, is_mass: bool = True,
                         scale: float = 1.0, block_n: int = 0, Sk: int = 0) -> torch.Tensor:
    """Adaptive top-k block mask from ``x [B, H, nbq, nbk]`` (the topk mode of
    ``transfer_attn_to_mask``): start from ``init_k`` blocks per row, grow
    rows under 60 % of the mass to 3x, then cut rows under 90 % to 2/3.
    Returns the uint8 mask ``[B, H, nbq, nbk]``."""
    dev = _require_cuda(x)
    if x.dim() != 4:
        raise ValueError("expected a [B, H, nbq, nbk] tensor")
    x = x.to(torch.float64).contiguous()
    B, H, nbq, nbk = x.shape
    mask = torch.empty(B, H, nbq, nbk, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.load().saf_topk_adaptive_select(x.data_ptr(), int(is_mass), B * H, nbq, nbk, int(block_n),
                                                  int(Sk), float(scale), int(init_k), int(text_blocks), None,
                                                  mask.data_ptr(), _stream_ptr(dev))
    _lib.check("saf_topk_adaptive_select", rc)
    return mask


def mask_to_csr(block_mask: torch.Tensor, block_m: int, block_n: int, dense_rows: int = 0) -> BlockCSR:
    """Dense boolean block mask ``[B, H, nbq, nbk]`` -> ``BlockCSR``.  ``dense_rows``
    tells ``bsa_fwd`` how many leading row blocks have the longest lists."""
    dev = _require_cuda(block_mask)
    if block_mask.dim() != 4:
        raise ValueError("block mask must be [B, H, nbq, nbk]")
    B, H, nbq, nbk = block_mask.shape
    m = block_mask
    if m.dtype == torch.bool:
        m = m.view(torch.uint8)
    elif m.dtype != torch.uint8:
        m = (m != 0).view(torch.uint8)
    if m.stride(-1) != 1 or m.stride(0) != H * m.stride(1):
        m = m.contiguous()
    row_ptr = torch.empty(B * H, nbq + 1, dtype=torch.int32, device=dev)
    col_idx = torch.empty(B * H * nbq * nbk, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.load().saf_mask_to_csr(m.data_ptr(), B * H, nbq, nbk, m.stride(1), m.stride(2),
                                         row_ptr.data_ptr(), col_idx.data_ptr(), _stream_ptr(dev))
    _lib.check("saf_mask_to_csr", rc)
    return BlockCSR(row_ptr, col_idx, B, H, nbq, nbk, block_m, block_n, dense_rows=dense_rows)


@dataclass
class FrameMask:
    """Per-head frame x frame visibility of a [text | frames x frame_len]
    sequence: ``bits`` int32 ``[B*H, frames]`` (bit f2 of word f1 set when
    video queries of frame f1 see the video keys of frame f2), ``mask`` uint8
    ``[B, H, frames, frames]`` and, when requested, the fp64 frame map."""

    bits: torch.Tensor
    mask: torch.Tensor
    map: Optional[torch.Tensor]
    text_len: int
    frames: int
    frame_len: int


def frame_mask(q: torch.Tensor, k: torch.Tensor, spatial: torch.Tensor, *, text_len: int, frames: int,
               frame_len: int, threshold: float = 0.9, sm_scale: float = 0.125,
               return_map: bool = False) -> FrameMask:
    """Frame-scope mask from the tokens sampled at every text position and at
    the ``spatial`` positions (int, in ``[0, frame_len)``) of every frame:
    the frame x frame attention map and the per-head energy rule of
    ``generate_attention_mask_frame_scope`` (saf_frame_mask)."""
    dev = _require_cuda(q, k)
    q, k = _d_last(q), _d_last(k)
    B, H, S, D = q.shape
    sp = spatial.to(device=dev, dtype=torch.int32).contiguous().reshape(-1)
    n = sp.numel()
    lib = _lib.load()
    ws_bytes = int(lib.saf_frame_mask_workspace_bytes(B * H, frames, n, text_len, D))
    ws = torch.empty(max(ws_bytes, 8), dtype=torch.uint8, device=dev)
    bits = torch.empty(B * H, frames, dtype=torch.int32, device=dev)
    mask = torch.empty(B, H, frames, frames, dtype=torch.uint8, device=dev)
    fmap = torch.empty(B, H, frames, frames, dtype=torch.float64, device=dev) if return_map else None
    tq, tk = _t4(q), _t4(k)
    with torch.cuda.device(dev):
        rc = lib.saf_frame_mask(ctypes.byref(tq), ctypes.byref(tk), sp.data_ptr(), n, text_len, frames,
                                frame_len, float(sm_scale), float(threshold), ws.data_ptr(), ws.numel(),
                                fmap.data_ptr() if fmap is not None else None, mask.data_ptr(),
                                bits.data_ptr(), _stream_ptr(dev))
    _lib.check("saf_frame_mask", rc)
    return FrameMask(bits, mask, fmap, text_len, frames, frame_len)


def frame_csr(fm: FrameMask, B: int, H: int, block_m: int = 128, block_n: int = 128) -> BlockCSR:
    """The key blocks each query block can touch under ``fm`` (saf_frame_csr)."""
    dev = _require_cuda(fm.bits)
    S = fm.text_len + fm.frames * fm.frame_len
    nbq, nbk = math.ceil(S / block_m), math.ceil(S / block_n)
    row_ptr = torch.empty(B * H, nbq + 1, dtype=torch.int32, device=dev)
    col_idx = torch.empty(B * H * nbq * nbk, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.load().saf_frame_csr(fm.bits.data_ptr(), B * H, fm.text_len, fm.frames, fm.frame_len, S,
                                       block_m, block_n, row_ptr.data_ptr(), col_idx.data_ptr(),
                                       _stream_ptr(dev))
    _lib.check("saf_frame_csr", rc)
    text_rows = min(nbq, math.ceil(fm.text_len / block_m))
    return BlockCSR(row_ptr, col_idx, B, H, nbq, nbk, block_m, block_n, dense_rows=text_rows)


def bsa_fwd_frames(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, csr: BlockCSR, fm: FrameMask,
                   sm_scale: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Block-sparse attention under the frame masks ``fm``: every visited
    block is masked to the keys the query row's frame may see
    (saf_bsa_fwd_frames)."""
    dev = _require_cuda(q, k, v, fm.bits)
    q, k, v = _d_last(q), _d_last(k), _d_last(v)
    B, H, Sq, D = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)} must match")
    if (csr.B, csr.H) != (B, H):
        raise ValueError("block list does not match q/k shapes")
    if out is None:
        out = torch.empty_like(q)
    tq, tk, tv, to = _t4(q), _t4(k), _t4(v), _t4(out)
    with torch.cuda.device(dev):
        rc = _lib.load().saf_bsa_fwd_frames(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(to),
                                            csr.row_ptr.data_ptr(), csr.col_idx.data_ptr(), csr.col_idx.numel(),
                                            csr.block_m, csr.block_n, fm.bits.data_ptr(), fm.text_len,
                                            fm.frames, fm.frame_len, float(sm_scale), int(csr.dense_rows),
                                            _stream_ptr(dev))
    _lib.check("saf_bsa_fwd_frames", rc)
    return out


def bsa_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, csr: BlockCSR, sm_scale: float,
            kv_bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
            row_ranges: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Block-sparse attention over the live blocks of ``csr``.

    ``kv_bias``: optional fp32 additive bias per key column, shape ``[Sk]``
    (shared by all heads), ``[B*H, Sk]`` or ``[B, H, Sk]`` / ``[B, H, 1, Sk]``;
    with 16-bit inputs it enters the scores through the tensor cores as
    ``bias / sm_scale`` rounded to the input type (the reference's attention
    mask is bf16 as well).
    ``row_ranges``: optional int32 ``[Sq, 4]`` -- query row r sees only the
    keys in ``[x, y) U [z, w)`` (frame-band masks; shared by all heads; not
    combinable with ``kv_bias``).
    """
    dev = _require_cuda(q, k, v)
    q, k, v = _d_last(q), _d_last(k), _d_last(v)
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    if k.shape[:2] != (B, H) or v.shape != k.shape or k.shape[3] != D:
        raise ValueError(f"q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)} do not match")
    if (csr.B, csr.H) != (B, H) or csr.nbq != math.ceil(Sq / csr.block_m) or \
            csr.nbk != math.ceil(Sk / csr.block_n):
        raise ValueError("block list does not match q/k shapes")
    if out is None:
        out = torch.empty_like(q)
    bias_ptr, bias_stride = None, 0
    if kv_bias is not None:
        _require_cuda(kv_bias)
        if kv_bias.dtype != torch.float32:
            raise ValueError("kv_bias must be float32")
        kb = kv_bias.reshape(-1, kv_bias.shape[-1])
        if kb.shape[-1] != Sk or kb.shape[0] not in (1, B * H):
            raise ValueError(f"kv_bias shape {tuple(kv_bias.shape)} does not match [B*H, Sk]")
        kb = kb.contiguous()
        kv_bias = kb  # keep alive for the launch
        bias_ptr = kb.data_ptr()
        bias_stride = 0 if kb.shape[0] == 1 else Sk
    rr_ptr = None
    if row_ranges is not None:
        _require_cuda(row_ranges)
        if row_ranges.dtype != torch.int32 or tuple(row_ranges.shape) != (Sq, 4) or \
                not row_ranges.is_contiguous():
            raise ValueError(f"row_ranges must be a contiguous int32 [{Sq}, 4] tensor")
        rr_ptr = row_ranges.data_ptr()
    tq, tk, tv, to = _t4(q), _t4(k), _t4(v), _t4(out)
    with torch.cuda.device(dev):
        rc = _lib.load().saf_bsa_fwd_ranges(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv),
                                            ctypes.byref(to), csr.row_ptr.data_ptr(),
                                            csr.col_idx.data_ptr(), csr.col_idx.numel(), csr.block_m,
                                            csr.block_n, bias_ptr, bias_stride, float(sm_scale),
                                            int(csr.dense_rows), rr_ptr, _stream_ptr(dev))
    _lib.check("saf_bsa_fwd", rc)
    return out


def bsa_fwd_pool(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, csr: BlockCSR, sm_scale: float,
                 pool_block: Optional[int] = None, out: Optional[torch.Tensor] = None):
    """Block-sparse attention plus the pooled attention map of
    ``attn_pooling_kernel.py``: returns ``(out, pool)`` with ``pool`` fp32
    ``[B, H, ceil(Sq / pool_block), nbk]``, entry (i, j) the largest
    normalised probability any query row of block i gives a key of block j
    (0 for blocks the row does not visit), each row divided by its sum.
    16-bit inputs; ``pool_block`` defaults to the key block size."""
    dev = _require_cuda(q, k, v)
    q, k, v = _d_last(q), _d_last(k), _d_last(v)
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    if k.shape[:2] != (B, H) or v.shape != k.shape or k.shape[3] != D:
        raise ValueError(f"q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)} do not match")
    if (csr.B, csr.H) != (B, H) or csr.nbq != math.ceil(Sq / csr.block_m) or \
            csr.nbk != math.ceil(Sk / csr.block_n):
        raise ValueError("block list does not match q/k shapes")
    pb = int(pool_block or csr.block_n)
    nbp = math.ceil(Sq / pb)
    if out is None:
        out = torch.empty_like(q)
    lib = _lib.load()
    ws_bytes = int(lib.saf_bsa_pool_workspace_bytes(B * H, Sq, csr.nbk))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    pool = torch.empty(B, H, nbp, csr.nbk, dtype=torch.float32, device=dev)
    tq, tk, tv, to = _t4(q), _t4(k), _t4(v), _t4(out)
    with torch.cuda.device(dev):
        rc = lib.saf_bsa_fwd_pool(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(to),
                                  csr.row_ptr.data_ptr(), csr.col_idx.data_ptr(), csr.col_idx.numel(),
                                  csr.block_m, csr.block_n, float(sm_scale), int(csr.dense_rows), pb,
                                  ws.data_ptr(), ws_bytes, pool.data_ptr(), _stream_ptr(dev))
    _lib.check("saf_bsa_fwd_pool", rc)
    return out, pool


def permute_tokens(x: torch.Tensor, perm: torch.Tensor, heads: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out[b, h, s] = x[b, h, perm[s]]`` for ``[B, H, S, D]`` tensors,
    ``s < len(perm)`` (``perm[s] == -1`` gives a zero row), for the flat heads
    ``b*H + h`` in ``heads`` (int32; all heads when None; other heads of
    ``out`` are left untouched)."""
    dev = _require_cuda(x, perm)
    x = _d_last(x)
    if x.dim() != 4 or x.dtype not in _DTYPES:
        raise ValueError("expected a [B, H, S, D] bf16 / f16 / f32 tensor")
    B, H, S, D = x.shape
    if perm.dtype != torch.int32 or perm.dim() != 1 or not perm.is_contiguous():
        raise ValueError("perm must be a contiguous 1-D int32 tensor")
    S_out = perm.numel()
    if out is None:
        out = torch.empty(B, H, S_out, D, dtype=x.dtype, device=dev)
    if tuple(out.shape) != (B, H, S_out, D) or out.dtype != x.dtype or out.stride(-1) != 1:
        raise ValueError(f"out must be [{B}, {H}, {S_out}, {D}] of x's dtype, D contiguous")
    hp, nh = None, 0
    if heads is not None:
        _require_cuda(heads)
        if heads.dtype != torch.int32 or not heads.is_contiguous():
            raise ValueError("heads must be a contiguous int32 tensor")
        hp, nh = heads.data_ptr(), heads.numel()
        if nh == 0:
            return out
    with torch.cuda.device(dev):
        rc = _lib.load().saf_permute_tokens(x.data_ptr(), out.data_ptr(), _DTYPES[x.dtype], B, H, S, S_out, D,
                                            x.stride(0), x.stride(1), x.stride(2), out.stride(0),
                                            out.stride(1), out.stride(2), perm.data_ptr(), hp, nh,
                                            _stream_ptr(dev))
    _lib.check("saf_permute_tokens", rc)
    return out


# --------------------------------------------------------------------------- ToMe

@dataclass
class TomePlan:
    """Result of a bipartite matching (see ``saf_tome_plan`` in saf_api.h).

    Positions refer to ``a_idx`` (src, length Ns) and ``b_idx`` (dst, length
    Nd), the video-token indices of the split.  ``token_map[b, t]`` is the row
    of the merged video sequence ``[unm | dst]`` that token ``t`` reads back
    on unmerge."""

    a_idx: torch.Tensor
    b_idx: torch.Tensor
    unm_idx: torch.Tensor
    src_idx: torch.Tensor
    dst_idx: torch.Tensor
    counter: torch.Tensor
    dst_ptr: torch.Tensor
    dst_src: torch.Tensor
    token_map: torch.Tensor
    log_count: torch.Tensor
    node_max: Optional[torch.Tensor]
    node_idx: Optional[torch.Tensor]
    B: int
    N: int
    r: int

    @property
    def Ns(self) -> int:
        return self.a_idx.numel()

    @property
    def Nd(self) -> int:
        return self.b_idx.numel()

    @property
    def merged_len(self) -> int:
        return self.Ns - self.r + self.Nd

    def _struct(self) -> _lib.TomePlan:
        ptr = lambda t: None if t is None else t.data_ptr()
        return _lib.TomePlan(ptr(self.unm_idx), ptr(self.src_idx), ptr(self.dst_idx),
                             ptr(self.counter), ptr(self.dst_ptr), ptr(self.dst_src),
                             ptr(self.token_map), ptr(self.log_count), ptr(self.node_max),
                             ptr(self.node_idx))


_T16 = {torch.bfloat16: _lib.SAF_BF16, torch.float16: _lib.SAF_F16}


def tome_match(metric: torch.Tensor, a_idx: torch.Tensor, b_idx: torch.Tensor, r: int,
               keep_node: bool = False) -> TomePlan:
    """Bipartite soft matching of ``metric [B, N, C]`` (bf16/f16, CUDA) between
    the src tokens ``a_idx`` and dst tokens ``b_idx`` (int32/int64 video-token
    indices on the same device); merges ``min(r, Ns)`` src tokens."""
    dev = _require_cuda(metric, a_idx, b_idx)
    if metric.dim() != 3 or metric.dtype not in _T16:
        raise ValueError("metric must be a bf16/f16 [B, N, C] CUDA tensor")
    if metric.stride(-1) != 1:
        metric = metric.contiguous()
    B, N, C = metric.shape
    a = a_idx.to(device=dev, dtype=torch.int32).contiguous().reshape(-1)
    b = b_idx.to(device=dev, dtype=torch.int32).contiguous().reshape(-1)
    Ns, Nd = a.numel(), b.numel()
    r = max(0, min(int(r), Ns))
    i32 = dict(dtype=torch.int32, device=dev)
    plan = TomePlan(
        a, b, torch.empty(B, Ns - r, **i32), torch.empty(B, r, **i32), torch.empty(B, r, **i32),
        torch.empty(B, Nd, **i32), torch.empty(B, Nd + 1, **i32), torch.empty(B, max(r, 1), **i32),
        torch.empty(B, N, **i32), torch.empty(B, Nd, dtype=torch.float32, device=dev),
        torch.empty(B, Ns, dtype=torch.float64, device=dev) if keep_node else None,
        torch.empty(B, Ns, **i32) if keep_node else None, B, N, r)
    lib = _lib.load()
    ws_bytes = lib.saf_tome_match_workspace_bytes(B, Ns, Nd, C, r)
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    st = plan._struct()
    with torch.cuda.device(dev):
        rc = lib.saf_tome_match(metric.data_ptr(), _T16[metric.dtype], B, N, C, metric.stride(0),
                                metric.stride(1), a.data_ptr(), Ns, b.data_ptr(), Nd, r,
                                ctypes.byref(st), ws.data_ptr(), ws.numel(), _stream_ptr(dev))
    _lib.check("saf_tome_match", rc)
    return plan


def tome_kv_metric(k: torch.Tensor, v: torch.Tensor, text_len: int) -> torch.Tensor:
    """MergeAttention's matching metric ``[k, |k|, v, |v|]`` of the video
    tokens (rows ``text_len..`` of ``[B, H, S, D]`` k / v) as
    ``[B*H, S - text_len, 2D + 2]``; norms from fp64 sums of squares."""
    dev = _require_cuda(k, v)
    k, v = _d_last(k), _d_last(v)
    if k.dtype not in _T16 or v.dtype != k.dtype:
        raise ValueError("k and v must be bf16 or f16 of the same dtype")
    B, H, S, D = k.shape
    out = torch.empty(B * H, S - text_len, 2 * D + 2, dtype=k.dtype, device=dev)
    tk, tv = _t4(k), _t4(v)
    with torch.cuda.device(dev):
        rc = _lib.load().saf_tome_kv_metric(ctypes.byref(tk), ctypes.byref(tv), int(text_len), out.data_ptr(),
                                            _stream_ptr(dev))
    _lib.check("saf_tome_kv_metric", rc)
    return out


def _rows3(x: torch.Tensor, B: int) -> torch.Tensor:
    """[B, rows, C] view of x; a 4-D [b, h, S, D] tensor with b*h == B is
    read as [b*h, S, D] (the per-head matching of MergeAttention)."""
    if x.dim() == 4 and x.shape[0] * x.shape[1] == B:
        x = x.reshape(B, x.shape[2], x.shape[3])
    if x.dim() != 3 or x.shape[0] != B:
        raise ValueError(f"tensor of shape {tuple(x.shape)} does not match the plan's batch {B}")
    return x if x.stride(-1) == 1 else x.contiguous()


def _rows_out(out, B, rows, like):
    if out is None:
        return torch.empty(B, rows, like.shape[-1], dtype=like.dtype, device=like.device)
    if tuple(out.shape) != (B, rows, like.shape[-1]) or out.dtype != like.dtype or out.stride(-1) != 1 \
            or out.device != like.device:
        raise ValueError(f"out must be a [{B}, {rows}, {like.shape[-1]}] {like.dtype} tensor on {like.device}")
    return out


def tome_merge(x: torch.Tensor, plan: TomePlan, text_len: int = 0,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x [B, text_len + N, C]`` -> ``[B, text_len + Ns - r + Nd, C]``."""
    dev = _require_cuda(x)
    x = _rows3(x, plan.B)
    if x.shape[1] != text_len + plan.N:
        raise ValueError(f"x has {x.shape[1]} rows, expected text_len + N = {text_len + plan.N}")
    out = _rows_out(out, plan.B, text_len + plan.merged_len, x)
    st = plan._struct()
    with torch.cuda.device(dev):
        rc = _lib.load().saf_tome_merge(x.data_ptr(), out.data_ptr(), _DTYPES[x.dtype], plan.B,
                                        x.shape[-1], x.stride(0), x.stride(1), out.stride(0),
                                        out.stride(1), text_len, plan.a_idx.data_ptr(), plan.Ns,
                                        plan.b_idx.data_ptr(), plan.Nd, plan.r, ctypes.byref(st),
                                        _stream_ptr(dev))
    _lib.check("saf_tome_merge", rc)
    return out


def tome_unmerge(y: torch.Tensor, plan: TomePlan, text_len: int = 0,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``y [B, text_len + Ns - r + Nd, C]`` -> ``[B, text_len + N, C]``."""
    dev = _require_cuda(y)
    y = _rows3(y, plan.B)
    if y.shape[1] != text_len + plan.merged_len:
        raise ValueError(f"y has {y.shape[1]} rows, expected {text_len + plan.merged_len}")
    out = _rows_out(out, plan.B, text_len + plan.N, y)
    with torch.cuda.device(dev):
        rc = _lib.load().saf_tome_unmerge(y.data_ptr(), out.data_ptr(), _DTYPES[y.dtype], plan.B,
                                          y.shape[-1], y.stride(0), y.stride(1), out.stride(0),
                                          out.stride(1), text_len, plan.N,
                                          plan.token_map.data_ptr(), _stream_ptr(dev))
    _lib.check("saf_tome_unmerge", rc)
    return out


# --------------------------------------------------------------------------- Ulysses layout

def head_split(H: int, P: int) -> list:
    """Contiguous head ranges of P peers, the first ``H % P`` one head larger
    (30 heads: 15,15 / 8,8,7,7 / 4,4,4,4,4,4,3,3).  Returns the P + 1 offsets."""
    if P < 1:
        raise ValueError("P must be >= 1")
    base, extra = divmod(H, P)
    off = [0]
    for j in range(P):
        off.append(off[-1] + base + (1 if j < extra else 0))
    return off


def _seq_args(tensors):
    x = tensors[0]
    if x.dim() != 4:
        raise ValueError("expected [B, s, H, D] tensors")
    for t in tensors[1:]:
        if t.shape != x.shape or t.stride() != x.stride() or t.dtype != x.dtype:
            raise ValueError("pack / unpack tensors must share shape, strides and dtype")
    if x.dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {x.dtype}")
    if x.stride(-1) != 1:
        raise ValueError("the last (D) dimension must be contiguous")
    return x


def ulysses_pack(tensors, head_off, buf: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Packs T sequence-sharded ``[B, s, H, D]`` tensors into the all-to-all
    send buffer (P chunks, chunk j = ``[s, B, T, h_j, D]``); returns it flat."""
    dev = _require_cuda(*tensors)
    x = _seq_args(tensors)
    B, s, H, D = x.shape
    T, P = len(tensors), len(head_off) - 1
    n = B * s * T * H * D
    if buf is None:
        buf = torch.empty(n, dtype=x.dtype, device=dev)
    elif buf.numel() < n or buf.dtype != x.dtype or not buf.is_contiguous():
        raise ValueError("send buffer too small, of another dtype or not contiguous")
    ptrs = (ctypes.c_void_p * T)(*[t.data_ptr() for t in tensors])
    offs = (ctypes.c_int32 * (P + 1))(*head_off)
    with torch.cuda.device(dev):
        rc = _lib.load().saf_ulysses_pack(ptrs, T, _DTYPES[x.dtype], B, s, H, D, x.stride(0), x.stride(1),
                                          x.stride(2), offs, P, buf.data_ptr(), _stream_ptr(dev))
    _lib.check("saf_ulysses_pack", rc)
    return buf


def ulysses_unpack(buf: torch.Tensor, outs, head_off) -> None:
    """Inverse of ``ulysses_pack``: scatters the P received chunks of ``buf``
    into the T sequence-sharded ``[B, s, H, D]`` tensors ``outs`` (in place)."""
    dev = _require_cuda(buf, *outs)
    x = _seq_args(outs)
    B, s, H, D = x.shape
    T, P = len(outs), len(head_off) - 1
    if buf.numel() < B * s * T * H * D or buf.dtype != x.dtype or not buf.is_contiguous():
        raise ValueError("receive buffer too small, of another dtype or not contiguous")
    ptrs = (ctypes.c_void_p * T)(*[t.data_ptr() for t in outs])
    offs = (ctypes.c_int32 * (P + 1))(*head_off)
    with torch.cuda.device(dev):
        rc = _lib.load().saf_ulysses_unpack(buf.data_ptr(), T, _DTYPES[x.dtype], B, s, H, D, x.stride(0),
                                            x.stride(1), x.stride(2), offs, P, ptrs, _stream_ptr(dev))
    _lib.check("saf_ulysses_unpack", rc)


def gather_rows(x: torch.Tensor, idx: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Row gather across batches: ``out[ob, h, s] = x[idx[ob, s] // Sx, h,
    idx[ob, s] % Sx]`` for ``x`` ``[Bx, H, Sx, D]`` and int64 ``idx``
    ``[Bo, So]`` (negative entries give zero rows); ``out`` ``[Bo, H, So, D]``
    may be a strided view (saf_gather_rows)."""
    dev = _require_cuda(x, idx)
    x = _d_last(x)
    if x.dim() != 4 or idx.dim() != 2 or idx.dtype != torch.int64:
        raise ValueError("expected x [B, H, S, D] and an int64 [Bo, So] index")
    idx = idx.contiguous()
    Bx, H, Sx, D = x.shape
    Bo, So = idx.shape
    if out is None:
        out = torch.empty(Bo, H, So, D, dtype=x.dtype, device=dev)
    elif tuple(out.shape) != (Bo, H, So, D) or out.dtype != x.dtype or out.stride(-1) != 1:
        raise ValueError(f"out must be a {x.dtype} [{Bo}, {H}, {So}, {D}] tensor with contiguous rows")
    with torch.cuda.device(dev):
        rc = _lib.load().saf_gather_rows(x.data_ptr(), _DTYPES[x.dtype], Bx, H, Sx, D, x.stride(0), x.stride(1),
                                         x.stride(2), out.data_ptr(), Bo, So, out.stride(0), out.stride(1),
                                         out.stride(2), idx.data_ptr(), _stream_ptr(dev))
    _lib.check("saf_gather_rows", rc)
    return out


def probe_mass(qs: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """Probe mass ``[B, Sk]`` fp64 of the sampled rows ``qs`` ``[B, H, R, 64]``
    over the keys ``k`` ``[B, H, Sk, 64]`` (both bf16 or both f16): the
    16-bit softmax probabilities of every sampled row summed over rows and
    heads, rounded as the reference's 16-bit matmul / softmax / sum
    (saf_probe_mass, tcgen05)."""
    dev = _require_cuda(qs, k)
    qs, k = _d_last(qs), _d_last(k)
    B, H, R, D = qs.shape
    Sk = k.shape[2]
    lib = _lib.load()
    ws_bytes = lib.saf_probe_workspace_bytes(B, H, Sk, R)
    ws = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device=dev)
    mass = torch.empty(B, Sk, dtype=torch.float64, device=dev)
    tq, tk = _t4(qs), _t4(k)
    with torch.cuda.device(dev):
        rc = lib.saf_probe_mass(ctypes.byref(tq), ctypes.byref(tk), ws.data_ptr(), ws.numel(), mass.data_ptr(),
                                _stream_ptr(dev))
    _lib.check("saf_probe_mass", rc)
    return mass


def masked_topn(mass: torch.Tensor, local_mask: torch.Tensor, n: int) -> torch.Tensor:
    """int32 ``[P * B, n]``: row ``p * B + b`` lists, ascending, the n keys of
    largest ``mass[b]`` outside ``local_mask[p]`` (ties to the lower key)
    (saf_masked_topn)."""
    dev = _require_cuda(mass, local_mask)
    if mass.dtype != torch.float64 or mass.dim() != 2:
        raise ValueError("mass must be a float64 [B, Sk] tensor")
    if local_mask.dim() != 2 or local_mask.shape[1] != mass.shape[1]:
        raise ValueError("local_mask must be [P, Sk]")
    mass = mass.contiguous()
    lm = local_mask.to(torch.uint8).contiguous()
    B, Sk = mass.shape
    P = lm.shape[0]
    out = torch.empty(P * B, n, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.load().saf_masked_topn(mass.data_ptr(), lm.data_ptr(), B, P, Sk, int(n), out.data_ptr(),
                                         _stream_ptr(dev))
    _lib.check("saf_masked_topn", rc)
    return out


def bsa_fwd_keys(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, key_list: torch.Tensor,
                 key_batch: torch.Tensor, sm_scale: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention of q ``[Bq, H, Sq, 64]`` over per-batch key lists: batch b
    attends the rows ``key_list[b]`` (int32 ``[Bq, L]``) of
    ``k[key_batch[b]]`` / ``v[key_batch[b]]`` (``[B_src, H, S_src, 64]``,
    contiguous), repeated keys counted as often as listed; the rows are
    fetched by TMA gather4 loads inside the attention kernel
    (saf_bsa_fwd_keys)."""
    dev = _require_cuda(q, k, v, key_list, key_batch)
    q = _d_last(q)
    k, v = k.contiguous(), v.contiguous()
    if key_list.dim() != 2 or key_list.shape[0] != q.shape[0]:
        raise ValueError(f"key_list must be [{q.shape[0]}, L]")
    kl = key_list.to(torch.int32).contiguous()
    kb = key_batch.to(torch.int32).contiguous()
    if kb.numel() != q.shape[0]:
        raise ValueError(f"key_batch must have {q.shape[0]} entries")
    if out is None:
        out = torch.empty_like(q)
    tq, tk, tv, to = _t4(q), _t4(k), _t4(v), _t4(out)
    with torch.cuda.device(dev):
        rc = _lib.load().saf_bsa_fwd_keys(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(to),
                                          kl.data_ptr(), kl.shape[1], kb.data_ptr(), float(sm_scale),
                                          _stream_ptr(dev))
    _lib.check("saf_bsa_fwd_keys", rc)
    return out

