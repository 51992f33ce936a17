"""Drop-in for special_attentions/LocalGlobalAttention.py.

The reference processor (LocalGlobalAttention.py:183-259) serves one
CogVideoX-2B layer shape (226 text tokens, 13 x 30 x 45 video, B = 2):

* the text rows and the rows of frame 0 (the first 226 + 1350) attend every
  key (slice_text / attention_text, :193-205);
* the video rows of frames 1-12 are cut into 18 patches of 6 x 10 x 15
  tokens (transform_q, :212-217); patch p of batch b attends its key list:
  the keys of a static window mask around the patch (get_mask, :114-179:
  text, frame 0 and a padded spatio-temporal box), cut to the first patch's
  key count in the order of a descending sort of the mask, followed by the
  ``int(0.05 S) + 1`` keys of largest probe mass outside the window
  (transform_kv_v1, :219-238);
* the probe mass (probe_solver._probe_num, :50-62) is the softmax over all
  keys of 1280 randomly sampled video query rows, summed over the sampled
  rows and the heads; it is recomputed every ``update_gap`` calls of the
  module-wide ``counter`` and whenever an instance has none yet.

Here the dense rows run on the block-sparse attention kernel with every
block live (written straight into the output rows), the probe is the
tcgen05 probe kernel (the reference's 16-bit roundings reproduced) plus the
masked top-n select, and the patch step gathers the patch rows of q and
every (patch, batch) key list of k / v once (duplicates included, as the
reference's torch.gather), runs the attention kernel over the gathered rows
and gathers the outputs back into token order.  With
``gather_in_kernel=True`` the attention kernel's key-list mode fetches the
listed k / v rows by TMA gather4 loads instead, with no gathered copy in
HBM (less memory, but slower at this size).
The sampled rows are drawn with the same ``torch.randint`` call as the
reference, and the window key lists come from the same ``torch.sort`` of
the window mask on the input's device, so both match the reference's on
the same device and generator state.

Not mirrored: ``ZipVLAttention`` (its forward reads ``self.device`` and
calls ``self._probe``, which the reference class does not define, so it
cannot run) -- ``probe_solver._probe_score`` is, on the probe kernel.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .. import kernels

video_shape = [13, 30, 45]
patch_shape = [6, 10, 15]
batch_size = 2
compression = torch.tensor([2, 3, 3], dtype=torch.int32)
sample_num = 1280
padding = [0.2, 0.1, 0.1]
percentile = 0.05
update_gap = 5
TEXT_LEN = 226

counter = 0


def _window_mask() -> torch.Tensor:
    """bool [18, 17776]: the reference's mask_fn (:120-163) per patch, in
    float32 as the reference evaluates it."""
    T, Hh, W = video_shape
    S = TEXT_LEN + T * Hh * W
    n_patch = int(torch.prod(compression).item())
    kv = torch.arange(S, dtype=torch.int64)
    sh = kv - TEXT_LEN
    w_idx = torch.remainder(sh, W).to(torch.float32)
    h_idx = torch.remainder(torch.div(sh, W, rounding_mode="floor"), Hh).to(torch.float32)
    t_idx = torch.div(sh, Hh * W, rounding_mode="floor")
    t_f = t_idx.to(torch.float32)
    pad = torch.tensor([video_shape[i] * padding[i] for i in range(3)], dtype=torch.float32)
    lo = torch.tensor([1, 0, 0], dtype=torch.float32)
    hi = torch.tensor(video_shape, dtype=torch.float32)
    gap = torch.tensor(patch_shape, dtype=torch.float32)
    c0, c1, c2 = (int(x) for x in compression)
    out = torch.empty(n_patch, S, dtype=torch.bool)
    for p in range(n_patch):
        nw, nh, nt = p % c2, (p // c2) % c1, (p // (c2 * c1)) % c0
        start = torch.tensor([nt * patch_shape[0] + 1, nh * patch_shape[1], nw * patch_shape[2]],
                             dtype=torch.float32) - pad
        start = torch.clamp(start, lo, hi)
        end = torch.clamp(start + gap + pad * 2, lo, hi)
        start = end - gap - pad * 2
        inside = ((w_idx >= start[2]) & (w_idx < end[2]) & (h_idx >= start[1]) & (h_idx < end[1]) &
                  (t_f >= start[0]) & (t_f < end[0]))
        out[p] = (kv < TEXT_LEN) | inside | (t_idx == 0)
    return out


_MASKS = {}


def get_mask(device: Optional[torch.device] = None):
    """(mask [36, 17776] bool, indices [36, remain_num] int64) as the
    reference's get_mask (:114-179): rows p * 2 + b, the indices the first
    remain_num entries of a descending sort of the mask (torch.sort on
    ``device``, as the reference sorts on its CUDA device)."""
    dev = torch.device(device) if device is not None else (
        torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
    if dev not in _MASKS:
        mask = _window_mask().repeat_interleave(batch_size, dim=0).to(dev)
        remain_num = int(mask[0].sum().item())
        _, indices = torch.sort(mask.to(torch.float16), descending=True)
        _MASKS[dev] = (mask, indices[:, :remain_num].contiguous())
    return _MASKS[dev]


def __getattr__(name):
    # the reference builds these at import; here on first use
    if name == "LocalGlobalAttention_Mask":
        return get_mask()[0]
    if name == "LocalGlobalAttention_Indices":
        return get_mask()[1]
    raise AttributeError(name)


class probe_solver:
    """probe_solver of the reference (:21-84) on the probe kernel."""

    def __init__(self, percentile=0.95, sample_num=256, device=None, type="num", mask=None):
        self.type = type
        self.compression_num = torch.prod(compression)
        self.percentile = percentile
        self.sample_num = sample_num
        self.device = device
        self.mask = mask

    def _sample_q(self, q_proj):
        B, H, N, _ = q_proj.shape
        return torch.randint(0, N, (B, 1, self.sample_num), device=q_proj.device)

    def _gather_samples(self, q_proj, indices):
        B, H, N, D = q_proj.shape
        base = torch.arange(B, device=q_proj.device, dtype=torch.int64).view(B, 1) * N
        return kernels.gather_rows(q_proj, indices.view(B, -1).to(torch.int64) + base)

    def _probe(self, q_proj, k_proj):
        if self.type == "num":
            return self._probe_num(q_proj, k_proj)
        elif self.type == "score":
            return self._probe_score(q_proj, k_proj)
        raise ValueError(f"Invalid type: {self.type}")

    def _mass(self, q_proj, k_proj):
        qs = self._gather_samples(q_proj, self._sample_q(q_proj))
        return kernels.probe_mass(qs, k_proj)  # [B, S] fp64, 16-bit values

    def _probe_num(self, q_proj, k_proj):
        """int64 [compression_num * B, int(percentile * S) + 1]: per row
        p * B + b the keys of largest probe mass of batch b outside mask row
        p * B + b, ascending (the reference lists them by descending mass;
        the attention over the gathered keys does not depend on the order)."""
        if self.percentile == 0:
            return None
        mass = self._mass(q_proj, k_proj)
        B, S = mass.shape
        n = int(self.percentile * S) + 1
        n_patch = int(self.compression_num.item())
        lmask = self.mask.view(n_patch, -1, S)[:, 0]  # every batch row of a patch is the same
        return kernels.masked_topn(mass, lmask, n).to(torch.int64)

    def _probe_score(self, q_proj, k_proj):
        """Per batch, the keys of largest mass up to a cumulative share of
        ``percentile`` (:64-84), in descending mass order."""
        mass = self._mass(q_proj, k_proj).to(q_proj.dtype)
        H, n = q_proj.shape[1], self.sample_num
        out = []
        for b in range(mass.shape[0]):
            values, indices = torch.sort(mass[b:b + 1], descending=True)
            values = (values / (H * n)).reshape(-1)
            cum = values.cumsum(dim=-1)
            cutoff = torch.searchsorted(cum, self.percentile)
            out.append(indices.reshape(-1)[:cutoff + 1])
        return out


class LocalGlobalAttention:
    def __init__(self, gather_in_kernel: bool = False):
        # gather_in_kernel: attend the key lists with the rows fetched inside
        # the attention kernel (no 2 x 0.98 GB of gathered k / v in HBM) --
        # measured slower than gathering first at CogVideoX-2B size (4.9
        # against 0.94 + 2.7 ms), so off by default
        self.gather_in_kernel = gather_in_kernel
        self.compression = compression.to(dtype=torch.int32)
        self.global_indices = None
        self.padding = 0.2
        self.max_dim = torch.tensor(video_shape, dtype=torch.int32)
        self.batch_size = batch_size
        self.mask = self.indices = None
        self.probe = None
        self._csr = {}
        self._idx = {}

    def _setup(self, device):
        if self.mask is None or self.mask.device != device:
            self.mask, self.indices = get_mask(device)
            self.probe = probe_solver(percentile=percentile, sample_num=sample_num, device=device, type="num",
                                      mask=self.mask)
            self.global_indices = None

    def _dense_csr(self, B, H, Sq, Sk, dev):
        key = (B, H, Sq, Sk, dev)
        if key not in self._csr:
            nbq, nbk = math.ceil(Sq / 128), math.ceil(Sk / 128)
            self._csr[key] = kernels.mask_to_csr(torch.ones(B, H, nbq, nbk, dtype=torch.bool, device=dev), 128, 128)
        return self._csr[key]

    def _patch_index(self, B, dev):
        """(q rows [P*B, 900] as b*S + token, output map [B, 16200] as
        (p*B + b)*900 + position), both int64."""
        key = (B, dev)
        if key not in self._idx:
            T, Hh, W = video_shape
            S = TEXT_LEN + T * Hh * W
            c0, c1, c2 = (int(x) for x in self.compression)
            tp, hp, wp = patch_shape
            n_patch = c0 * c1 * c2
            pos = torch.arange(tp * hp * wp)
            t_in, h_in, w_in = pos // (hp * wp), (pos // wp) % hp, pos % wp
            rows = []
            for p in range(n_patch):
                nw, nh, nt = p % c2, (p // c2) % c1, p // (c2 * c1)
                rows.append(TEXT_LEN + (1 + nt * tp + t_in) * (Hh * W) + (nh * hp + h_in) * W + nw * wp + w_in)
            rows = torch.stack(rows)  # [P, 900] token index
            b = torch.arange(B).view(1, B, 1)
            q_idx = (b * S + rows.view(n_patch, 1, -1)).reshape(n_patch * B, -1)
            dense = TEXT_LEN + W * Hh
            out_map = torch.empty(B, S - dense, dtype=torch.int64)
            src = (torch.arange(n_patch).view(n_patch, 1, 1) * B + b) * rows.shape[1] + pos.view(1, 1, -1)
            out_map[:, (rows - dense).view(-1)] = src.permute(1, 0, 2).reshape(B, -1)
            self._idx[key] = (q_idx.to(dev), out_map.to(dev))
        return self._idx[key]

    # ---- the reference's steps -------------------------------------------
    def slice_text(self, q):
        return q[:, :, :TEXT_LEN + video_shape[1] * video_shape[2], :]

    def slice_video(self, q):
        return q[:, :, TEXT_LEN + video_shape[1] * video_shape[2]:, :]

    def attention_text(self, q_text, k, v, out=None):
        B, H, Sq, D = q_text.shape
        csr = self._dense_csr(B, H, Sq, k.shape[2], q_text.device)
        return kernels.bsa_fwd(q_text, k, v, csr, 1.0 / math.sqrt(D), out=out)

    def attention_video(self, q_video, k, v):
        return self.attention_text(q_video, k, v)

    def transform_q(self, q):
        """[B, H, 17776, D] -> [(nt nh nw b), H, 900, D] (the patch rows of the
        full sequence)."""
        q_idx, _ = self._patch_index(q.shape[0], q.device)
        return kernels.gather_rows(q, q_idx)

    def patch_keys(self, q_video, k):
        """(keys int32 [P*B, L], source batch int32 [P*B]): the key list of
        every (patch, batch) row -- the window list then the probe's keys --
        and the batch of k / v it indexes; runs the probe on the reference's
        update_gap schedule (:221-226)."""
        global counter
        self._setup(k.device)
        if counter == 0 or self.global_indices is None:
            self.global_indices = self.probe._probe(q_video, k)
            counter = update_gap
        counter -= 1
        B = k.shape[0]
        n_patch = int(torch.prod(self.compression).item())
        # the window lists: row p * 2 + b of the reference's [36, remain] table
        fixed = self.indices.view(n_patch, batch_size, -1)
        fixed = fixed[:, [b if B == batch_size else 0 for b in range(B)]].reshape(n_patch * B, -1)
        lists = fixed if self.global_indices is None else torch.cat((fixed, self.global_indices), dim=-1)
        src = torch.arange(B, device=k.device, dtype=torch.int32).repeat(n_patch)
        return lists.to(torch.int32), src

    def key_lists(self, q_video, k):
        """int64 [P*B, L]: every (patch, batch) row's key list as b*S + key
        (the flattened rows saf_gather_rows reads)."""
        keys, src = self.patch_keys(q_video, k)
        return keys.to(torch.int64) + src.to(torch.int64).view(-1, 1) * k.shape[2]

    def transform_kv_v1(self, q, k, v):
        """The gathered k / v of every (patch, batch) list, as the reference
        builds them (the forward does not materialise them: the attention
        kernel reads the listed rows in place)."""
        idx = self.key_lists(q, k)
        return kernels.gather_rows(k, idx), kernels.gather_rows(v, idx)

    def transform_output(self, output, out=None):
        _, out_map = self._patch_index(output.shape[0] // int(torch.prod(self.compression).item()),
                                       output.device)
        return kernels.gather_rows(output, out_map, out=out)

    def forward(self, q, k, v):
        B, H, S, D = q.shape
        T, Hh, W = video_shape
        if S != TEXT_LEN + T * Hh * W or k.shape != q.shape or v.shape != q.shape:
            raise ValueError(f"LocalGlobalAttention serves [B, H, {TEXT_LEN + T * Hh * W}, D] inputs, "
                             f"got q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}")
        if q.dtype not in (torch.bfloat16, torch.float16) or D != 64:
            raise NotImplementedError("LocalGlobalAttention runs 16-bit inputs with head dim 64")
        self._setup(q.device)
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
        dense = TEXT_LEN + Hh * W
        self.attention_text(self.slice_text(q), k, v, out=out[:, :, :dense])
        qp = self.transform_q(q)
        if self.gather_in_kernel:
            keys, src = self.patch_keys(self.slice_video(q), k)
            op = kernels.bsa_fwd_keys(qp, k, v, keys, src, 1.0 / math.sqrt(D))
        else:
            kp, vp = self.transform_kv_v1(self.slice_video(q), k, v)
            op = self.attention_video(qp, kp, vp)
        self.transform_output(op, out=out[:, :, dense:])
        return out

    def __call__(self, q, k, v):
        return self.forward(q, k, v)
