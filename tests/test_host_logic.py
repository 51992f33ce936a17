"""Host-side layout logic on the CPU, against the oracle: the frame-band key
intervals and token orders of SmartAttention, the padded tile layout of
SildingTileAttention, the Ulysses head split, and the product path's refusal
of CPU tensors (there is no CPU fallback)."""
import math

import numpy as np
import pytest
import torch

from oracle import smart as osmart
from oracle import sta as osta
from sparseattnfunctions_b200 import kernels
from sparseattnfunctions_b200.geometry import VideoGeometry, frame_band_ranges, ranges_block_mask, \
    video_token_perm
from sparseattnfunctions_b200.special_attentions.SildingTileAttention import sta_layout


@pytest.mark.parametrize("diag", [1, 2])
def test_frame_band_ranges_match_the_band_mask(diag):
    geo = VideoGeometry(13, 6, 4, 5)  # 13 text tokens, 6 frames of 20
    r = frame_band_ranges(geo, diag=diag)
    got = osmart.ranges_mask(r.numpy(), geo.seq_len)
    want = osmart.band_mask(geo.text_len, geo.frames, geo.frame_len, diag)
    assert np.array_equal(got, want)


def test_ranges_block_mask_covers_exactly_the_visible_blocks():
    geo = VideoGeometry(13, 6, 4, 5)
    r = frame_band_ranges(geo)
    S, bm, bn = geo.seq_len, 16, 32
    dense = osmart.ranges_mask(r.numpy(), S)
    nbq, nbk = math.ceil(S / bm), math.ceil(S / bn)
    want = np.zeros((nbq, nbk), dtype=bool)
    for i in range(nbq):
        for j in range(nbk):
            want[i, j] = dense[i * bm:(i + 1) * bm, j * bn:(j + 1) * bn].any()
    assert np.array_equal(ranges_block_mask(r, S, bm, bn).numpy(), want)


def test_video_token_perm_is_process_and_process_back():
    geo = VideoGeometry(7, 3, 4, 5)
    perm, inv = video_token_perm(geo)
    operm, oinv = osmart.token_order(geo.text_len, geo.frames, geo.height, geo.width)
    assert np.array_equal(perm.numpy(), operm) and np.array_equal(inv.numpy(), oinv)


def test_sta_layout_matches_the_tile_window_mask():
    cfg = {"kernel_size": (1, 3, 3), "tile_size": (2, 3, 3), "img_size": (4, 9, 9), "text_length": 20}
    bs = 32
    pad_perm, unpad_perm, bias, mask = sta_layout(cfg, block=bs)
    T, Hc, W = cfg["img_size"]
    L = cfg["text_length"]
    n_tile = 18
    tiles = (T // 2) * (Hc // 3) * (W // 3)
    tb = math.ceil(L / bs)
    order = osta.token_order(cfg["img_size"], cfg["tile_size"], L)
    # every real token sits at its tile's block, in the reference's order
    real = pad_perm.numpy() >= 0
    assert np.array_equal(pad_perm.numpy()[real], order)
    assert np.array_equal(pad_perm.numpy()[unpad_perm.numpy()], np.arange(L + T * Hc * W))
    assert np.all(np.isneginf(bias.numpy()[~real])) and np.all(bias.numpy()[real] == 0)
    # block mask: text rows and columns dense, video tiles by the oracle's window
    m = osta.sta_mask(cfg["img_size"], cfg["kernel_size"], cfg["tile_size"], L)
    win = np.array([[m[L + a * n_tile, L + b * n_tile] for b in range(tiles)] for a in range(tiles)])
    got = mask.numpy()
    assert got[:tb].all() and got[:, :tb].all()
    assert np.array_equal(got[tb:, tb:], win)


@pytest.mark.parametrize("P,want", [(1, [30]), (2, [15, 15]), (4, [8, 8, 7, 7]), (8, [4, 4, 4, 4, 4, 4, 3, 3])])
def test_head_split(P, want):
    off = kernels.head_split(30, P)
    assert off[0] == 0 and off[-1] == 30 and list(np.diff(off)) == want


def test_cpu_tensors_are_refused():
    q = torch.zeros(1, 1, 128, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        kernels.pool_topk(q, q, block_m=128, block_n=128, topk=1)


def test_video_split_is_the_stable_argsort_partition():
    """merge_unmerge.py:52-67 orders the video tokens by a stable argsort of
    a {-1 (dst), 0 (src)} buffer; the mirror's prefix-count partition gives
    the same (a_idx, b_idx) for random and fixed dst picks, with and
    without a ragged border."""
    import torch

    from sparseattnfunctions_b200.special_attentions.utils import merge_unmerge as mu

    def by_argsort(w, h, t, sx, sy, st, rand_idx):
        tt = t - 1
        hsy, wsx, tst = h // sy, w // sx, tt // st
        if rand_idx is None:
            rand_idx = torch.zeros(tst, hsy, wsx, 1, dtype=torch.int64)
        buf = torch.zeros(tst, hsy, wsx, st * sy * sx, dtype=torch.int64)
        buf.scatter_(3, rand_idx.reshape(tst, hsy, wsx, 1), -torch.ones(tst, hsy, wsx, 1, dtype=torch.int64))
        buf = buf.view(tst, hsy, wsx, st, sy, sx).permute(0, 3, 1, 4, 2, 5).reshape(tst * st, hsy * sy, wsx * sx)
        full = torch.zeros(tt, h, w, dtype=torch.int64)
        full[:tst * st, :hsy * sy, :wsx * sx] = buf
        order = torch.argsort(full.reshape(-1), stable=True) + w * h
        n_dst = tst * hsy * wsx
        return order[n_dst:].to(torch.int32), torch.cat([torch.arange(w * h), order[:n_dst]]).to(torch.int32)

    g = torch.Generator().manual_seed(0)
    for w, h, t, sx, sy, st in [(45, 30, 13, 2, 2, 1), (45, 30, 13, 3, 2, 2), (7, 5, 4, 2, 2, 1), (9, 9, 6, 2, 3, 2)]:
        tst, hsy, wsx = (t - 1) // st, h // sy, w // sx
        for rnd in (None, torch.randint(st * sy * sx, (tst, hsy, wsx, 1), generator=g)):
            a_ref, b_ref = by_argsort(w, h, t, sx, sy, st, rnd)
            a, b = mu.video_split(w, h, t, sx, sy, st, "cpu", rnd)
            assert torch.equal(a, a_ref) and torch.equal(b, b_ref)
