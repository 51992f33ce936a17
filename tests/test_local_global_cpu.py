"""LocalGlobalAttention on the CPU: the oracle against the reference's own
outputs (tests/golden/local_global.npz, made by tests/golden/make_golden.py
from the reference's get_mask and probe_solver._probe_num), and the
mirror's host-side layout (window mask, patch rows, output map) against the
oracle.  No kernel runs here."""
import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import local_global as olg

GOLDEN = Path(__file__).resolve().parent / "golden"
_spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
mg = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(mg)


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN / "local_global.npz")


def test_window_mask_matches_reference(gold):
    shape = tuple(gold["mask_shape"])
    ref = np.unpackbits(gold["mask"])[:int(np.prod(shape))].reshape(shape).astype(bool)
    mine = olg.local_mask()
    assert np.array_equal(ref, np.repeat(mine, 2, axis=0))  # reference rows p * 2 + b
    assert int(gold["remain"]) == int(mine[0].sum()) == 6184
    # the keys after the window keys: none for the first frame group, 384
    # outside the window for the second (the reference's CPU sort picks
    # them in its own tie order; the GPU check pins the device's choice)
    off = gold["fill_off"]
    for r in range(36):
        fill = gold["fill_keys"][off[r]:off[r + 1]]
        p = r // 2
        assert fill.size == 6184 - int(mine[p].sum())
        assert not mine[p][fill].any()
    wl = olg.window_lists(mine)
    assert wl.shape == (18, 6184)
    for p in range(18):
        assert np.array_equal(np.sort(wl[p][:int(mine[p].sum())]), np.nonzero(mine[p])[0])


def test_probe_mass_matches_reference(gold):
    cfg = mg.LG_PROBE
    q, k = mg.lg_probe_inputs(cfg["seed"], cfg["H"], cfg["n_video"], cfg["S"], cfg["D"])
    mass = olg.probe_mass(q, k, gold["samples"], row_offset=0)
    ref = gold["att_probs"].astype(np.float64)
    # 16-bit sums: equal except where fp32 rounding of a sum lands on the
    # other side of a bf16 rounding boundary (then one bf16 ulp apart)
    diff = mass != ref
    assert diff.sum() <= 4, diff.sum()
    assert np.all(np.abs(mass - ref)[diff] <= np.abs(ref[diff]) * 2.0 ** -7)


def test_probe_selection_matches_reference_up_to_ties(gold):
    """The reference's indices against the stable top-n of the reference's
    own mass: every difference is a key tied at the n-th value (the
    reference's CPU sort is not stable; the GPU's is pinned on the GPU)."""
    ref = gold["att_probs"].astype(np.float64)
    lmask = olg.local_mask()
    n = int(0.05 * 17776) + 1
    assert n == olg.N_GLOBAL
    mine = olg.global_keys(ref, lmask, n)
    ri = gold["probe_indices"].astype(np.int64)
    assert ri.shape == (36, n)
    for r in range(36):
        p, b = divmod(r, 2)
        v = np.where(lmask[p], -np.inf, ref[b])
        thr = np.sort(v)[::-1][n - 1]
        sym = set(ri[r].tolist()) ^ set(mine[r].tolist())
        assert all(v[x] == thr for x in sym)
        assert len(set(ri[r].tolist())) == n


def test_mirror_layout_matches_oracle():
    from sparseattnfunctions_b200.special_attentions import LocalGlobalAttention as lga

    wm = lga._window_mask().numpy()
    assert np.array_equal(wm, olg.local_mask())
    mask, idx = lga.get_mask(torch.device("cpu"))
    assert tuple(mask.shape) == (36, 17776) and tuple(idx.shape) == (36, 6184)
    obj = lga.LocalGlobalAttention()
    q_idx, out_map = obj._patch_index(2, torch.device("cpu"))
    S = 17776
    for p in (0, 7, 17):
        for b in (0, 1):
            assert np.array_equal(q_idx[p * 2 + b].numpy(), b * S + olg.patch_rows(p))
    # the output map inverts the patch gather
    flat = q_idx.view(18, 2, 900).permute(1, 0, 2).reshape(2, -1)
    for b in (0, 1):
        src = out_map[b].numpy()
        rows = flat[b].numpy() - b * S - olg.DENSE_ROWS
        pos = np.empty(16200, dtype=np.int64)
        pos[rows] = np.arange(16200)
        p_of, within = np.divmod(src, 900)
        assert np.array_equal(p_of % 2, np.full(16200, b))
        assert np.array_equal((p_of // 2) * 900 + within, pos)


def test_alias_resolves_local_global():
    import importlib

    import sparseattnfunctions_b200

    sparseattnfunctions_b200.install_alias()
    mod = importlib.import_module("special_attentions.LocalGlobalAttention")
    assert hasattr(mod, "LocalGlobalAttention") and hasattr(mod, "probe_solver")
    assert mod.update_gap == 5 and mod.sample_num == 1280 and mod.percentile == 0.05
