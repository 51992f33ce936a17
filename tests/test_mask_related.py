"""The special_attentions.utils.mask_related mirror on the CPU: its layout
helpers against the reference's own outputs (tests/golden/mask_layout.npz)
and its reachability through install_alias()."""
from pathlib import Path

import numpy as np
import pytest
import torch

from sparseattnfunctions_b200.special_attentions.utils import mask_related as mr

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_get_block_mask_matches_reference():
    d = np.load(GOLDEN / "mask_layout.npz")
    rs = np.random.RandomState(601)
    frame = torch.from_numpy(rs.rand(2, 30, 13, 13) < 0.4)
    inner = torch.from_numpy(rs.rand(2, 30, 22, 21) < 0.8)
    got = mr.get_block_mask(inner, frame)
    shape = tuple(d["block_shape"])
    assert tuple(got.shape) == shape and got.dtype == torch.float32
    ref = np.unpackbits(d["block_mask"])[:int(np.prod(shape))].reshape(shape).astype(bool)
    assert np.array_equal(got.numpy() != 0, ref)


def test_preprocess_query_layout_matches_reference():
    d = np.load(GOLDEN / "mask_layout.npz")
    idx = torch.arange(1, 17777, dtype=torch.float64).view(1, 1, 17776, 1)
    qp, kp, vp = mr.preprocess_qkv(idx, idx.clone(), idx.clone(), generator=torch.Generator().manual_seed(0))
    assert np.array_equal(qp.reshape(-1).numpy().astype(np.int32), d["q_processed"])
    assert np.array_equal(mr.reverse_process_out(qp).reshape(-1).numpy().astype(np.int32), d["q_back"])
    # k / v: 13 frames of 1344 consecutive tokens of their frame, then the text
    k = kp.reshape(-1).numpy().astype(np.int64)
    assert k.size == 13 * 1344 + 226
    frames = (k[:13 * 1344].reshape(13, 1344) - 227) // 1350
    assert np.array_equal(frames, np.repeat(np.arange(13)[:, None], 1344, axis=1))
    assert np.all(np.diff(k[:13 * 1344].reshape(13, 1344), axis=1) == 1)
    assert np.array_equal(k[13 * 1344:], np.arange(1, 227))


def test_inner_frame_mask_threshold_one_keeps_every_block():
    q = torch.zeros(2, 3, 10, 64)
    m = mr.get_inner_frame_mask(q, q)
    assert tuple(m.shape) == (2, 3, 22, 21) and bool(m.all())
    with pytest.raises(NotImplementedError):
        mr.get_inner_frame_mask(q, q, threshold=0.9)


def test_alias_resolves_mask_related():
    import importlib

    import sparseattnfunctions_b200

    sparseattnfunctions_b200.install_alias()
    mod = importlib.import_module("special_attentions.utils.mask_related")
    assert mod is mr
    for name in ("calc_attn_block_sum_efficient", "generate_attention_mask_frame_scope", "get_block_mask",
                 "get_inner_frame_mask", "preprocess_qkv", "reverse_process_out", "pad_to_multiple"):
        assert callable(getattr(mod, name))
