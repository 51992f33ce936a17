"""GPU parity of SildingTileAttention (padded tile layout on the block-sparse
kernel) against the CPU oracle (oracle/sta.py, pinned to the reference's
mask_mod and preprocess by tests/golden/sta_layout.npz): 2e-2 max-abs."""
import numpy as np
import pytest
import torch

from oracle import sta as osta
from sparseattnfunctions_b200 import kernels
from sparseattnfunctions_b200.special_attentions.SildingTileAttention import SildingTileAttention

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg,block", [
    (dict(img_size=(4, 6, 9), tile_size=(2, 3, 3), kernel_size=(1, 3, 3), text_length=10), 64),
    (dict(img_size=(4, 12, 15), tile_size=(4, 3, 3), kernel_size=(1, 3, 3), text_length=40), 128),
])
def test_sta_against_oracle(cuda_device, cfg, block):
    T, Hc, W = cfg["img_size"]
    S = cfg["text_length"] + T * Hc * W
    g = torch.Generator().manual_seed(S)
    q, k, v = (torch.randn(2, 2, S, 64, generator=g).to(torch.bfloat16) for _ in range(3))
    sta = SildingTileAttention(cfg, block=block)
    out = sta(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    ref = osta.sta_attention(q, k, v, cfg["img_size"], cfg["kernel_size"], cfg["tile_size"], cfg["text_length"])
    assert out.shape == q.shape
    assert np.abs(out.double().cpu().numpy() - ref).max() <= 2e-2


def test_permute_tokens_pads_with_zeros(cuda_device):
    x = torch.randn(1, 2, 10, 64, device=cuda_device).to(torch.bfloat16)
    perm = torch.tensor([3, -1, 0, 9, -1], dtype=torch.int32, device=cuda_device)
    out = kernels.permute_tokens(x, perm)
    assert out.shape == (1, 2, 5, 64)
    assert torch.equal(out[:, :, 0], x[:, :, 3]) and torch.equal(out[:, :, 3], x[:, :, 9])
    assert int(torch.count_nonzero(out[:, :, 1])) == 0 and int(torch.count_nonzero(out[:, :, 4])) == 0
