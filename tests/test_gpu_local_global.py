"""LocalGlobalAttention on the GPU (special_attentions/LocalGlobalAttention.py
of the reference) against the CPU oracle (oracle/local_global.py, itself
pinned to the reference's get_mask and probe_solver._probe_num by
tests/golden/local_global.npz).

* saf_gather_rows: bit-exact against torch indexing (duplicates, negative
  entries, strided outputs); an out-of-range entry gives a zero row and the
  bad-index flag.
* saf_probe_mass: the 16-bit probe mass on the golden's inputs and sampled
  rows equals the oracle's and the reference's except for a handful of keys
  one 16-bit ulp apart (an fp32 sum on the other side of a rounding
  boundary); an f16 case with ragged row and key counts against the oracle.
* saf_masked_topn: bit-exact against the oracle's stable top-n, on the
  probe mass and on a tie-heavy integer mass.
* saf_bsa_fwd_keys (attention over per-batch key lists, rows fetched by TMA
  gather4 loads): within 2e-2 of the fp64 oracle, repeated keys and ragged
  lists included; an out-of-range key sets the bad-index flag.
* The processor at CogVideoX-2B size (B=2, H=30, bf16): window lists, the
  probe's keys (the stable top-n of its own mass), sampled output rows of
  the dense part and of both patch groups within 2e-2 of the fp64 oracle
  over the same key multisets, and the update_gap schedule of the probe.
"""
import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import local_global as olg
from sparseattnfunctions_b200 import _lib, kernels, workloads
from sparseattnfunctions_b200.geometry import COGVIDEOX_2B
from sparseattnfunctions_b200.special_attentions import LocalGlobalAttention as lga

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
_spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
mg = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(mg)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gather_rows_matches_torch(cuda_device, dtype):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, 4, 50, 64, generator=g).to(dtype).to(cuda_device)
    idx = torch.randint(-2, 150, (5, 37), generator=g)
    idx[0, :4] = torch.tensor([7, 7, 7, 149])  # duplicates
    got = kernels.gather_rows(x, idx.to(cuda_device))
    flat = x.permute(0, 2, 1, 3).reshape(150, 4, 64).cpu()
    ref = torch.zeros(5, 37, 4, 64, dtype=dtype)
    ok = idx >= 0
    ref[ok] = flat[idx[ok]]
    assert torch.equal(got.cpu(), ref.permute(0, 2, 1, 3))
    # strided output: every other row of a larger buffer
    big = torch.full((5, 4, 74, 64), 9.0, dtype=dtype, device=cuda_device)
    kernels.gather_rows(x, idx.to(cuda_device), out=big[:, :, ::2])
    assert torch.equal(big[:, :, ::2].cpu(), ref.permute(0, 2, 1, 3))
    assert bool((big[:, :, 1::2] == 9.0).all())


@pytest.mark.expects_device_status
def test_gather_rows_bad_index_sets_flag(cuda_device):
    _lib.read_device_status(0, clear=True)
    x = torch.ones(1, 2, 8, 64, dtype=torch.bfloat16, device=cuda_device)
    idx = torch.tensor([[0, 8, 3]], device=cuda_device)
    got = kernels.gather_rows(x, idx)
    torch.cuda.synchronize()
    assert bool((got[:, :, 1] == 0).all()) and bool((got[:, :, [0, 2]] == 1).all())
    assert _lib.read_device_status(0, clear=True) & _lib.SAF_DEV_BADINDEX


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_key_list_attention_matches_oracle(cuda_device, dtype):
    """saf_bsa_fwd_keys: every query batch attends its own list of rows of
    one k / v batch (gather4 loads), repeated keys counted twice, a ragged
    last block of the list and a ragged query tile."""
    g = torch.Generator().manual_seed(21)
    q = torch.randn(3, 2, 200, 64, generator=g).to(dtype)
    k = torch.randn(2, 2, 500, 64, generator=g).to(dtype)
    v = torch.randn(2, 2, 500, 64, generator=g).to(dtype)
    keys = torch.randint(0, 500, (3, 300), generator=g, dtype=torch.int32)
    keys[0, :10] = 7  # repeats
    src = torch.tensor([1, 0, 1], dtype=torch.int32)
    out = kernels.bsa_fwd_keys(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), keys.to(cuda_device),
                               src.to(cuda_device), 0.125).cpu()
    for b in range(3):
        kb, vb = k[src[b].item()][None], v[src[b].item()][None]
        rows = [(0, t) for t in range(200)]
        ref = olg.attention_rows(q[b][None], kb, vb, rows, lambda _b, _t: keys[b].numpy().astype(np.int64))
        assert np.abs(out[b].permute(1, 0, 2).float().numpy() - ref).max() < 2e-2


@pytest.mark.expects_device_status
def test_key_list_bad_index_sets_flag(cuda_device):
    _lib.read_device_status(0, clear=True)
    q = torch.randn(1, 1, 128, 64, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(1, 1, 256, 64, device=cuda_device).to(torch.bfloat16)
    keys = torch.arange(128, dtype=torch.int32, device=cuda_device).view(1, -1)
    keys[0, 5] = 256  # past the rows of k
    kernels.bsa_fwd_keys(q, k, k, keys, torch.zeros(1, dtype=torch.int32, device=cuda_device), 0.125)
    torch.cuda.synchronize()
    assert _lib.read_device_status(0, clear=True) & _lib.SAF_DEV_BADINDEX


def _golden_probe(cuda_device):
    d = np.load(GOLDEN / "local_global.npz")
    cfg = mg.LG_PROBE
    q, k = mg.lg_probe_inputs(cfg["seed"], cfg["H"], cfg["n_video"], cfg["S"], cfg["D"])
    samples = torch.from_numpy(d["samples"].astype(np.int64))
    base = torch.arange(2).view(2, 1) * cfg["n_video"]
    qs = kernels.gather_rows(q.to(cuda_device), (samples + base).to(cuda_device))
    mass = kernels.probe_mass(qs, k.to(cuda_device))
    torch.cuda.synchronize()
    return d, q, k, mass


def test_probe_mass_matches_oracle_and_reference(cuda_device):
    d, q, k, mass = _golden_probe(cuda_device)
    got = mass.cpu().numpy()
    ref = olg.probe_mass(q, k, d["samples"], row_offset=0)
    for other in (ref, d["att_probs"].astype(np.float64)):
        diff = got != other
        assert diff.sum() <= 8, diff.sum()
        assert np.all(np.abs(got - other)[diff] <= np.abs(other[diff]) * 2.0 ** -7)
    # deterministic
    mass2 = _golden_probe(cuda_device)[3]
    assert torch.equal(mass, mass2)


def test_probe_mass_f16_ragged(cuda_device):
    g = torch.Generator().manual_seed(11)
    q = (torch.randn(2, 3, 200, 64, generator=g) * 1.3).to(torch.float16)
    k = torch.randn(2, 3, 1000, 64, generator=g).to(torch.float16)
    mass = kernels.probe_mass(q.to(cuda_device), k.to(cuda_device)).cpu().numpy()
    ref = olg.probe_mass(q, k, np.tile(np.arange(200), (2, 1)), row_offset=0, kind="f16")
    diff = mass != ref
    assert diff.sum() <= 4, diff.sum()
    assert np.all(np.abs(mass - ref)[diff] <= np.abs(ref[diff]) * 2.0 ** -10)


def test_masked_topn_matches_oracle(cuda_device):
    d, q, k, mass = _golden_probe(cuda_device)
    lmask = olg.local_mask()
    got = kernels.masked_topn(mass, torch.from_numpy(lmask).to(cuda_device), olg.N_GLOBAL).cpu().numpy()
    assert np.array_equal(got, olg.global_keys(mass.cpu().numpy(), lmask, olg.N_GLOBAL))
    # tie-heavy: integer masses, ties broken to the lower key
    rs = np.random.RandomState(5)
    m = rs.randint(0, 40, size=(2, 5000)).astype(np.float64)
    lm = rs.rand(3, 5000) < 0.3
    got = kernels.masked_topn(torch.from_numpy(m).to(cuda_device), torch.from_numpy(lm).to(cuda_device),
                              300).cpu().numpy()
    assert np.array_equal(got, olg.global_keys(m, lm, 300))


@pytest.fixture(scope="module")
def full_run(cuda_device):
    q, k, v = workloads.video_qkv(COGVIDEOX_2B, B=2, H=30, device=cuda_device, seed=77)
    lga.counter = 0
    obj = lga.LocalGlobalAttention()
    torch.cuda.manual_seed(1234)
    out = obj(q, k, v)
    torch.cuda.synchronize()
    torch.cuda.manual_seed(1234)
    samples = torch.randint(0, 16200, (2, 1, 1280), device=cuda_device).view(2, -1)
    return q, k, v, obj, out, samples


def test_window_lists_follow_stable_sort(full_run):
    """torch.sort of the window mask on the GPU (the call the reference makes)
    lists, per patch, the window keys and then the first non-window keys in
    ascending order -- the oracle's stable-sort reading."""
    obj = full_run[3]
    wl = olg.window_lists(olg.local_mask())
    idx = obj.indices.cpu().numpy()
    for r in range(36):
        assert np.array_equal(np.sort(idx[r]), np.sort(wl[r // 2]))


def test_probe_keys_are_top_n_of_the_mass(full_run, cuda_device):
    q, k, v, obj, out, samples = full_run
    base = torch.arange(2, device=cuda_device).view(2, 1) * 16200
    qs = kernels.gather_rows(q[:, :, olg.DENSE_ROWS:], samples + base)
    mass = kernels.probe_mass(qs, k).cpu().numpy()
    gk = olg.global_keys(mass, olg.local_mask(), olg.N_GLOBAL)
    assert np.array_equal(obj.global_indices.cpu().numpy(), gk)


def test_output_rows_match_oracle(full_run):
    q, k, v, obj, out, samples = full_run
    idx = obj.indices.cpu().numpy()
    gk = obj.global_indices.cpu().numpy()

    def keys_of(b, t):
        if t < olg.DENSE_ROWS:
            return np.arange(17776)
        p = olg.patch_of(t)
        return np.concatenate([idx[p * 2 + b], gk[p * 2 + b]])  # a multiset, as the reference's gather

    rs = np.random.RandomState(9)
    rows = [(int(b), int(t)) for b, t in zip(rs.randint(0, 2, 12), rs.randint(0, olg.DENSE_ROWS, 12))]
    for p in (0, 4, 8, 9, 13, 17):  # both frame groups
        for t in rs.choice(olg.patch_rows(p), 5, replace=False):
            rows.append((int(rs.randint(0, 2)), int(t)))
    ref = olg.attention_rows(q.cpu(), k.cpu(), v.cpu(), rows, keys_of)
    got = np.stack([out[b, :, t].float().cpu().numpy() for b, t in rows])
    assert np.abs(got - ref).max() < 2e-2


def test_key_lists_in_kernel_equal_gathered_copies(full_run):
    """The processor's two patch paths -- attention over gathered k / v
    copies, and the kernel's key-list mode fetching the same rows by gather4
    -- read the same values in the same block order: identical outputs."""
    q, k, v, obj, out, samples = full_run
    lga.counter = 1 << 20  # keep the probe keys of the first call
    obj.gather_in_kernel = True
    try:
        out_keys = obj(q, k, v)
    finally:
        obj.gather_in_kernel = False
        lga.counter = lga.update_gap - 1
    assert torch.equal(out_keys, out)


def test_probe_update_gap(full_run, cuda_device):
    q, k, v, obj, out, samples = full_run
    assert lga.counter == lga.update_gap - 1
    g0 = obj.global_indices
    for i in range(lga.update_gap - 1):
        state = torch.cuda.get_rng_state(cuda_device)
        out2 = obj(q, k, v)
        assert torch.equal(torch.cuda.get_rng_state(cuda_device), state)  # no new probe
        assert obj.global_indices is g0
    assert torch.equal(out2, out)
    assert lga.counter == 0
    obj(q, k, v)  # the probe runs again
    assert obj.global_indices is not g0 and lga.counter == lga.update_gap - 1


def test_probe_score_mode_follows_the_cumulative_rule(cuda_device):
    """probe_solver(type="score") (:64-84): per batch, the keys by descending
    mass up to the first cumulative share >= percentile.  The rule is checked
    exactly on the probe kernel's own mass (the cumulative sum is a 16-bit
    scan, whose rounding differs between a CPU and a GPU), and that mass
    against the oracle's."""
    g = torch.Generator().manual_seed(41)
    q = (torch.randn(2, 2, 300, 64, generator=g) * 1.2).to(torch.bfloat16)
    k = torch.randn(2, 2, 700, 64, generator=g).to(torch.bfloat16)
    solver = lga.probe_solver(percentile=0.3, sample_num=64, type="score")
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    torch.cuda.manual_seed(7)
    got = solver._probe(qd, kd)
    torch.cuda.manual_seed(7)
    mass = solver._mass(qd, kd)
    torch.cuda.manual_seed(7)
    samples = torch.randint(0, 300, (2, 1, 64), device=cuda_device).view(2, -1).cpu().numpy()
    ref = olg.probe_mass(q, k, samples, row_offset=0)
    diff = mass.cpu().numpy() != ref
    assert diff.sum() <= 4, diff.sum()
    assert np.all(np.abs(mass.cpu().numpy() - ref)[diff] <= np.abs(ref[diff]) * 2.0 ** -7)
    for b in range(2):
        vals, idx = torch.sort(mass[b].to(torch.bfloat16), descending=True)
        cum = (vals / (2 * 64)).cumsum(dim=-1)
        n = int(torch.searchsorted(cum, 0.3)) + 1
        assert n < vals.numel()
        sel = got[b]
        assert sel.numel() == n
        # the first n by descending mass (a tie at the cut may go either way)
        assert float(vals[n - 1]) >= float(vals[n])
        picked = mass[b].to(torch.bfloat16)[sel].float()
        assert float(picked.min()) >= float(vals[n - 1])
        assert torch.unique(sel).numel() == n
