"""Generates the golden fixtures that pin the CPU oracle to the reference.

Run where the reference source tree is available (it is not on the GPU box):

    python tests/golden/make_golden.py /path/to/SparseAttnFunctions

It imports the reference's own Python modules from that tree -- with stub
modules for the imports this path does not use (sageattention, torch_kmeans,
matplotlib, torchmetrics and the external ``global_vars``) -- runs them on
the CPU on seeded inputs and writes ``tests/golden/*.npz``.  Inputs are not
stored: they are regenerated from ``numpy.random.RandomState(seed)`` (whose
streams numpy keeps stable), so the fixtures hold only seeds, parameters and
the reference's outputs.

Fixtures
  topk_masks.npz    get_sparse_attn_mask_from_topk (block_sparse_attn_kernel.py:31-39)
  energy_masks.npz  transfer_attn_to_mask(mode="energy") (SparseGen_Plus.py:12-84)
  topk_adaptive_masks.npz  transfer_attn_to_mask(mode="topk") (SparseGen_Plus.py:28-50)
  tome_*.npz        bipartite_soft_matching_video + merge / unmerge
                    (utils/merge_unmerge.py:34-154), fp64 metric;
                    tome_bf16_r4000.npz: the matching on a bf16 metric (the
                    reference normalises and multiplies in bf16), its split
                    order and the merged src / dst it chose
  sta_layout.npz    SildingTileAttention's tile-window mask_mod (small and
                    CogVideoX-2B configs) and its preprocess token order
                    (SildingTileAttention.py:18-136)
  smart_layout.npz  SmartAttention's frame-band mask_mod on a small geometry,
                    its per-frame key sets at CogVideoX-2B size, and the
                    process / process_back token orders (SmartAttention.py:
                    9-43, 90-95)
  attention_kat.npz block-sparse attention as the reference's own test oracle
                    defines it (the kron-mask statements of
                    test_topk_sparse_attention and
                    test_topk_sparse_attention_qlt_kl,
                    block_sparse_attn_kernel.py:326-334 and 366-384), run in
                    fp64 on the KAT shapes, a ragged case with an empty row
                    and the config-1 shape; stored as per-row sums and a
                    fixed random projection of each output row
  frame_scope.npz   generate_attention_mask_frame_scope (utils/mask_related.py:
                    194-245) on seeded fp64 q / k: the spatial sample it
                    drew (torch's CPU generator seeded before the call) and
                    the frame x frame mask it returned, at a small geometry
                    and at CogVideoX-2B's, for two thresholds
  mask_layout.npz   get_block_mask (utils/mask_related.py:397-404) on seeded
                    masks, and the query side of preprocess_qkv /
                    reverse_process_out (:87-187) on a token-index tensor
  local_global.npz  LocalGlobalAttention's get_mask (LocalGlobalAttention.py:
                    114-179: the patch window mask, remain_num and the keys
                    its CPU sort put after the window keys) and
                    probe_solver._probe_num (:50-62) on seeded bf16 q / k
                    with 2 heads: the rows torch.randint drew, the summed
                    probabilities (the softmax output summed as :57 does)
                    and the indices it returned
"""
from __future__ import annotations

import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def import_reference(root: str):
    for name in ["sageattention", "torch_kmeans", "matplotlib", "matplotlib.pyplot", "torchmetrics",
                 "torchmetrics.functional", "global_vars"]:
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["sageattention"].sageattn = None
    sys.modules["torch_kmeans"].KMeans = None
    sys.modules["matplotlib"].use = lambda *a, **k: None
    sys.modules["matplotlib"].pyplot = sys.modules["matplotlib.pyplot"]
    sys.modules["torchmetrics.functional"].mean_squared_error = None
    sys.modules["global_vars"].count = 0
    sys.path.insert(0, root)
    from special_attentions import SparseGen_Plus
    from special_attentions.utils import block_sparse_attn_kernel, merge_unmerge

    return block_sparse_attn_kernel, SparseGen_Plus, merge_unmerge


def sta_layout(root: str):
    """Evaluates SildingTileAttention's mask_mod and preprocess on the CPU.
    The module builds a CUDA block mask when imported, so its function and
    class definitions are taken from the source text and executed alone."""
    import ast
    import torch
    from einops import rearrange

    src = Path(root, "special_attentions", "SildingTileAttention.py").read_text()
    tree = ast.parse(src)
    keep = [n for n in tree.body if isinstance(n, (ast.FunctionDef, ast.ClassDef)) and
            n.name in ("generate_sta_mask", "SildingTileAttention")]
    ns = {"torch": torch, "rearrange": rearrange, "Tuple": tuple, "IntTensor": torch.Tensor,
          "BoolTensor": torch.Tensor}
    exec(compile(ast.Module(body=keep, type_ignores=[]), "sta", "exec"), ns)
    out = {}
    # small configuration: full token-level mask
    canvas, tile, kern, text = (4, 6, 9), (2, 3, 3), (1, 3, 3), 10
    mod = ns["generate_sta_mask"](canvas, kern, tile, text)
    S = text + canvas[0] * canvas[1] * canvas[2]
    qi, ki = torch.arange(S)[:, None], torch.arange(S)[None, :]
    out["small_mask"] = np.packbits(mod(0, 0, qi, ki).numpy())
    out["small_cfg"] = np.array([*canvas, *tile, *kern, text])
    # CogVideoX-2B configuration of the reference: every 7th query row, all keys
    canvas, tile, kern, text = (13, 30, 45), (13, 3, 3), (1, 9, 9), 226
    mod = ns["generate_sta_mask"](canvas, kern, tile, text)
    S = text + 13 * 30 * 45
    rows = torch.arange(0, S, 7)
    out["full_rows"] = rows.numpy().astype(np.int32)
    out["full_mask"] = np.packbits(mod(0, 0, rows[:, None], torch.arange(S)[None, :]).numpy())
    # preprocess order: the token index found at each position after the reordering
    obj = ns["SildingTileAttention"].__new__(ns["SildingTileAttention"])
    obj.config = {"kernel_size": kern, "tile_size": tile, "img_size": canvas, "text_length": text}
    idx = torch.arange(S, dtype=torch.float64).view(1, 1, S, 1).repeat(1, 1, 1, 1)
    q, _, _ = obj.preprocess(idx.clone(), idx.clone(), idx.clone())
    out["preprocess"] = q.reshape(-1).numpy().astype(np.int32)
    return out


def smart_layout(root: str):
    """Evaluates the reference's SmartAttention layout functions on the CPU."""
    import torch

    sys.path.insert(0, root)
    from special_attentions import SmartAttention as sa

    out = {}
    T, F, n, S = 26, 150, 5, 26 + 5 * 150  # small band: 26 text + 5 frames of 150 tokens
    mod = sa.generate_block_tridiagonal_mask_mod(prompt_length=T, num_frames=n, token_per_frame=F, diag=1)
    qi, ki = torch.arange(S)[:, None], torch.arange(S)[None, :]
    out["band_small"] = np.packbits(mod(0, 0, qi, ki).numpy())
    out["band_small_geom"] = np.array([T, n, 10, 15])
    full = sa.generate_block_tridiagonal_mask_mod()
    S2, rows = 17776, [226 + i * 1350 for i in range(13)]
    keys = [torch.where(full(0, 0, torch.tensor(r), torch.arange(S2)))[0].numpy() for r in rows]
    out["frame_keys"] = np.concatenate(keys).astype(np.int32)
    out["frame_keys_off"] = np.cumsum([0] + [k.size for k in keys]).astype(np.int32)
    idx = torch.arange(S2, dtype=torch.float64).view(1, 1, S2, 1)
    out["process"] = sa.process(idx).reshape(-1).numpy().astype(np.int32)
    out["process_back"] = sa.process_back(idx).reshape(-1).numpy().astype(np.int32)
    return out


class _CpuTorch:
    """The torch namespace for the reference's test-oracle statements: every
    attribute is torch's own, except that tensor factories given
    ``device='cuda'`` (the reference's tests run on a GPU) build CPU
    tensors."""

    def __init__(self):
        import torch

        self._torch = torch

    def __getattr__(self, name):
        attr = getattr(self._torch, name)
        if name in ("ones", "zeros", "arange", "full", "randn", "rand"):
            def factory(*args, **kwargs):
                if str(kwargs.get("device", "cpu")).startswith("cuda"):
                    kwargs["device"] = "cpu"
                return attr(*args, **kwargs)
            return factory
        return attr


def reference_kat_oracles(root: str):
    """The reference's own test-oracle statements as callables: the slice of
    ``test_topk_sparse_attention`` from ``full_mask = ...`` to ``ref_output
    = ...`` (block_sparse_attn_kernel.py:326-334) and of
    ``test_topk_sparse_attention_qlt_kl`` from ``past_len = ...`` to
    ``ref_output = ...`` (:366-384), taken from the source text and run with
    the inputs as arguments."""
    import ast
    import torch

    src = Path(root, "special_attentions", "utils", "block_sparse_attn_kernel.py").read_text()
    fns = {n.name: n for n in ast.parse(src).body if isinstance(n, ast.FunctionDef)}

    def assigned(st):
        return [t.id for t in getattr(st, "targets", []) if isinstance(t, ast.Name)]

    def make(fname, first, args):
        body = fns[fname].body
        i0 = next(i for i, st in enumerate(body) if first in assigned(st))
        i1 = next(i for i, st in enumerate(body) if i >= i0 and "ref_output" in assigned(st))
        stmts = body[i0:i1 + 1] + [ast.Return(value=ast.Name("ref_output", ast.Load()))]
        fn = ast.FunctionDef(name="kat_oracle", args=ast.arguments(
            posonlyargs=[], args=[ast.arg(a) for a in args], kwonlyargs=[], kw_defaults=[], defaults=[]),
            body=stmts, decorator_list=[], returns=None, type_params=[])
        mod = ast.fix_missing_locations(ast.Module(body=[fn], type_ignores=[]))
        ns = {"torch": _CpuTorch(), "F": torch.nn.functional}
        exec(compile(mod, f"{fname}-oracle", "exec"), ns)
        return ns["kat_oracle"]

    square = make("test_topk_sparse_attention", "full_mask", ["q", "k", "v", "block_mask", "sm_scale", "BLOCK",
                                                              "SEQ_LEN"])
    rect = make("test_topk_sparse_attention_qlt_kl", "past_len", ["q", "k", "v", "block_mask", "sm_scale",
                                                                  "BLOCK", "Q_LEN", "K_LEN"])
    return square, rect


# (name, seed, B, H, Sq, Sk, block, topk or None for all-ones, force first column, empty row)
ATTN_CASES = [("kat_ragged_ones", 301, 1, 3, 257, 257, 64, None, True, -1),
              ("kat_ragged_top2", 302, 1, 3, 257, 257, 64, 2, True, -1),
              ("kat_qlen_lt_klen", 303, 2, 4, 128, 256, 64, 1, True, -1),
              ("ragged_empty_row", 304, 2, 2, 300, 300, 64, 2, False, 3),
              ("config1_shape", 305, 1, 2, 2048, 2048, 64, 8, True, -1)]


def attn_inputs(seed, B, H, Sq, Sk, block, topk, force_first, empty_row, bsk=None):
    """Seeded fp64 q, k, v (N(0,1) / 8 for q and k) and the block mask.  The
    mask is the reference's get_sparse_attn_mask_from_topk of seeded scores
    (first column forced high like the reference's KAT); it is computed by
    the reference when ``bsk`` is given, else read back from the fixture."""
    import torch

    rs = np.random.RandomState(seed)
    q = rs.randn(B, H, Sq, 64) / 8.0
    k = rs.randn(B, H, Sk, 64) / 8.0
    v = rs.randn(B, H, Sk, 64)
    nbq, nbk = -(-Sq // block), -(-Sk // block)
    n = max(nbq, nbk)
    x = rs.randn(B, H, n, n)
    if force_first:
        x[..., 0] = 100.0
    if bsk is None:
        return q, k, v, None
    if topk is None:
        mask = torch.ones(B, H, n, n, dtype=torch.bool)
    else:
        mask = bsk.get_sparse_attn_mask_from_topk(torch.from_numpy(x), topk)
    if empty_row >= 0:
        mask[0, 0, empty_row, :] = False
    return q, k, v, mask


def attention_kat(root: str, bsk):
    import torch

    square, rect = reference_kat_oracles(root)
    out = {"cases": np.array([[-1 if x is None else int(x) for x in c[1:]] for c in ATTN_CASES],
                             dtype=np.int64)}
    for name, seed, B, H, Sq, Sk, block, topk, ff, er in ATTN_CASES:
        q, k, v, mask = attn_inputs(seed, B, H, Sq, Sk, block, topk, ff, er, bsk)
        tq, tk, tv = (torch.from_numpy(t) for t in (q, k, v))
        if Sq == Sk:
            ref = square(tq, tk, tv, mask, 0.125, block, Sq)
        else:
            ref = rect(tq, tk, tv, mask, 0.125, block, Sq, Sk)
        ref = ref.numpy()
        proj = np.random.RandomState(seed + 3000).randn(64)
        out[f"{name}_mask"] = np.packbits(mask.numpy())
        out[f"{name}_mask_shape"] = np.array(mask.shape)
        out[f"{name}_rowsum"] = ref.sum(-1)
        out[f"{name}_proj"] = ref @ proj
    return out


# (name, seed, B, H, text, frames, height, width, sample_num, threshold)
FRAME_CASES = [("small_t90", 401, 1, 2, 20, 5, 6, 8, 10, 0.9),
               ("small_t70", 402, 2, 2, 20, 5, 6, 8, 10, 0.7),
               ("cogvideox_t90", 403, 1, 2, 226, 13, 30, 45, 60, 0.9)]


def frame_inputs(seed, B, H, text, frames, height, width):
    """fp64 q, k [B, H, text + frames*height*width, 64]: a random vector per
    (head, frame) shared by its tokens plus N(0, 1) noise (text: noise only),
    so that frames attend to one another unevenly."""
    rs = np.random.RandomState(seed)
    fl = height * width
    out = []
    for _ in range(2):
        centre = rs.randn(B, H, frames, 1, 64) * 1.5
        vid = (centre + rs.randn(B, H, frames, fl, 64)).reshape(B, H, frames * fl, 64)
        out.append(np.concatenate([rs.randn(B, H, text, 64), vid], axis=2))
    return out[0], out[1]


def mask_layout(root: str):
    """The reference's get_block_mask on seeded frame / inner masks (it
    fixes B = 2, H = 30) and the query side of preprocess_qkv /
    reverse_process_out on a token-index tensor (positions + 1, so the
    zero padding reads 0)."""
    import torch

    sys.path.insert(0, root)
    from special_attentions.utils import mask_related as mr

    rs = np.random.RandomState(601)
    frame = torch.from_numpy(rs.rand(2, 30, 13, 13) < 0.4)
    inner = torch.from_numpy(rs.rand(2, 30, 22, 21) < 0.8)
    block = mr.get_block_mask(inner, frame)
    idx = torch.arange(1, 17777, dtype=torch.float64).view(1, 1, 17776, 1)
    qp, _, _ = mr.preprocess_qkv(idx, idx.clone(), idx.clone())
    back = mr.reverse_process_out(qp)
    return {"block_mask": np.packbits(block.numpy() != 0), "block_shape": np.array(block.shape),
            "q_processed": qp.reshape(-1).numpy().astype(np.int32),
            "q_back": back.reshape(-1).numpy().astype(np.int32)}


def frame_scope(root: str):
    import torch

    sys.path.insert(0, root)
    from special_attentions.utils import mask_related as mr

    out = {"cases": np.array([c[1:9] for c in FRAME_CASES], dtype=np.int64),
           "thresholds": np.array([c[9] for c in FRAME_CASES])}
    for name, seed, B, H, text, frames, height, width, n, thr in FRAME_CASES:
        q, k = frame_inputs(seed, B, H, text, frames, height, width)
        torch.manual_seed(seed)
        spatial = torch.randint(0, width * height, (n,))
        torch.manual_seed(seed)
        mask = mr.generate_attention_mask_frame_scope(
            torch.from_numpy(q), torch.from_numpy(k), text_length=text, f=frames, width=width,
            height=height, sample_num=n, scale_factor=1 / 8, base_threshold=thr)
        out[f"{name}_spatial"] = spatial.numpy().astype(np.int32)
        out[f"{name}_mask"] = mask.numpy()
    return out


LG_PROBE = dict(seed=701, H=2, n_video=16200, S=17776, D=64)


def lg_probe_inputs(seed, H, n_video, S, D):
    """bf16-representable q_video [2, H, n_video, D] and k [2, H, S, D]: a
    smooth field over the key index plus noise, so the probe mass varies."""
    rs = np.random.RandomState(seed)
    import torch

    base = rs.randn(2, H, S // 64 + 1, D).repeat(64, axis=2)[:, :, :S]
    k = torch.from_numpy(base + 0.7 * rs.randn(2, H, S, D)).to(torch.bfloat16)
    q = torch.from_numpy(rs.randn(2, H, n_video, D) * 1.5).to(torch.bfloat16)
    return q, k


def local_global(root: str):
    """get_mask and probe_solver._probe_num from the reference's source text
    (the module builds its mask on CUDA when imported), run on the CPU: the
    module constants, get_mask and probe_solver are executed alone, with
    create_mask on the CPU and torch.softmax wrapped to record its output."""
    import ast
    import torch
    from torch.nn.attention.flex_attention import create_mask as _create_mask

    src = Path(root, "special_attentions", "LocalGlobalAttention.py").read_text()
    tree = ast.parse(src)
    consts = {"video_shape", "patch_shape", "batch_size", "compression", "sample_num", "padding",
              "percentile", "update_gap"}
    keep = [n for n in tree.body
            if (isinstance(n, ast.Assign) and any(isinstance(t, ast.Name) and t.id in consts for t in n.targets))
            or (isinstance(n, (ast.FunctionDef, ast.ClassDef)) and n.name in ("get_mask", "probe_solver"))]
    seen = []

    class _Torch(_CpuTorch):
        def __getattr__(self, name):
            if name == "softmax":
                def softmax(x, *a, **k):
                    y = torch.softmax(x, *a, **k)
                    seen.append(y)
                    return y
                return softmax
            return super().__getattr__(name)

    def create_mask(fn, B, H, Q_LEN, KV_LEN, device="cuda"):
        return _create_mask(fn, B, H, Q_LEN, KV_LEN, device="cpu")

    ns = {"torch": _Torch(), "create_mask": create_mask, "print": lambda *a, **k: None}
    exec(compile(ast.Module(body=keep, type_ignores=[]), "local_global", "exec"), ns)
    mask, indices = ns["get_mask"]()
    remain = indices.shape[1]
    out = {"mask": np.packbits(mask.numpy()), "mask_shape": np.array(mask.shape), "remain": np.array(remain)}
    fill = [np.setdiff1d(indices[r].numpy(), np.nonzero(mask[r].numpy())[0]) for r in range(mask.shape[0])]
    out["fill_keys"] = np.concatenate(fill).astype(np.int32)
    out["fill_off"] = np.cumsum([0] + [f.size for f in fill]).astype(np.int32)
    cfg = LG_PROBE
    q, k = lg_probe_inputs(cfg["seed"], cfg["H"], cfg["n_video"], cfg["S"], cfg["D"])
    solver = ns["probe_solver"](percentile=ns["percentile"], sample_num=ns["sample_num"], device="cpu",
                                type="num", mask=mask)
    torch.manual_seed(cfg["seed"])
    samples = torch.randint(0, cfg["n_video"], (2, 1, ns["sample_num"]), device="cpu")
    torch.manual_seed(cfg["seed"])
    seen.clear()
    idx = solver._probe(q, k)
    out["samples"] = samples.reshape(2, -1).numpy().astype(np.int32)
    # the statement after the softmax (:57), before the repeat and masked_fill
    out["att_probs"] = seen[0].sum(dim=[1, 2]).float().numpy()
    out["probe_indices"] = idx.numpy().astype(np.int32)
    return out


def closure_vars(fn):
    return {name: cell.cell_contents for name, cell in zip(fn.__code__.co_freevars, fn.__closure__)}


TOPK_CASES = [  # (seed, B, H, n, topk)
    (101, 1, 2, 16, 4), (102, 2, 3, 33, 5), (103, 1, 1, 139, 14), (104, 1, 2, 64, 1)]
ENERGY_CASES = [  # (seed, B, H, n, thr, min_ratio, max_ratio)
    (201, 1, 2, 20, 0.9, 0.1, 0.8), (202, 2, 2, 45, 0.95, 0.1, 0.7), (203, 1, 3, 139, 0.98, 0.12, 1.0)]
TOME_BF16_CASE = ("tome_bf16_r4000", 13, 16, 4000)  # (name, metric seed, C, r), no_rand split
TOME_CASES = [  # (name, metric seed, C, r, generator seed or None)
    ("tome_norand_r4000", 11, 8, 4000, None), ("tome_gen_r9000", 12, 8, 9000, 5)]
GEOM = dict(w=45, h=30, t=13, sx=3, sy=3, st=4)
TEXT = 226
PROJ_C = 240  # channel count that lets the reference's unmerge reshape to (2, 30, -1, 64)


# (seed, B, H, n, init_k, power): inputs rand ** power, from flat to peaked rows
TOPK_ADAPTIVE_CASES = [(501, 1, 2, 40, 0.1, 3.0), (502, 2, 2, 139, 0.1, 8.0), (503, 1, 3, 139, 5, 1.0),
                       (504, 1, 2, 64, 0.25, 12.0)]


def topk_adaptive_input(seed, B, H, n, power):
    return np.random.RandomState(seed).rand(B, H, n, n) ** power


def topk_input(seed, B, H, n):
    return np.random.RandomState(seed).randn(B, H, n, n)


def energy_input(seed, B, H, n):
    return np.random.RandomState(seed).rand(B, H, n, n) ** 3


def tome_metric(seed, C):
    return np.random.RandomState(seed).randn(1, GEOM["w"] * GEOM["h"] * GEOM["t"], C)


def tome_x(seed, n_rows):
    return np.random.RandomState(seed + 1000).randn(1, n_rows, PROJ_C)


def projection(seed):
    return np.random.RandomState(seed + 2000).randn(PROJ_C)


def main(root: str):
    import torch

    bsk, sgp, mu = import_reference(root)

    masks = {}
    for seed, B, H, n, k in TOPK_CASES:
        x = torch.from_numpy(topk_input(seed, B, H, n))
        masks[f"case_{seed}"] = bsk.get_sparse_attn_mask_from_topk(x, k).numpy()
    np.savez_compressed(HERE / "topk_masks.npz", cases=np.array(TOPK_CASES), **masks)

    masks = {}
    for seed, B, H, n, thr, mn, mx in ENERGY_CASES:
        a = torch.from_numpy(energy_input(seed, B, H, n))
        masks[f"case_{seed}"] = sgp.transfer_attn_to_mask(
            a, mode="energy", max_retain_ratio=mx, min_retain_ratio=mn, energy_threshold=thr).numpy()
    np.savez_compressed(HERE / "energy_masks.npz", cases=np.array(ENERGY_CASES), **masks)

    masks = {}
    for seed, B, H, n, init_k, power in TOPK_ADAPTIVE_CASES:
        a = torch.from_numpy(topk_adaptive_input(seed, B, H, n, power))
        masks[f"case_{seed}"] = sgp.transfer_attn_to_mask(a, mode="topk", init_k=init_k).numpy()
    np.savez_compressed(HERE / "topk_adaptive_masks.npz", cases=np.array(TOPK_ADAPTIVE_CASES), **masks)

    for name, seed, C, r, gseed in TOME_CASES:
        metric = torch.from_numpy(tome_metric(seed, C))
        gen = None if gseed is None else torch.Generator().manual_seed(gseed)
        merge, unmerge = mu.bipartite_soft_matching_video(metric, **GEOM, r=r, no_rand=gseed is None,
                                                          generator=gen)
        cv = closure_vars(merge)
        uv = closure_vars(unmerge)
        sv = closure_vars(cv["split"])
        a_idx = sv["a_idx"].reshape(-1).numpy()  # video-token indices (reference order)
        b_idx = sv["b_idx"].reshape(-1).numpy()
        out = dict(a_idx=a_idx.astype(np.int32), b_idx=b_idx.astype(np.int32),
                   unm_idx=cv["unm_idx"].reshape(-1).numpy().astype(np.int32),
                   src_idx=cv["src_idx"].reshape(-1).numpy().astype(np.int32),
                   dst_idx=cv["dst_idx"].reshape(-1).numpy().astype(np.int32),
                   counter=mu.counter.reshape(-1).numpy().astype(np.int32),
                   params=np.array([seed, C, r, -1 if gseed is None else gseed]))
        if gseed is not None:
            g = torch.Generator().manual_seed(gseed)
            tst, hsy, wsx = (GEOM["t"] - 1) // GEOM["st"], GEOM["h"] // GEOM["sy"], GEOM["w"] // GEOM["sx"]
            out["rand_idx"] = torch.randint(GEOM["sy"] * GEOM["sx"] * GEOM["st"], size=(tst, hsy, wsx, 1),
                                            generator=g).reshape(-1).numpy().astype(np.int32)
        # merge of a 3-D tensor and unmerge of [text | merged]: stored as two
        # projections per row (row sums and a fixed random projection).
        n = metric.shape[1]
        proj = torch.from_numpy(projection(seed))
        x = torch.from_numpy(tome_x(seed, n))
        merged = merge(x)
        out["merge_rowsum"] = merged.sum(-1).reshape(-1).numpy()
        out["merge_proj"] = (merged @ proj).reshape(-1).numpy()
        y = torch.from_numpy(tome_x(seed + 1, TEXT + merged.shape[1]))
        un = unmerge(y).reshape(1, -1, PROJ_C)
        out["unmerge_rowsum"] = un.sum(-1).reshape(-1).numpy()
        out["unmerge_proj"] = (un @ proj).reshape(-1).numpy()
        np.savez_compressed(HERE / f"{name}.npz", **out)
    name, seed, C, r = TOME_BF16_CASE
    metric = torch.from_numpy(tome_metric(seed, C)).to(torch.bfloat16)
    merge, _ = mu.bipartite_soft_matching_video(metric, **GEOM, r=r, no_rand=True)
    cv = closure_vars(merge)
    sv = closure_vars(cv["split"])
    np.savez_compressed(HERE / f"{name}.npz", params=np.array([seed, C, r]),
                        a_idx=sv["a_idx"].reshape(-1).numpy().astype(np.int16),
                        b_idx=sv["b_idx"].reshape(-1).numpy().astype(np.int16),
                        src_idx=cv["src_idx"].reshape(-1).numpy().astype(np.int16),
                        dst_idx=cv["dst_idx"].reshape(-1).numpy().astype(np.int16))
    np.savez_compressed(HERE / "attention_kat.npz", **attention_kat(root, bsk))
    np.savez_compressed(HERE / "frame_scope.npz", **frame_scope(root))
    np.savez_compressed(HERE / "mask_layout.npz", **mask_layout(root))
    np.savez_compressed(HERE / "smart_layout.npz", **smart_layout(root))
    np.savez_compressed(HERE / "sta_layout.npz", **sta_layout(root))
    np.savez_compressed(HERE / "local_global.npz", **local_global(root))
    print("fixtures written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/SparseAttnFunctions")
    main(sys.argv[1])
