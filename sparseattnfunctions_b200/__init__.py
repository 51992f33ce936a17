"""B200 (sm_100a) implementation of the SparseAttnFunctions attention hot path.

Layout
  csrc/                 CUDA kernels and the C ABI (declared in include/saf_api.h)
  build.py              nvcc build of libsaf.so (in-tree)
  _lib.py               ctypes binding, status -> exception mapping
  kernels.py            torch-facing wrappers (pool_topk, mask_to_csr, bsa_fwd, ...)
  geometry.py           CogVideoX token geometry (text + t x h x w video grid)
  workloads.py          seeded synthetic inputs for the benchmark configurations
  special_attentions/   drop-in mirror of the reference package's public API

``install_alias()`` registers ``special_attentions`` as an importable alias of
``sparseattnfunctions_b200.special_attentions`` so code written against the
reference (``from special_attentions.utils.block_sparse_attn_kernel import
block_sparse_triton_fn``) runs unchanged.
"""
from __future__ import annotations

import sys

__all__ = ["install_alias"]


def install_alias() -> None:
    """Makes ``import special_attentions...`` resolve to this package's mirror."""
    import importlib

    pkg = importlib.import_module(__name__ + ".special_attentions")
    sys.modules.setdefault("special_attentions", pkg)
    for sub in ("utils", "utils.block_sparse_attn_kernel", "utils.merge_unmerge",
                "utils.mask_related", "utils.attn_pooling_kernel", "block_mask_attn", "MergeAttention",
                "combined_attn", "SmartAttention", "SparseGen_Plus", "SildingTileAttention",
                "LocalGlobalAttention"):
        try:
            mod = importlib.import_module(f"{pkg.__name__}.{sub}")
        except ImportError:
            continue
        sys.modules.setdefault(f"special_attentions.{sub}", mod)
