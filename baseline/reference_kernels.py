"""Loads the reference's own GPU kernels from its installed copy.

The reference (xiaolong-li1/SparseAttnFunctions) is installed, unmodified,
into ``baseline/_ref`` with

    python -m pip install --no-index --no-build-isolation \\
        --find-links /opt/wheelhouse --target baseline/_ref <reference>/special_attentions

Its setup.py packages only the ``utils`` directory, so the Triton modules
arrive as ``baseline/_ref/utils/{block_sparse_attn_kernel,attn_pooling_kernel}.py``.
They are loaded here under private module names.  ``block_sparse_attn_kernel``
imports matplotlib and torchmetrics at module level for its plotting test
(lines 393-400); neither is installed, and neither is on the kernel's path,
so empty stand-in modules are registered for them.

These kernels are the comparison bar and a GPU parity check for this
package's own kernels; nothing in ``sparseattnfunctions_b200`` imports this.
"""
from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

REF_DIR = Path(__file__).resolve().parent / "_ref" / "utils"


def available() -> bool:
    return (REF_DIR / "block_sparse_attn_kernel.py").exists()


def _stub_plotting() -> None:
    for name in ("matplotlib", "matplotlib.pyplot", "torchmetrics", "torchmetrics.functional"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["matplotlib"].use = lambda *a, **k: None
    sys.modules["matplotlib"].pyplot = sys.modules["matplotlib.pyplot"]
    sys.modules["torchmetrics.functional"].mean_squared_error = None


def load(name: str):
    """The reference module ``utils/<name>.py`` (e.g.
    ``"block_sparse_attn_kernel"``).  Raises ImportError when the reference
    is not installed."""
    mod_name = f"_saf_reference_{name}"
    if mod_name in sys.modules:
        return sys.modules[mod_name]
    path = REF_DIR / f"{name}.py"
    if not path.exists():
        raise ImportError(f"reference module {path} is not installed (see baseline/reference_kernels.py)")
    _stub_plotting()
    spec = importlib.util.spec_from_file_location(mod_name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[mod_name] = mod
    try:
        spec.loader.exec_module(mod)
    except Exception:
        del sys.modules[mod_name]
        raise
    return mod
