"""ctypes binding of ``libsaf.so`` (declared in ``include/saf_api.h``).

The library is loaded from the package directory.  There is no fallback: if
the library is missing or a call returns a non-OK status, the caller gets an
exception.  Status codes map to the exception types the reference raises for
the same situations (``AssertionError`` for shape asserts in
``special_attentions/utils/block_sparse_attn_kernel.py:226-231`` surfaces here
as ``ValueError``; CUDA failures as ``RuntimeError``).
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

# The in-tree build; SAF_LIBRARY may point at another build of the same ABI
# (used to compare kernel variants side by side).
LIB_PATH = Path(os.environ.get("SAF_LIBRARY") or Path(__file__).resolve().parent / "libsaf.so")

SAF_OK = 0
SAF_ERR_SHAPE = 1
SAF_ERR_DTYPE = 2
SAF_ERR_STRIDE = 3
SAF_ERR_CUDA = 4
SAF_ERR_TIMEOUT = 5
SAF_ERR_NCCL = 6
SAF_ERR_ARG = 7
SAF_ERR_UNSUPPORTED = 8
SAF_ERR_WORKSPACE = 9

SAF_BF16 = 0
SAF_F16 = 1
SAF_F32 = 2

SAF_DEV_TIMEOUT = 0x1
SAF_DEV_BADINDEX = 0x2

ABI_VERSION = 1


class SafError(RuntimeError):
    """A libsaf call returned a non-OK status."""

    def __init__(self, func: str, status: int, msg: str):
        super().__init__(f"{func}: {msg} (status {status})")
        self.status = status


class SafShapeError(SafError, ValueError):
    """Bad shape, dtype, stride or argument (the reference's assert cases)."""


class SafTimeoutError(SafError):
    """A device-side wait ran out of its budget."""


class Tensor4(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("B", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("S", ctypes.c_int64),
        ("D", ctypes.c_int64),
        ("stride_b", ctypes.c_int64),
        ("stride_h", ctypes.c_int64),
        ("stride_s", ctypes.c_int64),
    ]


class SelectCfg(ctypes.Structure):
    _fields_ = [
        ("block_m", ctypes.c_int32),
        ("block_n", ctypes.c_int32),
        ("topk", ctypes.c_int32),
        ("text_blocks_q", ctypes.c_int32),
        ("text_blocks_k", ctypes.c_int32),
        ("force_diag", ctypes.c_int32),
        ("forced_inside_topk", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class TomePlan(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "unm_idx", "src_idx", "dst_idx", "counter", "dst_ptr", "dst_src", "token_map", "log_count",
        "node_max", "node_idx")]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_U64 = ctypes.c_uint64
_SZ = ctypes.c_size_t
_F32 = ctypes.c_float
_PT4 = ctypes.POINTER(Tensor4)
_PCFG = ctypes.POINTER(SelectCfg)

# name -> (restype, argtypes); must match include/saf_api.h exactly.
SIGNATURES = {
    "saf_abi_version": (_I32, []),
    "saf_status_string": (ctypes.c_char_p, [_I32]),
    "saf_device_check": (_I32, [_I32]),
    "saf_set_wait_budget_ns": (None, [_U64]),
    "saf_get_wait_budget_ns": (_U64, []),
    "saf_read_device_status": (_I32, [_I32, ctypes.POINTER(ctypes.c_uint32), _I32]),
    "saf_selftest_timeout": (_I32, [_U64, _P]),
    "saf_pool_topk_workspace_bytes": (_SZ, [_PT4, _PT4, _PCFG]),
    "saf_pool_topk": (_I32, [_PT4, _PT4, _PCFG, _P, _P, _P, _P, _P, _SZ, _P]),
    "saf_pool_topk_noalloc": (_I32, [_PT4, _PT4, _PCFG, _P, _P, _P, _P, _P]),
    "saf_energy_select": (_I32, [_P, _I32, _I64, _I32, _I32, _I32, _I64, ctypes.c_double, ctypes.c_double,
                                 _I32, _I32, _I32, _P, _P, _P]),
    "saf_topk_adaptive_select": (_I32, [_P, _I32, _I64, _I32, _I32, _I32, _I64, ctypes.c_double, _I32, _I32,
                                        _P, _P, _P]),
    "saf_mask_to_csr": (_I32, [_P, _I64, _I32, _I32, _I64, _I64, _P, _P, _P]),
    "saf_bsa_fwd": (_I32, [_PT4, _PT4, _PT4, _PT4, _P, _P, _I64, _I32, _I32, _P, _I64, _F32, _I32,
                           _P]),
    "saf_bsa_fwd_ranges": (_I32, [_PT4, _PT4, _PT4, _PT4, _P, _P, _I64, _I32, _I32, _P, _I64, _F32,
                                  _I32, _P, _P]),
    "saf_frame_mask_workspace_bytes": (_SZ, [_I64, _I32, _I32, _I32, _I32]),
    "saf_frame_mask": (_I32, [_PT4, _PT4, _P, _I32, _I32, _I32, _I32, _F32, ctypes.c_double, _P, _SZ, _P,
                              _P, _P, _P]),
    "saf_frame_csr": (_I32, [_P, _I64, _I32, _I32, _I32, _I64, _I32, _I32, _P, _P, _P]),
    "saf_bsa_fwd_frames": (_I32, [_PT4, _PT4, _PT4, _PT4, _P, _P, _I64, _I32, _I32, _P, _I32, _I32, _I32,
                                  _F32, _I32, _P]),
    "saf_bsa_pool_workspace_bytes": (_I64, [_I64, _I64, _I32]),
    "saf_bsa_fwd_pool": (_I32, [_PT4, _PT4, _PT4, _PT4, _P, _P, _I64, _I32, _I32, _F32, _I32, _I32, _P,
                                _I64, _P, _P]),
    "saf_tome_match_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I64, _I32]),
    "saf_tome_match": (_I32, [_P, _I32, _I64, _I64, _I64, _I64, _I64, _P, _I64, _P, _I64, _I32,
                              ctypes.POINTER(TomePlan), _P, _SZ, _P]),
    "saf_tome_kv_metric": (_I32, [_PT4, _PT4, _I32, _P, _P]),
    "saf_tome_merge": (_I32, [_P, _P, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _P, _I64, _P,
                              _I64, _I32, ctypes.POINTER(TomePlan), _P]),
    "saf_tome_unmerge": (_I32, [_P, _P, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _I64, _P, _P]),
    "saf_permute_tokens": (_I32, [_P, _P, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                  _I64, _I64, _P, _P, _I64, _P]),
    "saf_ulysses_pack": (_I32, [_P, _I32, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I32, _P,
                                _P]),
    "saf_ulysses_unpack": (_I32, [_P, _I32, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I32,
                                  _P, _P]),
    "saf_gather_rows": (_I32, [_P, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I64, _I64,
                               _I64, _I64, _P, _P]),
    "saf_probe_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I32]),
    "saf_probe_mass": (_I32, [_PT4, _PT4, _P, _SZ, _P, _P]),
    "saf_masked_topn": (_I32, [_P, _P, _I64, _I64, _I64, _I32, _P, _P]),
    "saf_bsa_fwd_keys": (_I32, [_PT4, _PT4, _PT4, _PT4, _P, _I32, _P, _F32, _P]),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Loads libsaf.so once; raises if it is missing or its ABI differs."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m sparseattnfunctions_b200.build`"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.saf_abi_version() != ABI_VERSION:
                raise ImportError("libsaf.so ABI version mismatch; rebuild the library")
            _lib = lib
    return _lib


def check(func: str, status: int) -> None:
    """Raises the exception type matching a non-OK status."""
    if status == SAF_OK:
        return
    msg = load().saf_status_string(status).decode()
    if status in (SAF_ERR_SHAPE, SAF_ERR_DTYPE, SAF_ERR_STRIDE, SAF_ERR_ARG, SAF_ERR_WORKSPACE):
        raise SafShapeError(func, status, msg)
    if status == SAF_ERR_TIMEOUT:
        raise SafTimeoutError(func, status, msg)
    raise SafError(func, status, msg)


def set_wait_budget_ns(ns: int) -> None:
    load().saf_set_wait_budget_ns(int(ns))


def get_wait_budget_ns() -> int:
    return int(load().saf_get_wait_budget_ns())


def read_device_status(device: int, clear: bool = True) -> int:
    """Synchronises ``device`` and returns (and by default clears) its sticky
    status flags (``SAF_DEV_TIMEOUT``, ``SAF_DEV_BADINDEX``)."""
    flags = ctypes.c_uint32(0)
    check("saf_read_device_status", load().saf_read_device_status(device, ctypes.byref(flags), int(clear)))
    return int(flags.value)


def raise_on_device_status(device: int) -> None:
    """Reads and clears ``device``'s status flags; raises ``SafTimeoutError``
    when a device-side wait ran out and ``SafError`` when a kernel skipped an
    out-of-range index."""
    flags = read_device_status(device, clear=True)
    if flags & SAF_DEV_TIMEOUT:
        raise SafTimeoutError("device status", SAF_ERR_TIMEOUT, f"a device wait ran out (flags {flags:#x})")
    if flags:
        raise SafError("device status", SAF_ERR_ARG, f"a kernel skipped an out-of-range index (flags {flags:#x})")
