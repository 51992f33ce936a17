"""The C-ABI library loads, exports every symbol include/*.h declares with the
ctypes signatures the binding uses, and rejects bad arguments on the host
(no GPU work: every call here fails validation before touching the device)."""
import ctypes
import re
from pathlib import Path

import pytest

from sparseattnfunctions_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from sparseattnfunctions_b200 import build

        build.build()
    return _lib.load()


def declared_functions():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(saf_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_every_declared_symbol_is_exported_and_bound(lib):
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), f"{name} missing from libsaf.so"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_version_and_status_strings(lib):
    assert lib.saf_abi_version() == _lib.ABI_VERSION
    assert lib.saf_status_string(0) == b"ok"
    for code in range(1, 10):
        assert lib.saf_status_string(code) not in (b"", b"unknown status")
    assert lib.saf_status_string(1234) == b"unknown status"


def test_wait_budget_roundtrip(lib):
    old = _lib.get_wait_budget_ns()
    try:
        _lib.set_wait_budget_ns(12345)
        assert _lib.get_wait_budget_ns() == 12345
    finally:
        _lib.set_wait_budget_ns(old)


def _t4(dtype=_lib.SAF_BF16, data=0, B=1, H=2, S=256, D=64):
    t = _lib.Tensor4()
    t.data = data
    t.dtype = dtype
    t.B, t.H, t.S, t.D = B, H, S, D
    t.stride_s, t.stride_h, t.stride_b = D, S * D, H * S * D
    return t


def test_bsa_rejects_bad_arguments_on_host(lib):
    good = 0x10000
    q, k, v, o = _t4(data=good), _t4(data=good), _t4(data=good), _t4(data=good)
    args = lambda q_, k_, v_, o_, rp=good, ci=good: lib.saf_bsa_fwd(
        ctypes.byref(q_), ctypes.byref(k_), ctypes.byref(v_), ctypes.byref(o_), rp, ci, 16, 128, 128,
        None, 0, 0.125, 0, None)
    assert args(_t4(data=0), k, v, o) == _lib.SAF_ERR_ARG            # null data
    assert args(q, k, v, o, rp=None) == _lib.SAF_ERR_ARG             # null CSR
    assert args(_t4(data=good, dtype=9), k, v, o) == _lib.SAF_ERR_DTYPE
    assert args(q, _t4(data=good, dtype=_lib.SAF_F16), v, o) == _lib.SAF_ERR_DTYPE
    assert args(q, _t4(data=good, D=128), v, o) == _lib.SAF_ERR_SHAPE
    assert args(q, _t4(data=good, S=100), v, o) == _lib.SAF_ERR_SHAPE  # k/v length mismatch
    bad = _t4(data=good)
    bad.stride_s = 10  # < D
    assert args(bad, k, v, o) == _lib.SAF_ERR_STRIDE
    assert lib.saf_bsa_fwd(ctypes.byref(q), ctypes.byref(k), ctypes.byref(v), ctypes.byref(o), good,
                           good, 16, 128, 128, None, 0, 0.125, -1, None) == _lib.SAF_ERR_ARG


def test_pool_topk_rejects_bad_arguments_on_host(lib):
    q = _t4(data=0x10000)
    cfg = _lib.SelectCfg(128, 128, 4, 0, 0, 0, 0, 0)
    call = lambda q_, k_, cfg_, rp=0x10000: lib.saf_pool_topk(
        ctypes.byref(q_), ctypes.byref(k_), cfg_ if cfg_ is None else ctypes.byref(cfg_), rp, 0x10000,
        None, None, 0x10000, 1 << 20, None)
    assert call(q, q, None) == _lib.SAF_ERR_ARG
    assert call(q, q, cfg, rp=None) == _lib.SAF_ERR_ARG
    assert call(_t4(data=0), q, cfg) == _lib.SAF_ERR_ARG
    assert call(q, _t4(data=0x10000, D=128), cfg) == _lib.SAF_ERR_SHAPE
    unaligned = _t4(data=0x10008)
    assert call(unaligned, unaligned, cfg) == _lib.SAF_ERR_STRIDE
    assert lib.saf_pool_topk_workspace_bytes(ctypes.byref(q), ctypes.byref(q), ctypes.byref(cfg)) > 0


def test_mask_to_csr_rejects_bad_arguments_on_host(lib):
    assert lib.saf_mask_to_csr(None, 1, 4, 4, 16, 4, 0x10000, 0x10000, None) == _lib.SAF_ERR_ARG
    assert lib.saf_mask_to_csr(0x10000, 1, 0, 4, 16, 4, 0x10000, 0x10000, None) == _lib.SAF_ERR_SHAPE
    assert lib.saf_mask_to_csr(0x10000, 1, 4, 4, 16, 2, 0x10000, 0x10000, None) == _lib.SAF_ERR_STRIDE


def test_status_maps_to_exceptions(lib):
    with pytest.raises(ValueError):
        _lib.check("x", _lib.SAF_ERR_SHAPE)
    with pytest.raises(_lib.SafTimeoutError):
        _lib.check("x", _lib.SAF_ERR_TIMEOUT)
    with pytest.raises(_lib.SafError):
        _lib.check("x", _lib.SAF_ERR_CUDA)
    _lib.check("x", _lib.SAF_OK)
