"""The C-ABI library: it loads, exports every entry point that include/xe_b200.h
declares, and rejects invalid arguments before touching the device (no GPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from extended_einsum_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "xe_b200.h"


def header_functions() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"\b(xe_\w+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = header_functions()
    assert len(declared) >= 12
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in xe_b200.h but not exported"


def test_binding_covers_the_header():
    assert set(_lib.SIGNATURES) == header_functions()


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.xe_version() == 100
    assert isinstance(_lib.last_error(), str)


def test_workspace_size():
    lib = _lib.load()
    assert lib.xe_logspace_gemm_workspace_size(2, 100, 30, 8, 0, 0) == 1024 + 256
    assert lib.xe_logspace_gemm_workspace_size(2, 100, 30, 8, 1, 1) == 0
    assert lib.xe_logspace_gemm_workspace_size(1, 64, 64, 8, 1, 0) == 256


def _gemm(lib, a=1, b=1, c=1, k=4, mode=0, a2=None, a_linear=0, ws=0, ws_bytes=0):
    return lib.xe_logspace_gemm(a, a2, 0, 4, 1, a_linear, b, 0, 4, 1, 0, c, 0, 4, 1, 1, 4, 4, k, mode, ws, ws_bytes, None)


def test_invalid_arguments_are_rejected_without_launch():
    lib = _lib.load()
    assert _gemm(lib, a=None) == _lib.XE_ERR_INVALID_ARGUMENT
    assert "null" in _lib.last_error()
    assert _gemm(lib, k=0) == _lib.XE_ERR_INVALID_ARGUMENT
    assert _gemm(lib, mode=7) == _lib.XE_ERR_INVALID_ARGUMENT
    assert _gemm(lib, a2=1, a_linear=1) == _lib.XE_ERR_INVALID_ARGUMENT
    assert _gemm(lib, ws=0, ws_bytes=0) == _lib.XE_ERR_INVALID_ARGUMENT  # shifts need a workspace
    assert "workspace" in _lib.last_error()
    assert lib.xe_softmax(None, None, 1, 1, 1, 0, None) == _lib.XE_ERR_INVALID_ARGUMENT
    shape = _lib.int64_array([1] * 7)
    assert lib.xe_log_add(1, shape, 1, shape, 1, shape, 7, 0, None) == _lib.XE_ERR_NOT_SUPPORTED
    assert lib.xe_unary(1, 1, 4, 9, None) == _lib.XE_ERR_INVALID_ARGUMENT
    assert lib.xe_categorical_gather(1, 1, 1, None, 1, 1, 300, 4, 1, None) == _lib.XE_ERR_INVALID_ARGUMENT
    assert lib.xe_logspace_reduce(1, 0, 1, 1, 1, 1, 0, 0, 1, None) == _lib.XE_ERR_INVALID_ARGUMENT
    pair = (1, 64, 64, 4, 1, 8, None)  # table, strides, states, pixels, stride, var
    tail = (1, 256, 1, 64, 1, 1, 256, 64, 1, 2, 4, 4, 64, 0, None, 0, None)
    assert lib.xe_logspace_gemm_gather_pair(*pair, 0, *tail) == _lib.XE_ERR_INVALID_ARGUMENT
    assert "fold_offset" in _lib.last_error()
    assert lib.xe_logspace_gemm_gather_pair(*pair[:3], 300, *pair[4:], 2, *tail) == _lib.XE_ERR_INVALID_ARGUMENT


def test_status_maps_to_reference_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.XE_ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.XE_ERR_NOT_SUPPORTED, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.XE_ERR_CUDA, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.XE_ERR_DEVICE_TIMEOUT, "x")
    _lib.check(_lib.XE_OK, "x")


def test_wait_limit_range_is_checked_before_the_device():
    lib = _lib.load()
    assert lib.xe_set_wait_timeout_ns(999) == _lib.XE_ERR_INVALID_ARGUMENT
    assert "outside" in _lib.last_error()
    assert lib.xe_set_wait_timeout_ns(60_000_000_001) == _lib.XE_ERR_INVALID_ARGUMENT


def test_cp_layer_backward_rejects_bad_arguments_without_launch():
    lib = _lib.load()
    ws = lib.xe_cp_layer_backward_workspace_size(4, 100)
    assert ws > 0 and ws % 256 == 0 and lib.xe_cp_layer_backward_workspace_size(0, 100) == 0

    def call(a=16, y=16, g=16, g_folds=1, w=16, mode=0, folds=2, m=100, ws_bytes=1 << 30):
        return lib.xe_cp_layer_backward(a, None, y, g, g_folds, w, 16, 16, folds, m, mode, 16, ws_bytes, None)

    assert call(a=None) == _lib.XE_ERR_INVALID_ARGUMENT and "null" in _lib.last_error()
    assert call(g_folds=0) == _lib.XE_ERR_INVALID_ARGUMENT
    assert call(mode=3) == _lib.XE_ERR_INVALID_ARGUMENT
    assert call(m=-1) == _lib.XE_ERR_INVALID_ARGUMENT
    assert call(ws_bytes=16) == _lib.XE_ERR_INVALID_ARGUMENT and "workspace" in _lib.last_error()
    # the pair form checks its table and indices first
    st = lib.xe_cp_layer_backward_gather_pair(16, 3, 256, 16, 8, 1, 8, None, 2, 16, 16, 1, 16, 16, 16, 2, 100, 0, 16,
                                              1 << 30, None)
    assert st == _lib.XE_ERR_INVALID_ARGUMENT and "folds" in _lib.last_error()
    assert lib.xe_state_table_pair_grad(16, 2, 10, 16, 8, 1, 8, None, 2, 300, 16, None) == _lib.XE_ERR_NOT_SUPPORTED
    assert lib.xe_state_table_pair_grad(None, 2, 10, 16, 8, 1, 8, None, 2, 256, 16, None) == _lib.XE_ERR_INVALID_ARGUMENT
