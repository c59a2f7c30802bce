"""ctypes binding of libxe_b200.so (the C ABI in include/xe_b200.h).

The library is built in-tree by ``extended_einsum_b200.build``.  Loading it
never falls back to anything: if the shared object is missing the import of
the ops fails loudly.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().with_name("libxe_b200.so")

XE_OK = 0
XE_ERR_INVALID_ARGUMENT = 1
XE_ERR_NOT_SUPPORTED = 2
XE_ERR_CUDA = 3
XE_ERR_DEVICE_TIMEOUT = 4

XE_SHIFT_MAX = 0
XE_SHIFT_MIN = 1

XE_FIBER_SUM = 0
XE_FIBER_MAX = 1
XE_FIBER_MIN = 2
XE_FIBER_EXP = 3
XE_FIBER_LSE = 4

XE_OP_ADD = 0
XE_OP_SUB = 1
XE_OP_MUL = 2
XE_OP_DIV = 3
XE_OP_MAX = 4
XE_OP_MIN = 5
XE_OP_MUL_EXP = 6
XE_OP_LOG_ADD = 7
XE_OP_RESCALE = 8

_c_i32 = ctypes.c_int32
_c_i64 = ctypes.c_int64
_c_size = ctypes.c_size_t
_c_ptr = ctypes.c_void_p
_c_i64p = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); mirrors include/xe_b200.h
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "xe_version": (ctypes.c_int, []),
    "xe_last_error_string": (ctypes.c_char_p, []),
    "xe_device_status": (ctypes.c_int, [ctypes.c_int]),
    "xe_set_wait_timeout_ns": (_c_i32, [ctypes.c_uint64]),
    "xe_wait_probe": (_c_i32, [_c_i32, _c_ptr]),
    "xe_categorical_scatter_add": (
        _c_i32, [_c_ptr, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_ptr],
    ),
    "xe_logspace_gemm_workspace_size": (_c_size, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i32]),
    "xe_cp_layer_backward_workspace_size": (_c_size, [_c_i64, _c_i64]),
    "xe_cp_layer_backward": (
        _c_i32,
        [
            _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_ptr,  # a, a2, y, g, g_folds, w
            _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i32,  # da, dw, folds, m, shift_mode
            _c_ptr, _c_size, _c_ptr,  # workspace, bytes, stream
        ],
    ),
    "xe_cp_layer_backward_gather_pair": (
        _c_i32,
        [
            _c_ptr, _c_i64, _c_i64,  # table, folds, states
            _c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_i64,  # pixels, strides, variables, var, offset
            _c_ptr, _c_ptr, _c_i64, _c_ptr,  # y, g, g_folds, w
            _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i32,  # da, dw, folds, m, shift_mode
            _c_ptr, _c_size, _c_ptr,  # workspace, bytes, stream
        ],
    ),
    "xe_u8_transpose": (_c_i32, [_c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_ptr]),
    "xe_state_table_pair_grad": (
        _c_i32, [_c_ptr, _c_i64, _c_i64, _c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_i64, _c_i64, _c_ptr, _c_ptr],
    ),
    "xe_logspace_gemm": (
        _c_i32,
        [
            _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i32,  # a, a2, strides, a_linear
            _c_ptr, _c_i64, _c_i64, _c_i64, _c_i32,  # b, strides, b_linear
            _c_ptr, _c_i64, _c_i64, _c_i64,  # c, strides
            _c_i64, _c_i64, _c_i64, _c_i64,  # batch, m, n, k
            _c_i32, _c_ptr, _c_size, _c_ptr,  # shift_mode, workspace, bytes, stream
        ],
    ),
    "xe_logspace_gemm_noalloc": (
        _c_i32,
        [
            _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i32,  # a, a2, strides, a_linear
            _c_ptr, _c_i64, _c_i64, _c_i64, _c_i32,  # b, strides, b_linear
            _c_ptr, _c_i64, _c_i64, _c_i64,  # c, strides
            _c_i64, _c_i64, _c_i64, _c_i64,  # batch, m, n, k
            _c_i32, _c_ptr,  # shift_mode, stream
        ],
    ),
    "xe_logspace_gemm_shifted": (
        _c_i32,
        [
            _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr,  # a, a2, strides, shift_a
            _c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr,  # b, strides, shift_b
            _c_ptr, _c_i64, _c_i64, _c_i64,  # c, strides
            _c_i64, _c_i64, _c_i64, _c_i64, _c_ptr,  # batch, m, n, k, stream
        ],
    ),
    "xe_logspace_gemm_shifted_strided": (
        _c_i32,
        [
            _c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_i64, _c_i64,  # a, strides, shift_a, its strides
            _c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_i64, _c_i64,  # b, strides, shift_b, its strides
            _c_ptr, _c_i64, _c_i64, _c_i64,  # c, strides
            _c_i64, _c_i64, _c_i64, _c_i64, _c_ptr,  # batch, m, n, k, stream
        ],
    ),
    "xe_logspace_b_prepared_size": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "xe_logspace_gemm_workspace_size_prepared": (_c_size, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i32]),
    "xe_logspace_b_prepare": (
        _c_i32,
        [
            _c_ptr, _c_i64, _c_i64, _c_i64, _c_i32,  # b, strides, b_linear
            _c_i64, _c_i64, _c_i64, _c_i32,  # batch, n, k, shift_mode
            _c_ptr, _c_size, _c_ptr, _c_ptr,  # prepared, bytes, shift_b, stream
        ],
    ),
    "xe_logspace_gemm_prepared": (
        _c_i32,
        [
            _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr,  # a, a2, strides, shift_a
            _c_ptr, _c_ptr,  # prepared, shift_b
            _c_ptr, _c_i64, _c_i64, _c_i64,  # c, strides
            _c_i64, _c_i64, _c_i64, _c_i64, _c_ptr,  # batch, m, n, k, stream
        ],
    ),
    "xe_logspace_shift": (
        _c_i32,
        [_c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_ptr, _c_ptr],
    ),
    "xe_logspace_reduce": (
        _c_i32,
        [_c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_ptr, _c_ptr],
    ),
    "xe_softmax": (_c_i32, [_c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i32, _c_ptr]),
    "xe_log_add": (_c_i32, [_c_ptr, _c_i64p, _c_ptr, _c_i64p, _c_ptr, _c_i64p, _c_i32, _c_i32, _c_ptr]),
    "xe_log_add_exp": (
        _c_i32,
        [_c_ptr, _c_i64p, _c_i64, _c_ptr, _c_i64p, _c_i64, _c_ptr, _c_i64p, _c_i32, _c_i32, _c_i32, _c_ptr, _c_ptr],
    ),
    "xe_unary": (_c_i32, [_c_ptr, _c_ptr, _c_i64, _c_i32, _c_ptr]),
    "xe_categorical_gather": (
        _c_i32,
        [_c_ptr, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_ptr],
    ),
    "xe_logspace_tucker": (
        _c_i32,
        [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_ptr],
    ),
    "xe_logspace_tucker_strided": (
        _c_i32,
        [
            _c_ptr, _c_i64, _c_i64, _c_ptr, _c_i64, _c_i64,  # l, strides, r, strides
            _c_ptr, _c_ptr, _c_i64, _c_i64,  # w, y, strides
            _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_ptr,  # batch, folds, I, J, O, shift, stream
        ],
    ),
    "xe_logspace_gemm_gather": (
        _c_i32,
        [
            _c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_i64, _c_ptr,  # table, strides, states, pixels, stride, var
            _c_ptr, _c_i64, _c_i64, _c_i64, _c_i32,  # b, strides, b_linear
            _c_ptr, _c_i64, _c_i64, _c_i64,  # c, strides
            _c_i64, _c_i64, _c_i64, _c_i64,  # folds, batch, n, k
            _c_i32, _c_ptr, _c_size, _c_ptr,  # shift_mode, workspace, bytes, stream
        ],
    ),
    "xe_logspace_gemm_gather_pair": (
        _c_i32,
        [
            _c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_i64, _c_ptr,  # table, strides, states, pixels, stride, var
            _c_i64,  # fold_offset
            _c_ptr, _c_i64, _c_i64, _c_i64, _c_i32,  # b, strides, b_linear
            _c_ptr, _c_i64, _c_i64, _c_i64,  # c, strides
            _c_i64, _c_i64, _c_i64, _c_i64,  # folds, batch, n, k
            _c_i32, _c_ptr, _c_size, _c_ptr,  # shift_mode, workspace, bytes, stream
        ],
    ),
    "xe_scaled_gemm": (
        _c_i32,
        [
            _c_ptr, _c_i64, _c_i64, _c_i64,  # a, strides
            _c_ptr, _c_i64, _c_i64, _c_i64,  # b, strides
            _c_ptr, _c_i64, _c_i64, _c_i64,  # c, strides
            _c_i64, _c_i64, _c_i64, _c_i64, _c_ptr,  # batch, m, n, k, stream
        ],
    ),
    "xe_fiber_normalize": (_c_i32, [_c_ptr, _c_i64p, _c_i64p, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_ptr]),
    "xe_reduce": (_c_i32, [_c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_ptr, _c_ptr]),
    "xe_elementwise": (
        _c_i32,
        [_c_i32, _c_ptr, _c_i64p, _c_ptr, _c_i64p, _c_ptr, _c_i64p, _c_ptr, _c_i64p, _c_i32, _c_ptr],
    ),
}

_lock = threading.Lock()
_handle: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads libxe_b200.so once and declares every entry point's signature."""
    global _handle
    if _handle is not None:
        return _handle
    with _lock:
        if _handle is None:
            if not LIBRARY_PATH.exists():
                raise ImportError(
                    f"{LIBRARY_PATH.name} is not built; run `python -m extended_einsum_b200.build` "
                    "(nvcc, sm_100a) before using the B200 kernels"
                )
            handle = ctypes.CDLL(str(LIBRARY_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _handle = handle
    return _handle


def last_error() -> str:
    msg = load().xe_last_error_string()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    """Turns a non-OK xe_status into the exception the reference raises for it."""
    if status == XE_OK:
        return
    message = f"{what}: {last_error()}"
    if status == XE_ERR_INVALID_ARGUMENT:
        raise ValueError(message)
    if status == XE_ERR_NOT_SUPPORTED:
        raise NotImplementedError(message)
    raise RuntimeError(message)


def int64_array(values) -> ctypes.Array:
    values = [int(v) for v in values]
    return (ctypes.c_int64 * max(1, len(values)))(*values)
