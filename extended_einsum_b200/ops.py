"""Torch-tensor entry points over the sm_100a C ABI.

Each function validates its operands (CUDA, float32, one device), allocates
the outputs and the scratch buffers with torch's caching allocator, and calls
one entry point of libxe_b200.so on torch's current stream.  There is no CPU
path: a CPU tensor is a ValueError, exactly like an unsupported shape in the
reference raises instead of silently switching implementations.
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import torch

from . import _lib

SHIFT_MODES = {"max": _lib.XE_SHIFT_MAX, "min": _lib.XE_SHIFT_MIN}


def _check_tensors(what: str, *tensors: torch.Tensor) -> torch.device:
    device = None
    for t in tensors:
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{what}: expected torch.Tensor, got {type(t).__name__}")
        if t.device.type != "cuda":
            raise ValueError(f"{what}: the B200 kernels take CUDA tensors, got a tensor on {t.device}")
        if t.dtype != torch.float32:
            raise NotImplementedError(f"{what}: only float32 is implemented, got {t.dtype}")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError(f"{what}: tensors on different devices ({device} and {t.device})")
    assert device is not None
    return device


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _shift(mode: str) -> int:
    try:
        return SHIFT_MODES[mode]
    except KeyError:
        raise ValueError(f"unknown shift mode {mode!r}; expected 'max' or 'min'") from None


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _needs_grad(*tensors: torch.Tensor | None) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def _no_backward(what: str, *tensors: torch.Tensor | None) -> None:
    if _needs_grad(*tensors):
        raise NotImplementedError(f"{what}: no backward pass on this path")


# ---------------------------------------------------------------------------
# log-space contraction


def logspace_gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    a2: torch.Tensor | None = None,
    a_linear: bool = False,
    b_linear: bool = False,
    shift: str = "max",
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """C[t,m,n] = log(sum_k A'[t,m,k] B'[t,k,n]) + shifts (xe_logspace_gemm).

    ``a`` is (batch, M, K) and ``b`` (batch, K, N), any strides; a log-domain
    operand X enters as exp(X - shift) with shift = max (or min) over k and the
    shift is added back, a linear operand enters as is.  ``a2`` (same shape
    and strides as ``a``) is added to ``a`` in the log domain first.
    Differentiable (autograd.LogspaceGemm) when an operand requires grad.
    """
    if out is None and _needs_grad(a, b, a2):
        from .autograd import LogspaceGemm

        return LogspaceGemm.apply(a, b, a2, a_linear, b_linear, shift)
    tensors = [a, b] + ([a2] if a2 is not None else []) + ([out] if out is not None else [])
    device = _check_tensors("logspace_gemm", *tensors)
    if a.dim() != 3 or b.dim() != 3:
        raise ValueError("logspace_gemm: operands must be 3-D (batch, M, K) and (batch, K, N)")
    batch, m, k = a.shape
    if b.shape[0] != batch or b.shape[1] != k:
        raise ValueError(f"logspace_gemm: incompatible shapes {tuple(a.shape)} and {tuple(b.shape)}")
    n = b.shape[2]
    if a2 is not None and (a2.shape != a.shape or a2.stride() != a.stride()):
        raise ValueError("logspace_gemm: the fused addend must have the shape and strides of A")
    if out is None:
        out = torch.empty((batch, m, n), device=device, dtype=torch.float32)
    elif out.shape != (batch, m, n):
        raise ValueError(f"logspace_gemm: out has shape {tuple(out.shape)}, expected {(batch, m, n)}")
    lib = _lib.load()
    # room for the prepared B too, where the contraction prepares it (xe_logspace_b_prepare)
    ws_bytes = lib.xe_logspace_gemm_workspace_size_prepared(batch, m, n, k, int(a_linear), int(b_linear))
    ws = torch.empty(ws_bytes, device=device, dtype=torch.uint8) if ws_bytes else None
    status = lib.xe_logspace_gemm(
        a.data_ptr(), _ptr(a2), a.stride(0), a.stride(1), a.stride(2), int(a_linear),
        b.data_ptr(), b.stride(0), b.stride(1), b.stride(2), int(b_linear),
        out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
        batch, m, n, k, _shift(shift), _ptr(ws), ws_bytes, _stream(device),
    )
    _lib.check(status, "xe_logspace_gemm")
    return out


def logspace_gemm_shifted(
    a: torch.Tensor,
    b: torch.Tensor,
    shift_a: torch.Tensor | None,
    shift_b: torch.Tensor | None,
    *,
    a2: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """The contraction kernel alone with given shifts (None = linear operand), xe_logspace_gemm_shifted."""
    _no_backward("logspace_gemm_shifted", a, b)
    extra = [t for t in (a2, out, shift_a, shift_b) if t is not None]
    device = _check_tensors("logspace_gemm_shifted", a, b, *extra)
    batch, m, k = a.shape
    n = b.shape[2]
    if b.shape[:2] != (batch, k):
        raise ValueError(f"logspace_gemm_shifted: incompatible shapes {tuple(a.shape)} and {tuple(b.shape)}")
    for s, size in ((shift_a, m), (shift_b, n)):
        if s is not None and (not s.is_contiguous() or s.numel() != batch * size):
            raise ValueError("logspace_gemm_shifted: shifts must be contiguous (batch, rows) vectors")
    if out is None:
        out = torch.empty((batch, m, n), device=device, dtype=torch.float32)
    status = _lib.load().xe_logspace_gemm_shifted(
        a.data_ptr(), _ptr(a2), a.stride(0), a.stride(1), a.stride(2), _ptr(shift_a),
        b.data_ptr(), b.stride(0), b.stride(1), b.stride(2), _ptr(shift_b),
        out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
        batch, m, n, k, _stream(device),
    )
    _lib.check(status, "xe_logspace_gemm_shifted")
    return out


def logspace_gemm_shifted_strided(
    a: torch.Tensor, b: torch.Tensor, shift_a: torch.Tensor, sa_strides: tuple[int, int], shift_b: torch.Tensor,
    sb_strides: tuple[int, int], *, out: torch.Tensor | None = None,
) -> torch.Tensor:
    """The contraction of two log-domain operands with caller-chosen shifts
    (xe_logspace_gemm_shifted_strided): row m of batch entry t is shifted by
    shift_a[t * sa_strides[0] + m * sa_strides[1]], column n by shift_b[t * sb_strides[0] + n * sb_strides[1]]."""
    _no_backward("logspace_gemm_shifted_strided", a, b)
    device = _check_tensors("logspace_gemm_shifted_strided", a, b, shift_a, shift_b, *([out] if out is not None else []))
    batch, m, k = a.shape
    n = b.shape[2]
    if b.shape[:2] != (batch, k):
        raise ValueError(f"logspace_gemm_shifted_strided: incompatible shapes {tuple(a.shape)} and {tuple(b.shape)}")
    for s, (st_b, st_r), rows in ((shift_a, sa_strides, m), (shift_b, sb_strides, n)):
        if not s.is_contiguous() or (batch - 1) * st_b + (rows - 1) * st_r >= s.numel():
            raise ValueError("logspace_gemm_shifted_strided: a shift vector is shorter than its strides address")
    if out is None:
        out = torch.empty((batch, m, n), device=device, dtype=torch.float32)
    status = _lib.load().xe_logspace_gemm_shifted_strided(
        a.data_ptr(), a.stride(0), a.stride(1), a.stride(2), shift_a.data_ptr(), sa_strides[0], sa_strides[1],
        b.data_ptr(), b.stride(0), b.stride(1), b.stride(2), shift_b.data_ptr(), sb_strides[0], sb_strides[1],
        out.data_ptr(), out.stride(0), out.stride(1), out.stride(2), batch, m, n, k, _stream(device),
    )
    _lib.check(status, "xe_logspace_gemm_shifted_strided")
    return out


class PreparedB:
    """A B operand prepared once (xe_logspace_b_prepare) for contractions against several A.

    ``b`` is (batch, K, N) with N or K contiguous; a log-domain B enters as exp(B - shift) with its
    column shift (max or min over k), a linear one as is.  ``logspace_gemm_prepared`` contracts an A
    with it; the result equals ``logspace_gemm(a, b, ...)`` bit for bit.
    """

    def __init__(self, b: torch.Tensor, *, linear: bool = False, shift: str = "max") -> None:
        _no_backward("PreparedB", b)
        device = _check_tensors("PreparedB", b)
        if b.dim() != 3:
            raise ValueError("PreparedB: expected a (batch, K, N) tensor")
        batch, k, n = b.shape
        lib = _lib.load()
        self.shape = (batch, k, n)
        self.linear = linear
        # opaque: the tiled hi / lo stages (a multiple of 32 KB), held as float32
        self.buffer = torch.empty(lib.xe_logspace_b_prepared_size(batch, n, k) // 4, device=device, dtype=torch.float32)
        self.shift = None if linear else torch.empty((batch, n), device=device, dtype=torch.float32)
        status = lib.xe_logspace_b_prepare(
            b.data_ptr(), b.stride(0), b.stride(1), b.stride(2), int(linear), batch, n, k, _shift(shift),
            self.buffer.data_ptr(), self.buffer.numel() * 4, _ptr(self.shift), _stream(device),
        )
        _lib.check(status, "xe_logspace_b_prepare")


def logspace_gemm_prepared(
    a: torch.Tensor,
    prepared: PreparedB,
    shift_a: torch.Tensor | None,
    *,
    a2: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """The contraction kernel with a prepared B (xe_logspace_gemm_prepared); shift_a None = linear A."""
    _no_backward("logspace_gemm_prepared", a)
    extra = [t for t in (a2, out, shift_a) if t is not None]
    device = _check_tensors("logspace_gemm_prepared", a, prepared.buffer, *extra)
    batch, m, k = a.shape
    if prepared.shape[:2] != (batch, k):
        raise ValueError(f"logspace_gemm_prepared: A {tuple(a.shape)} does not match the prepared B {prepared.shape}")
    n = prepared.shape[2]
    if shift_a is not None and (not shift_a.is_contiguous() or shift_a.numel() != batch * m):
        raise ValueError("logspace_gemm_prepared: shift_a must be a contiguous (batch, M) vector")
    if out is None:
        out = torch.empty((batch, m, n), device=device, dtype=torch.float32)
    status = _lib.load().xe_logspace_gemm_prepared(
        a.data_ptr(), _ptr(a2), a.stride(0), a.stride(1), a.stride(2), _ptr(shift_a),
        prepared.buffer.data_ptr(), _ptr(prepared.shift),
        out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
        batch, m, n, k, _stream(device),
    )
    _lib.check(status, "xe_logspace_gemm_prepared")
    return out


def logspace_shift(x: torch.Tensor, *, shift: str = "max", x2: torch.Tensor | None = None) -> torch.Tensor:
    """Per-row max (or min) over the last axis of a (batch, rows, k) view."""
    device = _check_tensors("logspace_shift", x, *([x2] if x2 is not None else []))
    if x.dim() != 3:
        raise ValueError("logspace_shift: expected a (batch, rows, k) tensor")
    batch, rows, k = x.shape
    out = torch.empty((batch, rows), device=device, dtype=torch.float32)
    status = _lib.load().xe_logspace_shift(
        x.data_ptr(), _ptr(x2), x.stride(0), x.stride(1), x.stride(2), batch, rows, k, _shift(shift),
        out.data_ptr(), _stream(device),
    )
    _lib.check(status, "xe_logspace_shift")
    return out


def logspace_reduce(x: torch.Tensor, *, shift: str = "max") -> torch.Tensor:
    """y[t,r] = log(sum_k exp(x[t,r,k] - s)) + s over a (batch, rows, k) view."""
    if _needs_grad(x):
        from .autograd import LogspaceReduce

        return LogspaceReduce.apply(x, shift)
    device = _check_tensors("logspace_reduce", x)
    if x.dim() != 3:
        raise ValueError("logspace_reduce: expected a (batch, rows, k) tensor")
    batch, rows, k = x.shape
    out = torch.empty((batch, rows), device=device, dtype=torch.float32)
    status = _lib.load().xe_logspace_reduce(
        x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), batch, rows, k, _shift(shift), out.data_ptr(),
        _stream(device),
    )
    _lib.check(status, "xe_logspace_reduce")
    return out


# ---------------------------------------------------------------------------
# softmax


def softmax(x: torch.Tensor, axis: int | Sequence[int], *, log_output: bool = False) -> torch.Tensor:
    """Softmax over one axis or a set of axes (TorchBackendFunctions.softmax semantics).

    A consecutive block of axes is flattened into one reduced axis (as
    backends/torch.py:107-110 does for a trailing block); other axis sets are
    moved to the end first.
    """
    if _needs_grad(x):
        from .autograd import Softmax

        return Softmax.apply(x, axis, log_output)
    device = _check_tensors("softmax", x)
    if x.dim() == 0:
        raise ValueError("softmax requires an input tensor with at least one axis")
    axes = (axis,) if isinstance(axis, int) else tuple(axis)
    if not axes:
        raise ValueError("softmax requires at least one axis")
    nd = x.dim()
    axes = tuple(sorted(a + nd if a < 0 else a for a in axes))
    if any(not 0 <= a < nd for a in axes) or len(set(axes)) != len(axes):
        raise ValueError(f"softmax axes {axis} are invalid for a {nd}-D tensor")
    permuted = None
    if axes != tuple(range(axes[0], axes[-1] + 1)):
        keep = [d for d in range(nd) if d not in axes]
        permuted = keep + list(axes)
        x = x.permute(permuted)
        axes = tuple(range(nd - len(axes), nd))
    x = x.contiguous()
    shape = x.shape
    outer = math.prod(shape[: axes[0]])
    length = math.prod(shape[axes[0] : axes[-1] + 1])
    inner = math.prod(shape[axes[-1] + 1 :])
    y = torch.empty_like(x)
    status = _lib.load().xe_softmax(x.data_ptr(), y.data_ptr(), outer, length, inner, int(log_output), _stream(device))
    _lib.check(status, "xe_softmax")
    if permuted is not None:
        inverse = [0] * nd
        for i, d in enumerate(permuted):
            inverse[d] = i
        y = y.permute(inverse)
    return y


# ---------------------------------------------------------------------------
# elementwise log-space arithmetic


def _broadcast_strides(t: torch.Tensor, shape: torch.Size) -> list[int]:
    return list(t.expand(shape).stride())


def log_add(a: torch.Tensor, b: torch.Tensor, *, negate_b: bool = False) -> torch.Tensor:
    """y = a + b (or a - b) with numpy broadcasting: a log-space product (quotient)."""
    if _needs_grad(a, b):
        from .autograd import LogAdd

        return LogAdd.apply(a, b, negate_b)
    device = _check_tensors("log_add", a, b)
    shape = torch.broadcast_shapes(a.shape, b.shape)
    if len(shape) > 6:
        raise NotImplementedError(f"log_add: rank {len(shape)} above 6 is not supported")
    y = torch.empty(shape, device=device, dtype=torch.float32)
    status = _lib.load().xe_log_add(
        a.data_ptr(), _lib.int64_array(_broadcast_strides(a, shape)),
        b.data_ptr(), _lib.int64_array(_broadcast_strides(b, shape)),
        y.data_ptr(), _lib.int64_array(shape), len(shape), int(negate_b), _stream(device),
    )
    _lib.check(status, "xe_log_add")
    return y


def log_add_exp(a: torch.Tensor, b: torch.Tensor, *, subtract: bool = False, shift: str = "max") -> torch.Tensor:
    """y = log(exp(a - m) +/- exp(b - m)) + m with the scalar m = extreme of a and b.

    Differentiable (autograd.LogAddExp, m detached) when an operand requires grad."""
    if _needs_grad(a, b):
        from .autograd import LogAddExp

        return LogAddExp.apply(a, b, subtract, shift)
    device = _check_tensors("log_add_exp", a, b)
    a = a.contiguous()
    b = b.contiguous()
    shape = torch.broadcast_shapes(a.shape, b.shape)
    if len(shape) > 6:
        raise NotImplementedError(f"log_add_exp: rank {len(shape)} above 6 is not supported")
    y = torch.empty(shape, device=device, dtype=torch.float32)
    scratch = torch.empty(1, device=device, dtype=torch.float32)
    status = _lib.load().xe_log_add_exp(
        a.data_ptr(), _lib.int64_array(_broadcast_strides(a, shape)), a.numel(),
        b.data_ptr(), _lib.int64_array(_broadcast_strides(b, shape)), b.numel(),
        y.data_ptr(), _lib.int64_array(shape), len(shape), int(subtract), _shift(shift), scratch.data_ptr(),
        _stream(device),
    )
    _lib.check(status, "xe_log_add_exp")
    return y


def _unary(x: torch.Tensor, op: int, what: str) -> torch.Tensor:
    device = _check_tensors(what, x)
    x = x.contiguous()
    y = torch.empty_like(x)
    _lib.check(_lib.load().xe_unary(x.data_ptr(), y.data_ptr(), x.numel(), op, _stream(device)), what)
    return y


def exp(x: torch.Tensor) -> torch.Tensor:
    """Log space -> raw (translate.py:631-636)."""
    if _needs_grad(x):
        from .autograd import Exp

        return Exp.apply(x)
    return _unary(x, 0, "exp")


def log(x: torch.Tensor) -> torch.Tensor:
    """Raw -> log space (translate.py:639-644)."""
    if _needs_grad(x):
        from .autograd import Log

        return Log.apply(x)
    return _unary(x, 1, "log")


# ---------------------------------------------------------------------------
# circuit inputs


def categorical_gather(
    log_table: torch.Tensor, pixels: torch.Tensor, var_of_fold: torch.Tensor | None = None
) -> torch.Tensor:
    """y[f,b,:] = log_table[f, pixels[b, var_of_fold[f]], :] for uint8 pixels (batch, variables).

    Differentiable in the table (autograd.CategoricalGather: a scatter-add)."""
    if _needs_grad(log_table):
        from .autograd import CategoricalGather

        return CategoricalGather.apply(log_table, pixels, var_of_fold)
    device = _check_tensors("categorical_gather", log_table)
    if pixels.device != device or pixels.dtype != torch.uint8 or pixels.dim() != 2:
        raise ValueError("categorical_gather: pixels must be a (batch, variables) uint8 tensor on the table's device")
    if pixels.stride(1) != 1:
        pixels = pixels.contiguous()
    folds, states, units = log_table.shape
    log_table = log_table.contiguous()
    batch = pixels.shape[0]
    if var_of_fold is not None:
        if var_of_fold.dtype != torch.int32 or var_of_fold.device != device or var_of_fold.numel() != folds:
            raise ValueError("categorical_gather: var_of_fold must be int32 with one entry per fold")
        var_of_fold = var_of_fold.contiguous()
    elif pixels.shape[1] < folds:
        raise ValueError("categorical_gather: fewer pixel variables than folds")
    y = torch.empty((folds, batch, units), device=device, dtype=torch.float32)
    status = _lib.load().xe_categorical_gather(
        log_table.data_ptr(), pixels.data_ptr(), pixels.stride(0), _ptr(var_of_fold), y.data_ptr(),
        folds, states, units, batch, _stream(device),
    )
    _lib.check(status, "xe_categorical_gather")
    return y


def categorical_scatter_add(
    grad: torch.Tensor,
    pixels: torch.Tensor,
    var_of_fold: torch.Tensor | None,
    table_grad: torch.Tensor,
    *,
    fold_offset: int = 0,
) -> torch.Tensor:
    """table_grad[f + off, pixels[b, var[f + off]], :] += grad[f, b, :] (xe_categorical_scatter_add), in place.

    The backward of categorical_gather: ``grad`` is (folds, batch, units), ``table_grad`` a
    contiguous (>= off + folds, states, units) accumulator."""
    device = _check_tensors("categorical_scatter_add", grad, table_grad)
    if pixels.device != device or pixels.dtype != torch.uint8 or pixels.dim() != 2:
        raise ValueError("categorical_scatter_add: pixels must be a (batch, variables) uint8 tensor on the table's device")
    if pixels.stride(1) != 1:
        pixels = pixels.contiguous()
    if grad.dim() != 3 or table_grad.dim() != 3 or not table_grad.is_contiguous():
        raise ValueError("categorical_scatter_add: expected a (folds, batch, units) gradient and a contiguous table")
    folds, batch, units = grad.shape
    table_folds, states, table_units = table_grad.shape
    if table_units != units or table_folds < fold_offset + folds or pixels.shape[0] != batch:
        raise ValueError("categorical_scatter_add: incompatible shapes")
    if var_of_fold is not None:
        if var_of_fold.dtype != torch.int32 or var_of_fold.device != device or var_of_fold.numel() < fold_offset + folds:
            raise ValueError("categorical_scatter_add: var_of_fold must be int32 with an entry per table fold")
        var_of_fold = var_of_fold.contiguous()
    elif pixels.shape[1] < fold_offset + folds:
        raise ValueError("categorical_scatter_add: fewer pixel variables than table folds")
    grad = grad.contiguous()
    status = _lib.load().xe_categorical_scatter_add(
        grad.data_ptr(), pixels.data_ptr(), pixels.stride(0), _ptr(var_of_fold), table_grad.data_ptr(),
        folds, states, units, batch, fold_offset, _stream(device),
    )
    _lib.check(status, "xe_categorical_scatter_add")
    return table_grad


def logspace_gemm_gather(
    log_table: torch.Tensor,
    pixels: torch.Tensor,
    var_of_fold: torch.Tensor | None,
    b: torch.Tensor,
    *,
    b_linear: bool = False,
    shift: str = "max",
) -> torch.Tensor:
    """C[f,b,n] = log(sum_k exp(T[f, pixels[b, var[f]], k] - s) B'[f,k,n]) + shifts (xe_logspace_gemm_gather).

    The categorical input gather fused into the first sum layer: ``log_table``
    is (folds, states, K) with K contiguous, ``pixels`` (batch, variables)
    uint8, ``b`` (folds, K, N).  Returns (folds, batch, N).
    """
    return _gather_gemm("logspace_gemm_gather", log_table, pixels, var_of_fold, b, 0, b_linear, shift)


def logspace_gemm_gather_pair(
    state_table: torch.Tensor,
    pixels: torch.Tensor,
    var_of_fold: torch.Tensor | None,
    b: torch.Tensor,
    *,
    b_linear: bool = False,
    shift: str = "max",
) -> torch.Tensor:
    """The sum layer over the Hadamard product of two gathered halves (xe_logspace_gemm_gather_pair).

    ``state_table`` is (2F, states, K): row (f, s) is the log-domain output
    of the previous layer for pixel value s of fold f's variable.  With
    A[f,b,:] = T[f, pixels[b, var[f]], :] + T[f+F, pixels[b, var[f+F]], :],
    returns C[f,b,n] = log(sum_k exp(A[f,b,k] - s) B'[f,k,n]) + shifts, (F, batch, N)
    for ``b`` (F, K, N).
    """
    if state_table.dim() != 3 or state_table.shape[0] % 2:
        raise ValueError("logspace_gemm_gather_pair: expected a (2F, states, K) state table")
    return _gather_gemm("logspace_gemm_gather_pair", state_table, pixels, var_of_fold, b,
                        state_table.shape[0] // 2, b_linear, shift)


def _gather_gemm(name, log_table, pixels, var_of_fold, b, fold_offset, b_linear, shift):
    if _needs_grad(log_table, b):
        from .autograd import LogspaceGemmGather

        return LogspaceGemmGather.apply(log_table, pixels, var_of_fold, b, b_linear, shift, fold_offset > 0)
    device = _check_tensors(name, log_table, b)
    if pixels.device != device or pixels.dtype != torch.uint8 or pixels.dim() != 2:
        raise ValueError(f"{name}: pixels must be a (batch, variables) uint8 tensor on the table's device")
    if pixels.stride(1) != 1:
        pixels = pixels.contiguous()
    if log_table.dim() != 3 or b.dim() != 3:
        raise ValueError(f"{name}: expected a (folds, states, K) table and a (folds, K, N) operand")
    if log_table.stride(2) != 1:
        log_table = log_table.contiguous()
    table_folds, states, k = log_table.shape
    folds = table_folds - fold_offset
    if b.shape[0] != folds or b.shape[1] != k:
        raise ValueError(f"{name}: incompatible shapes {tuple(log_table.shape)} and {tuple(b.shape)}")
    if var_of_fold is not None:
        if var_of_fold.dtype != torch.int32 or var_of_fold.device != device or var_of_fold.numel() != table_folds:
            raise ValueError(f"{name}: var_of_fold must be int32 with one entry per table fold")
        var_of_fold = var_of_fold.contiguous()
    elif pixels.shape[1] < table_folds:
        raise ValueError(f"{name}: fewer pixel variables than table folds")
    batch = pixels.shape[0]
    n = b.shape[2]
    out = torch.empty((folds, batch, n), device=device, dtype=torch.float32)
    lib = _lib.load()
    ws_bytes = lib.xe_logspace_gemm_workspace_size(folds, batch, n, k, 1, int(b_linear))
    ws = torch.empty(ws_bytes, device=device, dtype=torch.uint8) if ws_bytes else None
    head = (log_table.data_ptr(), log_table.stride(0), log_table.stride(1), states, pixels.data_ptr(),
            pixels.stride(0), _ptr(var_of_fold))
    tail = (b.data_ptr(), b.stride(0), b.stride(1), b.stride(2), int(b_linear),
            out.data_ptr(), out.stride(0), out.stride(1), out.stride(2), folds, batch, n, k, _shift(shift),
            _ptr(ws), ws_bytes, _stream(device))
    if fold_offset:
        status = lib.xe_logspace_gemm_gather_pair(*head, fold_offset, *tail)
    else:
        status = lib.xe_logspace_gemm_gather(*head, *tail)
    _lib.check(status, "xe_" + name)
    return out


def cp_layer_backward(
    a: torch.Tensor,
    y: torch.Tensor,
    g: torch.Tensor,
    w: torch.Tensor,
    *,
    a2: torch.Tensor | None = None,
    shift: str = "max",
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gradients of the folded CP sum layer y = logspace_gemm(a, w.permute(0, 2, 1), a2=a2,
    b_linear=True) (xe_cp_layer_backward): returns (dA, dw), dA also the gradient of a2.

    a, a2, y are (F, M, 64); g is dL/dy, (F, M, 64) or (F / r, M, 64) with fold f reading
    g[f % g.shape[0]] (the next layer's dA, the gradient of both halves of its input); w is the
    (F, 64, 64) linear weights (o, k).  All contiguous float32 on one device.
    """
    device = _check_tensors("cp_layer_backward", a, y, g, w, *([a2] if a2 is not None else []))
    folds, m, _ = _cp_backward_shapes("cp_layer_backward", a, y, g, w)
    if a2 is not None and (tuple(a2.shape) != tuple(a.shape) or not a2.is_contiguous()):
        raise ValueError("cp_layer_backward: a2 must be contiguous with a's shape")
    da = torch.empty_like(y)
    dw = torch.empty_like(w)
    lib = _lib.load()
    ws_bytes = lib.xe_cp_layer_backward_workspace_size(folds, m)
    ws = torch.empty(ws_bytes, device=device, dtype=torch.uint8) if ws_bytes else None
    status = lib.xe_cp_layer_backward(a.data_ptr(), _ptr(a2), y.data_ptr(), g.data_ptr(), g.shape[0], w.data_ptr(),
                                      da.data_ptr(), dw.data_ptr(), folds, m, _shift(shift), _ptr(ws), ws_bytes,
                                      _stream(device))
    _lib.check(status, "xe_cp_layer_backward")
    return da, dw


def cp_layer_backward_gather_pair(
    state_table: torch.Tensor,
    pixels: torch.Tensor,
    var_of_fold: torch.Tensor | None,
    y: torch.Tensor,
    g: torch.Tensor,
    w: torch.Tensor,
    *,
    shift: str = "max",
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gradients of y = logspace_gemm_gather_pair(state_table, pixels, var_of_fold, w^T, b_linear=True)
    (xe_cp_layer_backward_gather_pair): returns (dA, dw), dA (F, batch, 64) the gradient of both
    gathered rows (state_table_pair_grad turns it into the table's gradient)."""
    device = _check_tensors("cp_layer_backward_gather_pair", state_table, y, g, w)
    folds, m, _ = _cp_backward_shapes("cp_layer_backward_gather_pair", y, y, g, w)
    pixels, var_of_fold = _pair_indices("cp_layer_backward_gather_pair", state_table, pixels, var_of_fold, folds, m,
                                        device)
    da = torch.empty_like(y)
    dw = torch.empty_like(w)
    lib = _lib.load()
    ws_bytes = lib.xe_cp_layer_backward_workspace_size(folds, m)
    ws = torch.empty(ws_bytes, device=device, dtype=torch.uint8) if ws_bytes else None
    status = lib.xe_cp_layer_backward_gather_pair(
        state_table.data_ptr(), state_table.shape[0], state_table.shape[1], pixels.data_ptr(), pixels.stride(0),
        pixels.stride(1), pixels.shape[1], _ptr(var_of_fold), folds, y.data_ptr(), g.data_ptr(), g.shape[0],
        w.data_ptr(), da.data_ptr(), dw.data_ptr(), folds, m, _shift(shift), _ptr(ws), ws_bytes, _stream(device))
    _lib.check(status, "xe_cp_layer_backward_gather_pair")
    return da, dw


def state_table_pair_grad(
    da: torch.Tensor, pixels: torch.Tensor, var_of_fold: torch.Tensor | None, states: int
) -> torch.Tensor:
    """The (2F, states, 64) gradient of the state table from dA (F, batch, 64) (xe_state_table_pair_grad):
    row (t, s) sums dA[t mod F, b] over the samples b whose pixel of variable var[t] is s."""
    device = _check_tensors("state_table_pair_grad", da)
    if da.dim() != 3 or not da.is_contiguous():
        raise ValueError("state_table_pair_grad: dA must be a contiguous (F, batch, units) tensor")
    folds, m, units = da.shape
    table = torch.empty((2 * folds, states, units), device=device, dtype=torch.float32)
    pixels, var_of_fold = _pair_indices("state_table_pair_grad", table, pixels, var_of_fold, folds, m, device)
    if units != 64:
        raise NotImplementedError("state_table_pair_grad: 64 units")
    status = _lib.load().xe_state_table_pair_grad(da.data_ptr(), folds, m, pixels.data_ptr(), pixels.stride(0),
                                                  pixels.stride(1), pixels.shape[1], _ptr(var_of_fold), folds, states,
                                                  table.data_ptr(), _stream(device))
    _lib.check(status, "xe_state_table_pair_grad")
    return table


def variable_major(pixels: torch.Tensor) -> torch.Tensor:
    """The (batch, variables) uint8 pixels as a (batch, variables) view of a variable-major copy
    (strides (1, batch)), made by xe_u8_transpose: the layout the state-table backward reads."""
    device = pixels.device
    if device.type != "cuda" or pixels.dtype != torch.uint8 or pixels.dim() != 2 or pixels.stride(1) != 1:
        raise ValueError("variable_major: a CUDA uint8 (batch, variables) tensor with unit column stride")
    batch, variables = pixels.shape
    out = torch.empty((variables, batch), device=device, dtype=torch.uint8)
    status = _lib.load().xe_u8_transpose(pixels.data_ptr(), batch, variables, pixels.stride(0), out.data_ptr(),
                                         _stream(device))
    _lib.check(status, "xe_u8_transpose")
    return out.t()


def _cp_backward_shapes(name, a, y, g, w):
    for t, what in ((a, "a"), (y, "y"), (g, "g"), (w, "w")):
        if t.dim() != 3 or not t.is_contiguous():
            raise ValueError(f"{name}: {what} must be a contiguous 3-d tensor")
    folds, m, units = y.shape
    if units != 64 or tuple(w.shape) != (folds, 64, 64):
        raise NotImplementedError(f"{name}: the CP layer backward takes K = N = 64 (w of shape (F, 64, 64))")
    if tuple(a.shape) != tuple(y.shape) or g.shape[1:] != y.shape[1:] or g.shape[0] < 1 or folds % g.shape[0]:
        raise ValueError(f"{name}: incompatible shapes a {tuple(a.shape)}, y {tuple(y.shape)}, g {tuple(g.shape)}")
    return folds, m, units


def _pair_indices(name, table, pixels, var_of_fold, folds, m, device):
    if pixels.device != device or pixels.dtype != torch.uint8 or pixels.dim() != 2 or pixels.shape[0] != m:
        raise ValueError(f"{name}: pixels must be a (batch, variables) uint8 tensor on the table's device")
    if table.dim() != 3 or table.shape[0] != 2 * folds or not table.is_contiguous():
        raise ValueError(f"{name}: expected a contiguous (2F, states, 64) state table")
    if var_of_fold is not None:
        if var_of_fold.dtype != torch.int32 or var_of_fold.device != device or var_of_fold.numel() != 2 * folds:
            raise ValueError(f"{name}: var_of_fold must be int32 with one entry per table fold")
        var_of_fold = var_of_fold.contiguous()
    elif pixels.shape[1] < 2 * folds:
        raise ValueError(f"{name}: fewer pixel variables than table folds")
    return pixels, var_of_fold


def logspace_tucker(
    left: torch.Tensor,
    right: torch.Tensor,
    weights: torch.Tensor,
    *,
    shift: str = "max",
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """y[b,f,o] = log(sum_ij exp(l-sl) exp(r-sr) w[f,o,i,j]) + sl + sr (xe_logspace_tucker_strided).

    ``left`` (B, F, I) and ``right`` (B, F, J) may be any views whose unit axis is contiguous and
    whose batch and fold strides are multiples of 4 elements (the fold-major (F, B, I) tensors of a
    folded circuit, permuted, qualify); other layouts are copied.  ``out`` (B, F, O) may be any
    view with contiguous units.
    ``weights`` is (F, O, I, J).  Differentiable (autograd.LogspaceTucker, shifts detached) when an
    operand requires grad."""
    if out is None and _needs_grad(left, right, weights):
        from .autograd import LogspaceTucker

        return LogspaceTucker.apply(left, right, weights, shift)
    _no_backward("logspace_tucker", left, right, weights)
    device = _check_tensors("logspace_tucker", left, right, weights, *([out] if out is not None else []))
    if left.dim() != 3 or right.dim() != 3 or weights.dim() != 4:
        raise ValueError("logspace_tucker: expected (B,F,I), (B,F,J) and (F,O,I,J) tensors")
    batch, folds, i_dim = left.shape
    j_dim = right.shape[2]
    o_dim = weights.shape[1]
    if right.shape[:2] != (batch, folds) or weights.shape != (folds, o_dim, i_dim, j_dim):
        raise ValueError("logspace_tucker: incompatible shapes")

    def rows(t: torch.Tensor) -> torch.Tensor:
        ok = t.stride(2) == 1 and t.stride(0) % 4 == 0 and t.stride(1) % 4 == 0 and t.data_ptr() % 16 == 0
        return t if ok else t.contiguous()

    left, right, weights = rows(left), rows(right), weights.contiguous()
    if out is None:
        out = torch.empty((batch, folds, o_dim), device=device, dtype=torch.float32)
    elif out.shape != (batch, folds, o_dim) or out.stride(2) != 1 or min(out.stride()) < 0:
        raise ValueError("logspace_tucker: out must be a (B, F, O) view with contiguous units")
    status = _lib.load().xe_logspace_tucker_strided(
        left.data_ptr(), left.stride(0), left.stride(1), right.data_ptr(), right.stride(0), right.stride(1),
        weights.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1), batch, folds, i_dim, j_dim, o_dim,
        _shift(shift), _stream(device),
    )
    _lib.check(status, "xe_logspace_tucker")
    return out


# ---------------------------------------------------------------------------
# scaled stability modes: a value is (normalized, log_scale) with
# raw = normalized * exp(log_scale), one scale per last-axis fibre

FIBER_KINDS = {"sum": _lib.XE_FIBER_SUM, "max": _lib.XE_FIBER_MAX, "min": _lib.XE_FIBER_MIN,
               "exp": _lib.XE_FIBER_EXP, "lse": _lib.XE_FIBER_LSE}
ELEMENTWISE_OPS = {
    "add": _lib.XE_OP_ADD, "sub": _lib.XE_OP_SUB, "mul": _lib.XE_OP_MUL, "div": _lib.XE_OP_DIV,
    "max": _lib.XE_OP_MAX, "min": _lib.XE_OP_MIN, "mul_exp": _lib.XE_OP_MUL_EXP, "log_add": _lib.XE_OP_LOG_ADD,
    "rescale": _lib.XE_OP_RESCALE,
}


def scaled_gemm(a: torch.Tensor, b: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """C[t,m,n] = sum_k A[t,m,k] B[t,k,n] for linear fp32 operands (xe_scaled_gemm), any strides."""
    _no_backward("scaled_gemm", a, b)
    tensors = [a, b] + ([out] if out is not None else [])
    device = _check_tensors("scaled_gemm", *tensors)
    if a.dim() != 3 or b.dim() != 3:
        raise ValueError("scaled_gemm: operands must be 3-D (batch, M, K) and (batch, K, N)")
    batch, m, k = a.shape
    if b.shape[0] != batch or b.shape[1] != k:
        raise ValueError(f"scaled_gemm: incompatible shapes {tuple(a.shape)} and {tuple(b.shape)}")
    n = b.shape[2]
    if out is None:
        out = torch.empty((batch, m, n), device=device, dtype=torch.float32)
    elif out.shape != (batch, m, n):
        raise ValueError(f"scaled_gemm: out has shape {tuple(out.shape)}, expected {(batch, m, n)}")
    if k == 0:  # an empty contraction is zero (torch.einsum semantics)
        return out.zero_()
    status = _lib.load().xe_scaled_gemm(
        a.data_ptr(), a.stride(0), a.stride(1), a.stride(2),
        b.data_ptr(), b.stride(0), b.stride(1), b.stride(2),
        out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
        batch, m, n, k, _stream(device),
    )
    _lib.check(status, "xe_scaled_gemm")
    return out


def fiber_normalize(x: torch.Tensor, kind: str) -> tuple[torch.Tensor, torch.Tensor]:
    """(normalized, log_scale) of x over its last axis (xe_fiber_normalize).

    kind 'sum' / 'max' / 'min' normalise a raw x by that fibre statistic
    (translate.py:174-199); 'exp' gives the pair of exp(x) for a raw x
    (translate.py:436-444); 'lse' gives the sum-normalised pair of exp(x) for
    a log-domain x.  log_scale has x's shape with the last axis 1 (a rank-0 x
    gives rank-0 results).
    """
    _no_backward("fiber_normalize", x)
    device = _check_tensors("fiber_normalize", x)
    try:
        code = FIBER_KINDS[kind]
    except KeyError:
        raise ValueError(f"fiber_normalize: unknown kind {kind!r}") from None
    if x.dim() > 7:
        raise NotImplementedError(f"fiber_normalize: rank {x.dim()} above 7 is not supported")
    normalized = torch.empty(x.shape, device=device, dtype=torch.float32)
    scale_shape = (*x.shape[:-1], 1) if x.dim() else ()
    log_scale = torch.empty(scale_shape, device=device, dtype=torch.float32)
    status = _lib.load().xe_fiber_normalize(
        x.data_ptr(), _lib.int64_array(x.shape), _lib.int64_array(x.stride()), x.dim(), code,
        normalized.data_ptr(), log_scale.data_ptr(), _stream(device),
    )
    _lib.check(status, "xe_fiber_normalize")
    return normalized, log_scale


def reduce(x: torch.Tensor, axes: Sequence[int] | None, kind: str, *, keepdims: bool = False) -> torch.Tensor:
    """sum / amax / amin of x over ``axes`` (None = all), xe_reduce."""
    _no_backward("reduce", x)
    device = _check_tensors("reduce", x)
    if kind not in ("sum", "max", "min"):
        raise ValueError(f"reduce: unknown kind {kind!r}")
    nd = x.dim()
    axes = tuple(range(nd)) if axes is None else tuple(sorted({a + nd if a < 0 else a for a in axes}))
    if any(not 0 <= a < nd for a in axes):
        raise ValueError(f"reduce: axes out of range for a {nd}-D tensor")
    keep = [d for d in range(nd) if d not in axes]
    kept_shape = [x.shape[d] for d in keep]
    rows = math.prod(kept_shape)
    k = math.prod(x.shape[d] for d in axes)
    y = torch.empty(rows, device=device, dtype=torch.float32)
    after = math.prod(x.shape[axes[-1] + 1:]) if axes else 1
    block = bool(axes) and x.is_contiguous() and axes == tuple(range(axes[0], axes[-1] + 1)) and 1 < after <= 256
    if block and rows == after and k >= 8192 and k % 64 == 0:
        # one long leading block: 64-row chunks reduced as a batch, then the chunks (two passes in
        # a fixed order)
        partial = reduce(x.reshape(k // 64, 64, after), (1,), kind)
        return reduce(partial, (0,), kind, keepdims=keepdims).reshape(
            [1 if d in axes else x.shape[d] for d in range(nd)] if keepdims else kept_shape)
    if block:
        # a middle (or leading) block of a contiguous tensor: (before, k, after) with the outputs
        # contiguous, no copy
        before = rows // after
        args = (x.data_ptr(), k * after, 1, after, before, after, k)
    else:
        view = x.permute(keep + list(axes)).reshape(1, rows, k)
        args = (view.data_ptr(), view.stride(0), view.stride(1), view.stride(2), 1, rows, k)
    status = _lib.load().xe_reduce(*args, FIBER_KINDS[kind], y.data_ptr(), _stream(device))
    _lib.check(status, "xe_reduce")
    if keepdims:
        return y.reshape([1 if d in axes else x.shape[d] for d in range(nd)])
    return y.reshape(kept_shape)


def elementwise(op: str, a: torch.Tensor, b: torch.Tensor, c: torch.Tensor | None = None) -> torch.Tensor:
    """Broadcast elementwise glue of the scaled modes (xe_elementwise): add, sub, mul, div, max, min,
    mul_exp (a*exp(b)), log_add (log(a)+b), rescale (a*exp(b-c))."""
    _no_backward("elementwise", a, b, c)
    operands = [a, b] + ([c] if c is not None else [])
    device = _check_tensors("elementwise", *operands)
    try:
        code = ELEMENTWISE_OPS[op]
    except KeyError:
        raise ValueError(f"elementwise: unknown op {op!r}") from None
    if (op == "rescale") != (c is not None):
        raise ValueError("elementwise: the third operand belongs to 'rescale' only")
    shape = torch.broadcast_shapes(*(t.shape for t in operands))
    if len(shape) > 6:
        raise NotImplementedError(f"elementwise: rank {len(shape)} above 6 is not supported")
    y = torch.empty(shape, device=device, dtype=torch.float32)
    c_strides = _lib.int64_array(_broadcast_strides(c, shape)) if c is not None else None
    status = _lib.load().xe_elementwise(
        code, a.data_ptr(), _lib.int64_array(_broadcast_strides(a, shape)),
        b.data_ptr(), _lib.int64_array(_broadcast_strides(b, shape)),
        _ptr(c), c_strides, y.data_ptr(), _lib.int64_array(shape), len(shape), _stream(device),
    )
    _lib.check(status, "xe_elementwise")
    return y


def device_status(clear: bool = True) -> int:
    """The device-side status word (non-zero after a bounded wait ran out)."""
    return int(_lib.load().xe_device_status(int(clear)))


def set_wait_timeout_ns(ns: int) -> None:
    """Limit of the kernels' bounded waits on the current device, in ns (0 restores the 2 s default).

    Waits for the work already queued first, so that no running kernel sees the change."""
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    _lib.check(_lib.load().xe_set_wait_timeout_ns(int(ns)), "xe_set_wait_timeout_ns")
