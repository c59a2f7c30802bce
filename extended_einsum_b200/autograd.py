"""Backward passes of the log-space path (torch.autograd) on the same kernels.

The reference differentiates its torch executor's call sequence, in which
every shift is a ``stop_gradient`` (backend_translation/translate.py:727-740,
backends/torch.py:14-16), so a shift contributes no gradient.  For the
contraction C = log(sum_k A'_ik B'_kj) + sA_i + sB_j with A' = exp(A - sA)
(log-domain A) or A' = A (linear A), and likewise B', that gives

    P = exp(C - sA - sB),  W = G / P,
    dA' = W B'^T,  dB' = A'^T W,
    dA = dA' * A' (log-domain) or dA' (linear),  and the same for B.

Both products are the split-TF32 tensor-core product of linear operands
(``xe_scaled_gemm``); every elementwise step is one ``xe_elementwise`` launch
and every sum over broadcast axes one ``xe_reduce``.  Softmax, the log-space
product (``log_add``), ``exp`` / ``log`` and the log-space reduction follow
the derivatives of the reference's torch calls.

The Tucker layer (y = log sum_ij L'_i R'_j w_oij + sl + sr) differentiates the
same way with W = G exp(sl + sr - y): dL'_i = sum_o W_o sum_j R'_j w_oij,
dR'_j = sum_o W_o sum_i L'_i w_oij, dw_oij = sum_b W_o L'_i R'_j, each a
tensor-core product of linear operands (contraction.linear_einsum).  The
log-space sum / difference with its scalar shift m (translate.py:647-664,
774-789) gives da = G exp(a - y), db = +/- G exp(b - y).  The categorical
gathers (demo/cirkit.py:525-527), alone or fused into the first two circuit
layers, scatter their row gradients back into the table
(xe_categorical_scatter_add), which is the backward of torch's indexing.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from . import ops


def needs_grad(*tensors: torch.Tensor | None) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def _ones_like_scalar(t: torch.Tensor) -> torch.Tensor:
    return torch.ones((), device=t.device, dtype=t.dtype)


def _exp_shifted(x: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """exp(x - s) with s broadcast (xe_elementwise 'rescale' of a unit)."""
    return ops.elementwise("rescale", _ones_like_scalar(x), x, s)


def _sum_to(g: torch.Tensor, shape: Sequence[int]) -> torch.Tensor:
    """g summed over the axes along which an operand of ``shape`` was broadcast."""
    shape = tuple(shape)
    if tuple(g.shape) == shape:
        return g
    lead = g.dim() - len(shape)
    axes = list(range(lead)) + [lead + i for i, n in enumerate(shape) if n == 1 and g.shape[lead + i] != 1]
    reduced = ops.reduce(g, axes, "sum", keepdims=True) if axes else g
    return reduced.reshape(shape)


class LogspaceGemm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, a2, a_linear: bool, b_linear: bool, shift: str):
        c = ops.logspace_gemm(a, b, a2=a2, a_linear=a_linear, b_linear=b_linear, shift=shift)
        ctx.save_for_backward(a, b, a2, c)
        ctx.flags = (a_linear, b_linear, shift)
        return c

    @staticmethod
    def backward(ctx, g):
        a, b, a2, c = ctx.saved_tensors
        a_linear, b_linear, shift = ctx.flags
        need_a = ctx.needs_input_grad[0] or (a2 is not None and ctx.needs_input_grad[2])
        grad_a, grad_b = _gemm_backward(a, b, a2, c, g, a_linear, b_linear, shift, need_a, ctx.needs_input_grad[1])
        return grad_a, grad_b, grad_a if a2 is not None else None, None, None, None


def _gemm_backward(a, b, a2, c, g, a_linear, b_linear, shift, need_a, need_b):
    """Gradients of C = log(sum_k A'B') + sA + sB with respect to A (and its addend) and B."""
    g = g.contiguous()
    a_tot = ops.elementwise("add", a, a2) if a2 is not None else a
    # operands as the tensor core saw them, and the log of P = sum_k A'B'
    if a_linear:
        a_op, sa = a_tot, None
    else:
        sa = ops.logspace_shift(a_tot, shift=shift).unsqueeze(2)  # (batch, M, 1)
        a_op = _exp_shifted(a_tot, sa)
    if b_linear:
        b_op, sb = b, None
    else:
        sb = ops.logspace_shift(b.transpose(1, 2), shift=shift).unsqueeze(1)  # (batch, 1, N)
        b_op = _exp_shifted(b, sb)
    # W = G / P = G * exp(sA + sB - C)
    log_p = c
    if sb is not None:
        log_p = ops.elementwise("sub", log_p, sb)
    zero = torch.zeros((), device=c.device, dtype=c.dtype)
    w = ops.elementwise("rescale", g, sa if sa is not None else zero, log_p)
    grad_a = grad_b = None
    if need_a:
        d_aop = ops.scaled_gemm(w, b_op.transpose(1, 2))
        grad_a = d_aop if a_linear else ops.elementwise("mul", d_aop, a_op)
    if need_b:
        d_bop = ops.scaled_gemm(a_op.transpose(1, 2), w)
        grad_b = d_bop if b_linear else ops.elementwise("mul", d_bop, b_op)
    return grad_a, grad_b


class LogspaceTucker(torch.autograd.Function):
    """y[b,f,o] = log sum_ij exp(l_i - sl) exp(r_j - sr) w[f,o,i,j] + sl + sr, shifts detached."""

    @staticmethod
    def forward(ctx, left, right, weights, shift: str):
        y = ops.logspace_tucker(left, right, weights, shift=shift)
        ctx.save_for_backward(left, right, weights, y)
        ctx.shift = shift
        return y

    @staticmethod
    def backward(ctx, g):
        from .contraction import linear_einsum

        left, right, weights, y = ctx.saved_tensors
        batch, folds, _ = left.shape
        left, right, g = left.contiguous(), right.contiguous(), g.contiguous()
        sl = ops.logspace_shift(left.reshape(1, batch * folds, -1), shift=ctx.shift).reshape(batch, folds, 1)
        sr = ops.logspace_shift(right.reshape(1, batch * folds, -1), shift=ctx.shift).reshape(batch, folds, 1)
        lp, rp = _exp_shifted(left, sl), _exp_shifted(right, sr)
        w = ops.elementwise("rescale", g, ops.elementwise("add", sl, sr), y)  # G / P
        grad_l = grad_r = grad_w = None
        if ctx.needs_input_grad[0]:
            u = linear_einsum("bfj,foij->bfoi", rp, weights)
            grad_l = ops.elementwise("mul", linear_einsum("bfo,bfoi->bfi", w, u), lp)
        if ctx.needs_input_grad[1]:
            v = linear_einsum("bfi,foij->bfoj", lp, weights)
            grad_r = ops.elementwise("mul", linear_einsum("bfo,bfoj->bfj", w, v), rp)
        if ctx.needs_input_grad[2]:
            grad_w = linear_einsum("bfo,bfij->foij", w, linear_einsum("bfi,bfj->bfij", lp, rp))
        return grad_l, grad_r, grad_w, None


class LogAddExp(torch.autograd.Function):
    """y = log(exp(a - m) +/- exp(b - m)) + m, m the detached scalar extreme: da = G exp(a - y), db = +/- G exp(b - y)."""

    @staticmethod
    def forward(ctx, a, b, subtract: bool, shift: str):
        y = ops.log_add_exp(a, b, subtract=subtract, shift=shift)
        ctx.save_for_backward(a, b, y)
        ctx.subtract = subtract
        return y

    @staticmethod
    def backward(ctx, g):
        a, b, y = ctx.saved_tensors
        g = g.contiguous()
        ga = gb = None
        if ctx.needs_input_grad[0]:
            ga = _sum_to(ops.elementwise("rescale", g, a, y), a.shape)
        if ctx.needs_input_grad[1]:
            gb = _sum_to(ops.elementwise("rescale", g, b, y), b.shape)
            if ctx.subtract:
                gb = ops.elementwise("mul", gb, torch.full((), -1.0, device=g.device, dtype=g.dtype))
        return ga, gb, None, None


def _scatter_rows(grad_rows, pixels, var_of_fold, table, fold_offsets):
    """d(table) from the gradients of rows gathered at fold offsets 0 (and F, for the pair gather)."""
    table_grad = torch.zeros_like(table)
    for offset in fold_offsets:
        ops.categorical_scatter_add(grad_rows, pixels, var_of_fold, table_grad, fold_offset=offset)
    return table_grad


class CategoricalGather(torch.autograd.Function):
    """y[f,b,:] = table[f, pixels[b, var[f]], :]; d(table) is the scatter-add of G."""

    @staticmethod
    def forward(ctx, table, pixels, var_of_fold):
        ctx.save_for_backward(table, pixels, var_of_fold)
        return ops.categorical_gather(table, pixels, var_of_fold)

    @staticmethod
    def backward(ctx, g):
        table, pixels, var_of_fold = ctx.saved_tensors
        return _scatter_rows(g.contiguous(), pixels, var_of_fold, table, (0,)), None, None


class LogspaceGemmGather(torch.autograd.Function):
    """The first circuit layers with their gathers fused: A[f,b,:] = T[f, x_b,var(f)] (+ T[f+F, x_b,var(f+F)]
    for the pair form), C = the log-space contraction of A and B.  The backward gathers A again, takes the
    contraction's gradients and scatters dA into the table."""

    @staticmethod
    def forward(ctx, table, pixels, var_of_fold, b, b_linear: bool, shift: str, pair: bool):
        gather = ops.logspace_gemm_gather_pair if pair else ops.logspace_gemm_gather
        c = gather(table, pixels, var_of_fold, b, b_linear=b_linear, shift=shift)
        ctx.save_for_backward(table, pixels, var_of_fold, b, c)
        ctx.flags = (b_linear, shift, pair)
        return c

    @staticmethod
    def backward(ctx, g):
        table, pixels, var_of_fold, b, c = ctx.saved_tensors
        b_linear, shift, pair = ctx.flags
        folds = b.shape[0]
        if pair:
            var = var_of_fold if var_of_fold is not None else torch.arange(2 * folds, device=table.device, dtype=torch.int32)
            a = ops.categorical_gather(table[:folds], pixels, var[:folds].contiguous())
            a2 = ops.categorical_gather(table[folds:], pixels, var[folds:].contiguous())
        else:
            a, a2 = ops.categorical_gather(table, pixels, var_of_fold), None
        grad_a, grad_b = _gemm_backward(a, b, a2, c, g, False, b_linear, shift, ctx.needs_input_grad[0], ctx.needs_input_grad[3])
        table_grad = None
        if ctx.needs_input_grad[0]:
            table_grad = _scatter_rows(grad_a.contiguous(), pixels, var_of_fold, table, (0, folds) if pair else (0,))
        return table_grad, None, None, grad_b, None, None, None


class LogspaceReduce(torch.autograd.Function):
    """y[t,r] = log sum_k exp(x[t,r,k]) (shifted); dx = g * exp(x - y)."""

    @staticmethod
    def forward(ctx, x, shift: str):
        y = ops.logspace_reduce(x, shift=shift)
        ctx.save_for_backward(x, y)
        return y

    @staticmethod
    def backward(ctx, g):
        x, y = ctx.saved_tensors
        return ops.elementwise("rescale", g.unsqueeze(2), x, y.unsqueeze(2)), None


class Softmax(torch.autograd.Function):
    """y = softmax(x) over ``axes`` (or its log): dx = y (g - sum(g y)), or g - exp(y) sum(g)."""

    @staticmethod
    def forward(ctx, x, axes, log_output: bool):
        y = ops.softmax(x, axes, log_output=log_output)
        ctx.save_for_backward(y)
        ctx.axes, ctx.log_output = ((axes,) if isinstance(axes, int) else tuple(axes)), log_output
        return y

    @staticmethod
    def backward(ctx, g):
        (y,) = ctx.saved_tensors
        g = g.contiguous()
        if ctx.log_output:
            total = ops.reduce(g, ctx.axes, "sum", keepdims=True)
            return ops.elementwise("sub", g, ops.elementwise("mul_exp", total, y)), None, None
        dot = ops.reduce(ops.elementwise("mul", g, y), ctx.axes, "sum", keepdims=True)
        return ops.elementwise("mul", y, ops.elementwise("sub", g, dot)), None, None


class LogAdd(torch.autograd.Function):
    """y = a + b (or a - b), broadcast: the log-space product (quotient)."""

    @staticmethod
    def forward(ctx, a, b, negate_b: bool):
        ctx.shapes = (tuple(a.shape), tuple(b.shape))
        ctx.negate_b = negate_b
        return ops.log_add(a, b, negate_b=negate_b)

    @staticmethod
    def backward(ctx, g):
        sa, sb = ctx.shapes
        ga = _sum_to(g, sa) if ctx.needs_input_grad[0] else None
        gb = None
        if ctx.needs_input_grad[1]:
            gb = _sum_to(g, sb)
            if ctx.negate_b:
                gb = ops.elementwise("mul", gb, torch.full((), -1.0, device=g.device, dtype=g.dtype))
        return ga, gb, None


class Exp(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        y = ops.exp(x)
        ctx.save_for_backward(y)
        return y

    @staticmethod
    def backward(ctx, g):
        (y,) = ctx.saved_tensors
        return ops.elementwise("mul", g, y)


class Log(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        ctx.save_for_backward(x)
        return ops.log(x)

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        return ops.elementwise("div", g, x)
