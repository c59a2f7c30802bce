"""Maps one stable einsum onto one kernel call.

_append_logspace_einsum (backend_translation/translate.py:686-750) lowers an
einsum whose operands are log-space values (or linear parameter-derived
values) into max / exp / einsum / log / shift-add backend calls.  Here the
same arithmetic is one launch:

* one operand            -> xe_logspace_reduce (log-sum-exp over the reduced labels)
* two operands           -> xe_logspace_gemm with the labels grouped into
                            batch (both operands and output), M (first operand
                            and output), N (second operand and output) and K
                            (both operands, not output)
* 'bfi,bfj,foij->bfo'    -> xe_logspace_tucker_strided (the fused Tucker layer,
                            preprocess.py:1095-1106), also in the folded
                            circuits' fold-major form 'acde,abd,abe->abc' and
                            their root 'bcd,ac,ad->ab'
* contraction-free       -> xe_log_add (translate.py:706-718)
* a Hadamard product of two log operands feeding a two-operand contraction
  (the folded circuit's 'cab,cab->cab' -> 'dac,dbc->dab')
                         -> xe_logspace_gemm with the second factor as the
                            fused addend of A

Grouped labels are flattened with ``reshape``, which is a view for the
layouts that reach this path; a layout that cannot be viewed is copied.
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import torch

from . import ops
from .frontend import parse_format_string


def _check_labels(input_strings: list[str], output_string: str) -> None:
    for s in input_strings + [output_string]:
        if len(set(s)) != len(s):
            raise NotImplementedError(f"einsum: repeated labels in {s!r} (diagonals) are not supported on this path")


def _sizes(input_strings: list[str], operands: Sequence[torch.Tensor]) -> dict[str, int]:
    sizes: dict[str, int] = {}
    for labels, operand in zip(input_strings, operands, strict=True):
        if len(labels) != operand.dim():
            raise ValueError(f"einsum: operand of rank {operand.dim()} for labels {labels!r}")
        for label, size in zip(labels, operand.shape):
            if sizes.setdefault(label, size) != size:
                raise RuntimeError(f"Incompatible axis sizes for index {label}: {sizes[label]} and {size}.")
    return sizes


def _group(t: torch.Tensor, labels: str, groups: Sequence[str], sizes: dict[str, int]) -> torch.Tensor:
    """Permutes ``t`` (labelled ``labels``) into ``groups`` order and flattens each group.

    Labels of a group that ``t`` lacks get size 1.
    """
    order = [labels.index(label) for group in groups for label in group if label in labels]
    shape = [math.prod(sizes[label] for label in group if label in labels) for group in groups]
    return t.permute(order).reshape(shape)


def log_broadcast_product(format_string: str, *log_operands: torch.Tensor) -> torch.Tensor:
    """Contraction-free einsum in log space: the broadcast sum of the operands."""
    input_strings, output_string = parse_format_string(format_string)
    _check_labels(input_strings, output_string)
    sizes = _sizes(input_strings, log_operands)
    aligned = []
    for labels, operand in zip(input_strings, log_operands, strict=True):
        order = [labels.index(label) for label in output_string if label in labels]
        view = operand.permute(order) if order else operand
        shape = [sizes[label] if label in labels else 1 for label in output_string]
        aligned.append(view.reshape(shape))
    result = aligned[0]
    for operand in aligned[1:]:
        result = ops.log_add(result, operand)
    return result


def logspace_einsum(
    format_string: str, linear: Sequence[bool], shift: str, *operands: torch.Tensor
) -> torch.Tensor:
    """The log of the einsum of exp(log operands) and linear operands, shifted per operand.

    ``linear[i]`` marks operand i as a raw (parameter-derived) value; the
    others are log-space values.  Returns the log-space result.
    """
    input_strings, output_string = parse_format_string(format_string)
    if len(input_strings) != len(operands):
        raise ValueError(f"The einsum format string has {len(input_strings)} inputs, but the instruction has {len(operands)} arguments.")
    _check_labels(input_strings, output_string)
    sizes = _sizes(input_strings, operands)
    if len(operands) == 1:
        return _reduce(input_strings[0], output_string, operands[0], linear[0], shift, sizes)
    if len(operands) == 2:
        return _binary(input_strings, output_string, operands, linear, shift, sizes)
    if len(operands) == 3:
        tucker = _match_tucker(input_strings, output_string, linear)
        if tucker is not None:
            return _tucker(tucker, operands, shift)
    raise NotImplementedError(
        f"einsum {format_string!r} with {len(operands)} operands has no fused log-space kernel on this path"
    )


def _reduce(labels: str, output_string: str, x: torch.Tensor, linear: bool, shift: str, sizes) -> torch.Tensor:
    reduced = "".join(label for label in labels if label not in output_string)
    if linear:
        # log(sum(x)) of a positive linear operand = log-sum-exp of log(x)
        x = ops.log(x)
    if not reduced:
        return log_broadcast_product(f"{labels}->{output_string}", x)
    view = _group(x, labels, ["", output_string, reduced], sizes)
    y = ops.logspace_reduce(view, shift=shift)
    return y.reshape([sizes[label] for label in output_string])


def logspace_einsum_hadamard(
    format_string: str, b_linear: bool, shift: str, a: torch.Tensor, a2: torch.Tensor, b: torch.Tensor
) -> torch.Tensor:
    """The log-space einsum of (a + a2) and b, where a + a2 is a log-domain Hadamard product.

    ``a`` and ``a2`` carry the first operand's labels; the kernel adds them in
    fp32 before the row shift (the addend ``a2`` of xe_logspace_gemm), which
    is the separate log add (translate.py:706-718) followed by the contraction
    (:686-750) without the intermediate tensor.  Operands whose grouped views
    differ in strides are added first.
    """
    input_strings, output_string = parse_format_string(format_string)
    _check_labels(input_strings, output_string)
    sizes = _sizes(input_strings, (a, b))
    if a2.shape != a.shape:
        raise ValueError(f"einsum: Hadamard factors of shapes {tuple(a.shape)} and {tuple(a2.shape)}")
    if a.stride() != a2.stride():
        return _binary(input_strings, output_string, (ops.log_add(a, a2), b), (False, b_linear), shift, sizes)
    return _binary(input_strings, output_string, (a, b), (False, b_linear), shift, sizes, a2=a2)


def _binary(input_strings, output_string, operands, linear, shift, sizes, a2: torch.Tensor | None = None) -> torch.Tensor:
    la, lb = input_strings
    batch = "".join(label for label in output_string if label in la and label in lb)
    m_labels = "".join(label for label in output_string if label in la and label not in lb)
    n_labels = "".join(label for label in output_string if label in lb and label not in la)
    k_labels = "".join(label for label in la if label in lb and label not in output_string)
    private = [label for s in (la, lb) for label in s if label not in output_string and label not in k_labels]
    if private:
        raise NotImplementedError(
            f"einsum {la},{lb}->{output_string}: labels {''.join(private)!r} are summed within one operand only"
        )
    a = _group(operands[0], la, [batch, m_labels, k_labels], sizes)
    b = _group(operands[1], lb, [batch, k_labels, n_labels], sizes)
    if a2 is not None:
        a2 = _group(a2, la, [batch, m_labels, k_labels], sizes)
        if a2.stride() != a.stride():  # one of the two views had to be copied
            a, a2 = ops.log_add(a, a2), None
    c = ops.logspace_gemm(a, b, a2=a2, a_linear=linear[0], b_linear=linear[1], shift=shift)
    grouped = batch + m_labels + n_labels
    c = c.reshape([sizes[label] for label in grouped])
    return c.permute([grouped.index(label) for label in output_string])


def _scaled_log_plan(format_string: str):
    """Label plan of ``scaled_log_einsum`` (None when the einsum does not take that path).

    Two operands, at least one contracted label, no label summed within one operand, and for each
    operand a last label that is either contracted (its exp fibre runs along the contraction: one
    shift per row of the grouped operand) or the operand's only retained non-batch label (the
    shift is then one value per batch entry).
    """
    input_strings, output_string = parse_format_string(format_string)
    if len(input_strings) != 2 or len(set(output_string)) != len(output_string):
        return None
    la, lb = input_strings
    if len(set(la)) != len(la) or len(set(lb)) != len(lb) or not la or not lb:
        return None
    if any(label not in lb and label not in output_string for label in la) or any(
        label not in la and label not in output_string for label in lb
    ):
        return None
    batch = "".join(label for label in output_string if label in la and label in lb)
    m_labels = "".join(label for label in output_string if label in la and label not in lb)
    n_labels = "".join(label for label in output_string if label in lb and label not in la)
    k_labels = "".join(label for label in la if label in lb and label not in output_string)
    if not k_labels or any(label not in la and label not in lb for label in output_string):
        return None
    kinds = []
    for labels, own in ((la, m_labels), (lb, n_labels)):
        last = labels[-1]
        if last in k_labels:
            kinds.append("row")
        elif own == last:
            kinds.append("batch")
        else:
            return None
    return input_strings, output_string, batch, m_labels, k_labels, n_labels, tuple(kinds)


def scaled_log_einsum_supported(format_string: str) -> bool:
    return _scaled_log_plan(format_string) is not None


def scaled_log_einsum(format_string: str, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """log(einsum(exp(a), exp(b))) as the scaled modes compute it, in one contraction.

    In the scaled modes exp(x) becomes the pair (exp(x - m), m) with m the maximum of x's last-axis
    fibres (translate.py:410-420); the einsum brings each operand's scale to its maximum over the
    contracted axes (:329-340), contracts the normalised operands and renormalises the result per
    fibre; log(n * e^s) = log(n) + s (:421-425).  The norms cancel in the log, so the value is
    log(sum_k exp(a - sa) exp(b - sb)) + sa + sb with sa (sb) the maximum of a (b) over its
    contracted labels and its last label: the log-space contraction with those shifts
    (xe_logspace_gemm_shifted_strided).  ``a`` and ``b`` are the raw (log-domain) arguments of the
    two exp instructions.
    """
    plan = _scaled_log_plan(format_string)
    if plan is None:
        raise NotImplementedError(f"einsum {format_string!r} has no fused scaled log contraction on this path")
    (la, lb), output_string, batch, m_labels, k_labels, n_labels, kinds = plan
    sizes = _sizes([la, lb], (a, b))
    ag = _group(a, la, [batch, m_labels, k_labels], sizes)
    bg = _group(b, lb, [batch, k_labels, n_labels], sizes)
    nb, m, k = ag.shape
    n = bg.shape[2]
    # shift of A: per (batch, row) over k, or per batch over (m, k) -- the row maxima, then their
    # maximum (max is exact: the same value as one pass, with the rows' parallelism); strides
    # index a (batch, m) view
    sa = ops.logspace_shift(ag)
    if kinds[0] == "row":
        sa_strides = (m, 1)
    else:
        sa, sa_strides = ops.logspace_shift(sa.view(nb, 1, m)), (1, 0)
    sb = ops.logspace_shift(bg.transpose(1, 2))
    if kinds[1] == "row":
        sb_strides = (n, 1)
    else:
        sb, sb_strides = ops.logspace_shift(sb.view(nb, 1, n)), (1, 0)
    c = ops.logspace_gemm_shifted_strided(ag, bg, sa, sa_strides, sb, sb_strides)
    grouped = batch + m_labels + n_labels
    c = c.reshape([sizes[label] for label in grouped])
    return c.permute([grouped.index(label) for label in output_string])


def _match_tucker(input_strings, output_string, linear):
    """(left, right, weights, fold_first, has_fold) operand roles if the einsum is a Tucker layer.

    Three forms reach this path: the layer as written, 'bfi,bfj,foij->bfo' (batch-major); the
    folded circuits' layer after FoldSameShapedOperations and OptimizeContractionPaths
    (preprocess.py:1095-1106, 1310-1393), 'acde,abd,abe->abc' with the fold label first; and their
    root, 'bcd,ac,ad->ab', a single layer without a fold label.  The weights are the operand with
    the o, i, j labels (linear[w] must be set when ``linear`` is given); left and right end in i
    and j and share their leading labels with the output, which ends in o.
    """
    for w in range(3):
        if linear is not None and not linear[w]:
            continue
        others = [i for i in range(3) if i != w]
        if linear is not None and (linear[others[0]] or linear[others[1]]):
            continue
        l_lab, r_lab, w_lab = input_strings[others[0]], input_strings[others[1]], input_strings[w]
        if len(w_lab) == 4 and len(l_lab) == 3 and len(r_lab) == 3 and len(output_string) == 3:
            f, o, i, j = w_lab
            lead = l_lab[:2]
            b = lead.replace(f, "")
            if f not in lead or len(b) != 1 or len({b, f, o, i, j}) != 5:
                continue
            if l_lab != lead + i or r_lab != lead + j or output_string != lead + o:
                continue
            return others[0], others[1], w, lead[0] == f, True
        if len(w_lab) == 3 and len(l_lab) == 2 and len(r_lab) == 2 and len(output_string) == 2:
            o, i, j = w_lab
            b = l_lab[0]
            if len({b, o, i, j}) != 4 or l_lab != b + i or r_lab != b + j or output_string != b + o:
                continue
            return others[0], others[1], w, False, False
    return None


def _tucker(match, operands, shift: str) -> torch.Tensor:
    """The matched Tucker layer on xe_logspace_tucker_strided, in the layout the einsum names."""
    l_idx, r_idx, w_idx, fold_first, has_fold = match
    left, right, weights = operands[l_idx], operands[r_idx], operands[w_idx]
    if not has_fold:
        y = ops.logspace_tucker(left.unsqueeze(1), right.unsqueeze(1), weights.unsqueeze(0), shift=shift)
        return y[:, 0, :]
    if not fold_first:
        return ops.logspace_tucker(left, right, weights, shift=shift)
    # fold-major (F, B, I) operands and output, addressed as (B, F, I) views
    lt, rt = left.transpose(0, 1), right.transpose(0, 1)
    if ops._needs_grad(left, right, weights):
        return ops.logspace_tucker(lt, rt, weights, shift=shift).transpose(0, 1)
    folds, batch, o_dim = weights.shape[0], left.shape[1], weights.shape[1]
    out = torch.empty((folds, batch, o_dim), device=left.device, dtype=torch.float32)
    ops.logspace_tucker(lt, rt, weights, shift=shift, out=out.transpose(0, 1))
    return out


# ---------------------------------------------------------------------------
# linear einsum (the scaled modes' einsum of normalized operands,
# translate.py:372, and einsums of parameter-derived values, :306-309)


def linear_einsum(format_string: str, *operands: torch.Tensor) -> torch.Tensor:
    """torch.einsum semantics for fp32 CUDA operands on the B200 kernels.

    * one operand: a permutation, or xe_reduce (sum) over the dropped labels;
    * contraction-free: a broadcast product (xe_elementwise mul);
    * two operands: labels summed within one operand are summed first, then
      xe_scaled_gemm over the batch / M / N / K grouping;
    * 'bfi,bfj,foij->bfo': the Tucker kernel on the logs of the operands.
    """
    input_strings, output_string = parse_format_string(format_string)
    if len(input_strings) != len(operands):
        raise ValueError(f"The einsum format string has {len(input_strings)} inputs, but the instruction has {len(operands)} arguments.")
    _check_labels(input_strings, output_string)
    sizes = _sizes(input_strings, operands)
    missing = set(output_string) - set("".join(input_strings))
    if missing:
        raise ValueError(f"einsum: output labels {''.join(sorted(missing))!r} appear in no operand")
    if len(operands) == 1:
        return _linear_reduce(input_strings[0], output_string, operands[0], sizes)
    if _contraction_free(input_strings, output_string):
        return _linear_broadcast_product(input_strings, output_string, operands, sizes)
    if len(operands) == 2:
        return _linear_binary(input_strings, output_string, operands, sizes)
    if len(operands) == 3:
        tucker = _match_tucker(input_strings, output_string, None)
        if tucker is not None:
            logs = [operand if i == tucker[2] else ops.log(operand) for i, operand in enumerate(operands)]
            return ops.exp(_tucker(tucker, logs, "max"))
    raise NotImplementedError(f"einsum {format_string!r} with {len(operands)} operands has no fused kernel on this path")


def _contraction_free(input_strings: list[str], output_string: str) -> bool:
    out = set(output_string)
    return all(set(s) <= out for s in input_strings)


def _linear_reduce(labels: str, output_string: str, x: torch.Tensor, sizes: dict[str, int]) -> torch.Tensor:
    reduced = [axis for axis, label in enumerate(labels) if label not in output_string]
    kept = "".join(label for label in labels if label in output_string)
    if reduced:
        x = ops.reduce(x, reduced, "sum")
    if kept != output_string:
        x = x.permute([kept.index(label) for label in output_string])
    return x


def _aligned(labels: str, output_string: str, operand: torch.Tensor, sizes: dict[str, int]) -> torch.Tensor:
    order = [labels.index(label) for label in output_string if label in labels]
    view = operand.permute(order) if order else operand
    return view.reshape([sizes[label] if label in labels else 1 for label in output_string])


def _linear_broadcast_product(input_strings, output_string, operands, sizes) -> torch.Tensor:
    result = _aligned(input_strings[0], output_string, operands[0], sizes)
    for labels, operand in zip(input_strings[1:], operands[1:], strict=True):
        result = ops.elementwise("mul", result, _aligned(labels, output_string, operand, sizes))
    shape = [sizes[label] for label in output_string]
    if list(result.shape) != shape:  # a single operand broadcast to the output
        result = ops.elementwise("mul", result, torch.ones((), device=result.device, dtype=result.dtype).expand(shape))
    return result


def _linear_binary(input_strings, output_string, operands, sizes) -> torch.Tensor:
    la, lb = input_strings
    a, b = operands
    # a label present in one operand only and absent from the output is summed there first
    private_a = "".join(label for label in la if label not in lb and label not in output_string)
    private_b = "".join(label for label in lb if label not in la and label not in output_string)
    if private_a:
        a = ops.reduce(a, [la.index(label) for label in private_a], "sum")
        la = "".join(label for label in la if label not in private_a)
    if private_b:
        b = ops.reduce(b, [lb.index(label) for label in private_b], "sum")
        lb = "".join(label for label in lb if label not in private_b)
    batch = "".join(label for label in output_string if label in la and label in lb)
    m_labels = "".join(label for label in output_string if label in la and label not in lb)
    n_labels = "".join(label for label in output_string if label in lb and label not in la)
    k_labels = "".join(label for label in la if label in lb and label not in output_string)
    a3 = _group(a, la, [batch, m_labels, k_labels], sizes)
    b3 = _group(b, lb, [batch, k_labels, n_labels], sizes)
    c = ops.scaled_gemm(a3, b3)
    grouped = batch + m_labels + n_labels
    c = c.reshape([sizes[label] for label in grouped])
    return c.permute([grouped.index(label) for label in output_string])
