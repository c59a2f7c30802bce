"""Lowering of a RichProgram in a scaled stability mode onto the sm_100a kernels.

The scaled modes (scaled_sum, scaled_max, scaled_min) keep every value as a
pair (normalized, log_scale) with raw = normalized * exp(log_scale) and one
log scale per last-axis fibre, normalised lazily by the fibre's sum, maximum
or minimum (backend_translation/translate.py:115-162).  ``_ScaledLowering``
walks the program exactly like ``_translate_scaled`` and
``_append_scaled_instruction`` (translate.py:164-585): the same positions,
the same shape bookkeeping for the scales, the same decisions about which
scales to reduce, broadcast or keep.  What differs is what each step emits:

* a fibre normalisation (norm, divide, log; translate.py:183-197, 373-382)
  and the exp rule (max, subtract, exp; :436-444) are one xe_fiber_normalize
  launch that returns the pair;
* the einsum of normalized operands (:372) is one xe_scaled_gemm launch
  (tensor cores, split TF32) for a binary contraction;
* scale arithmetic such as subtract + exp + multiply (:253-257, :336-339) is
  one xe_elementwise launch (``rescale``), and so are exp + multiply back to
  raw (:168-170) and log + add (:445-449).

Structural operators (stack, concat, take, select, slice, reshape) are
torch views or copies, as in the log-space lowering.
"""

from __future__ import annotations

from functools import partial
from typing import Any

import numpy as np
import torch

from . import ops
from .contraction import linear_einsum, scaled_log_einsum, scaled_log_einsum_supported
from .frontend import is_contraction_free_einsum, normalize_axis, parse_format_string

SCALED_NORMS = {"scaled_sum": "sum", "scaled_max": "max", "scaled_min": "min"}

Shape = tuple[int, ...]


def _infer_binary_shape(shape_1: Shape, shape_2: Shape) -> Shape:
    """numpy broadcasting of two shapes (shapes.py:23-24)."""
    return tuple(np.broadcast_shapes(shape_1, shape_2))


def _fiber_scale_shape(value_shape: Shape) -> Shape:
    """Shape of the per-fibre log scale of a value (translate.py:202-205)."""
    if not value_shape:
        return ()
    return (*value_shape[:-1], 1)


def _first(pair: tuple[torch.Tensor, torch.Tensor]) -> torch.Tensor:
    return pair[0]


def _second(pair: tuple[torch.Tensor, torch.Tensor]) -> torch.Tensor:
    return pair[1]


def _reshape_einsum_shift(retained_labels: str, output_string: str, shift: torch.Tensor) -> torch.Tensor:
    """Reshapes a scale over retained labels to broadcast over the output (translate.py:667-672)."""
    dims = iter(shift.shape)
    return torch.reshape(shift, tuple(next(dims) if label in retained_labels else 1 for label in output_string))


def _broadcast_einsum_operand(input_string: str, output_string: str, operand: torch.Tensor) -> torch.Tensor:
    """Reorders a contraction-free operand's scale for broadcasting (translate.py:675-683)."""
    retained = "".join(label for label in output_string if label in input_string)
    if input_string != retained:
        operand = linear_einsum(f"{input_string}->{retained}", operand)
    dims = iter(operand.shape)
    return torch.reshape(operand, tuple(next(dims) if label in retained else 1 for label in output_string))


def _slice_broadcast_scale(call, axis: int, scale: torch.Tensor) -> torch.Tensor:
    """Slices a scale only when it varies along the sliced axis (translate.py:208-216)."""
    if not scale.shape:
        return scale
    normalized = axis if axis >= 0 else axis + scale.dim()
    if scale.shape[normalized] == 1:
        return scale
    return call(scale)


def _select_broadcast_scale(axis: int, index: int, scale: torch.Tensor) -> torch.Tensor:
    """Selects from a scale, index 0 along a broadcast axis (translate.py:219-226)."""
    if not scale.shape:
        return scale
    normalized = axis if axis >= 0 else axis + scale.dim()
    return torch.select(scale, axis, 0 if scale.shape[normalized] == 1 else index)


def _take_broadcast_scale(axis: int, scale: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """Takes from a scale only when it varies along the axis (translate.py:229-237)."""
    if not scale.shape:
        return scale
    normalized = axis if axis >= 0 else axis + scale.dim()
    if scale.shape[normalized] == 1:
        return scale
    return torch.index_select(scale, axis, indices)


def _reshape_stack_scale(axis: int, scale: torch.Tensor) -> torch.Tensor:
    """Inserts the stack axis into a non-scalar scale (translate.py:283-290)."""
    if not scale.shape:
        return scale
    normalized = axis if axis >= 0 else axis + scale.dim() + 1
    return torch.reshape(scale, (*scale.shape[:normalized], 1, *scale.shape[normalized:]))


def _stack(axis: int, *tensors: torch.Tensor) -> torch.Tensor:
    return torch.stack(tensors, dim=axis)


def _concat(axis: int, *tensors: torch.Tensor) -> torch.Tensor:
    return torch.cat(tensors, dim=axis)


def _take(axis: int, source: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    return torch.index_select(source, axis, indices)


def _select(axis: int, index: int, source: torch.Tensor) -> torch.Tensor:
    return torch.select(source, axis, index)


def _slice(start: int, stop: int, axis: int, source: torch.Tensor) -> torch.Tensor:
    dim = axis if axis >= 0 else axis + source.dim()
    return source.narrow(dim, start, stop - start)


def _broadcast_to(shape: Shape, t: torch.Tensor) -> torch.Tensor:
    return torch.broadcast_to(t, shape)


class _ScaledLowering:
    def __init__(self, program: Any, norm: str, builder: Any, parameter_derived: frozenset[int]) -> None:
        self.program = program
        self.norm = norm
        self.b = builder
        self.positions: dict[tuple[int, str], int] = {(i, "raw"): i for i in range(program.n_inputs)}
        self.scale_shapes: dict[int, Shape] = {}
        self.value_shapes: list[Shape] = [tuple(s) for s in program.shapes]
        self.parameter_derived = parameter_derived
        # exp results whose scaled pair is made only when something asks for it (position of the
        # raw argument), and log results that a fused contraction already computed
        self.lazy_exp: dict[int, int] = {}
        self.fused_log: dict[int, int] = {}
        self.uses: dict[int, list[int]] = {}
        for index, instruction in enumerate(program.instructions):
            for a in instruction.argument_ssa_ids:
                self.uses.setdefault(a, []).append(program.n_inputs + index)

    def run(self):
        for index, instruction in enumerate(self.program.instructions):
            self._instruction(instruction, self.program.n_inputs + index)
        output = self._raw(self.program.output_ssa)
        if output != self.b.last_position:
            raise ValueError("The raw value of the program's output must be the last computed tensor, because the runtime returns the last tensor.")
        return self.b.build()

    # ---------------------------------------------------------------- parts
    def _raw(self, ssa: int) -> int:
        """raw = normalized * exp(log_scale), at most once (translate.py:164-171)."""
        if (ssa, "raw") not in self.positions:
            normalized, log_scale = self._scaled(ssa)
            self.positions[ssa, "raw"] = self.b.append(partial(ops.elementwise, "mul_exp"), (normalized, log_scale))
        return self.positions[ssa, "raw"]

    def _pair(self, normalize: Any, argument: int) -> tuple[int, int]:
        pair = self.b.append(normalize, (argument,))
        return self.b.append(_first, (pair,)), self.b.append(_second, (pair,))

    def _scaled(self, ssa: int) -> tuple[int, int]:
        """The fibre-normalised pair of a raw value, at most once (translate.py:174-199)."""
        if (ssa, "normalized") not in self.positions and ssa in self.lazy_exp:
            # the exp rule (translate.py:410-420), made when first needed
            normalized, log_scale = self._pair(partial(ops.fiber_normalize, kind="exp"), self.lazy_exp[ssa])
            self.positions[ssa, "normalized"], self.positions[ssa, "log_scale"] = normalized, log_scale
            return normalized, log_scale
        if (ssa, "normalized") not in self.positions:
            raw = self.positions[ssa, "raw"]
            normalized, log_scale = self._pair(partial(ops.fiber_normalize, kind=self.norm), raw)
            self.positions[ssa, "normalized"] = normalized
            self.positions[ssa, "log_scale"] = log_scale
            self.scale_shapes[ssa] = _fiber_scale_shape(self.value_shapes[ssa])
        return self.positions[ssa, "normalized"], self.positions[ssa, "log_scale"]

    def _rescaled(self, pairs: list[tuple[int, int]], shapes: list[Shape], to_scalar: bool = False) -> tuple[list[int], int, Shape]:
        """Brings pairs to the maximum of their log scales (translate.py:240-280)."""
        if not pairs:
            raise ValueError("At least one scaled pair is required")
        if len(pairs) != len(shapes):
            raise ValueError("Every scaled pair must have a scale shape")
        scales = [s for _, s in pairs]
        if to_scalar:
            scales = [self.b.append(partial(ops.reduce, axes=None, kind="max"), (s,)) for s in scales]
        common = scales[0]
        common_shape: Shape = () if to_scalar else shapes[0]
        for scale, shape in zip(scales[1:], shapes[1:], strict=True):
            common = self.b.append(partial(ops.elementwise, "max"), (common, scale))
            if not to_scalar:
                common_shape = _infer_binary_shape(common_shape, shape)
        rescaled = [self.b.append(partial(ops.elementwise, "rescale"), (n, s, common)) for n, s in pairs]
        return rescaled, common, common_shape

    # -------------------------------------------------------- instructions
    def _instruction(self, instruction: Any, result: int) -> None:
        op = instruction.operator
        args = instruction.argument_ssa_ids
        name = op.name
        b, pos, shapes = self.b, self.positions, self.scale_shapes
        if name == "exp":
            # translate.py:410-420: the raw argument's fibre maximum becomes the log scale (the pair
            # is made when a consumer needs it: a fused contraction takes the raw argument instead)
            self.lazy_exp[result] = self._raw(args[0])
            shapes[result] = _fiber_scale_shape(self.value_shapes[result])
        elif name == "log" and args[0] in self.fused_log:
            # the contraction already produced log(n) + s (scaled_log_einsum)
            pos[result, "raw"] = self.fused_log[args[0]]
        elif name == "log":
            # translate.py:421-425: log(n * e^s) = log(n) + s, stored raw
            n, s = self._scaled(args[0])
            pos[result, "raw"] = b.append(partial(ops.elementwise, "log_add"), (n, s))
        elif name == "softmax":
            pos[result, "raw"] = b.append(partial(ops.softmax, axis=op.axis), (self._raw(args[0]),))
        elif name in ("+", "-"):
            pairs = [self._scaled(a) for a in args]
            rescaled, common, common_shape = self._rescaled(pairs, [shapes[a] for a in args])
            combine = "add" if name == "+" else "sub"
            pos[result, "normalized"] = b.append(partial(ops.elementwise, combine), tuple(rescaled))
            pos[result, "log_scale"] = common
            shapes[result] = common_shape
        elif name in ("*", "/"):
            (n1, s1), (n2, s2) = (self._scaled(a) for a in args)
            value_op, scale_op = ("mul", "add") if name == "*" else ("div", "sub")
            pos[result, "normalized"] = b.append(partial(ops.elementwise, value_op), (n1, n2))
            pos[result, "log_scale"] = b.append(partial(ops.elementwise, scale_op), (s1, s2))
            shapes[result] = _infer_binary_shape(shapes[args[0]], shapes[args[1]])
        elif name == "stack":
            self._stack(op.axis, args, result)
        elif name == "concat":
            self._concat(op.axis, args, result)
        elif name == "take":
            self._take(op.axis, args, result)
        elif name == "select":
            self._indexing(op, partial(_select, op.axis, op.index), partial(_select_broadcast_scale, op.axis, op.index), args, result)
        elif name == "slice":
            call = partial(_slice, op.start, op.stop, op.axis)
            self._indexing(op, call, partial(_slice_broadcast_scale, call, op.axis), args, result)
        elif name == "einsum":
            self._einsum(op.format_string, args, result)
        else:
            raise NotImplementedError(f"The operator {name} has no scaled backend translation.")

    def _stack(self, axis: int, args: tuple[int, ...], result: int) -> None:
        """translate.py:475-483."""
        pairs = [self._scaled(a) for a in args]
        rescaled, common, common_shape = self._rescaled(pairs, [self.scale_shapes[a] for a in args])
        self.positions[result, "normalized"] = self.b.append(partial(_stack, axis), tuple(rescaled))
        self.positions[result, "log_scale"] = self.b.append(partial(_reshape_stack_scale, axis), (common,))
        value_shape = self.value_shapes[result]
        normalized_axis = normalize_axis(axis, len(value_shape)) if value_shape else 0
        self.scale_shapes[result] = (
            common_shape if not common_shape else (*common_shape[:normalized_axis], 1, *common_shape[normalized_axis:])
        )

    def _concat(self, axis: int, args: tuple[int, ...], result: int) -> None:
        """translate.py:484-555: one scalar scale within a fibre, per-operand scales across fibres."""
        pairs = [self._scaled(a) for a in args]
        value_shape = self.value_shapes[result]
        normalized_axis = normalize_axis(axis, len(value_shape))
        if normalized_axis == len(value_shape) - 1:
            rescaled, common, common_shape = self._rescaled(pairs, [self.scale_shapes[a] for a in args], to_scalar=True)
            self.positions[result, "normalized"] = self.b.append(partial(_concat, axis), tuple(rescaled))
            self.positions[result, "log_scale"] = common
            self.scale_shapes[result] = common_shape
            return
        normalized_positions = [n for n, _ in pairs]
        expanded: list[int] = []
        for index, (a, (_, log_scale)) in enumerate(zip(args, pairs, strict=True)):
            target = _fiber_scale_shape(self.value_shapes[a])
            scale_shape = self.scale_shapes[a]
            if scale_shape and scale_shape[-1] != 1:
                common = self.b.append(partial(ops.reduce, axes=(-1,), kind="max", keepdims=True), (log_scale,))
                normalized_positions[index] = self.b.append(
                    partial(ops.elementwise, "rescale"), (normalized_positions[index], log_scale, common)
                )
                log_scale = common
                scale_shape = (*scale_shape[:-1], 1)
            if scale_shape != target:
                log_scale = self.b.append(partial(_broadcast_to, target), (log_scale,))
            expanded.append(log_scale)
        self.positions[result, "normalized"] = self.b.append(partial(_concat, axis), tuple(normalized_positions))
        self.positions[result, "log_scale"] = self.b.append(partial(_concat, axis), tuple(expanded))
        self.scale_shapes[result] = _fiber_scale_shape(value_shape)

    def _take(self, axis: int, args: tuple[int, ...], result: int) -> None:
        """translate.py:556-569."""
        n, s = self._scaled(args[0])
        indices = self._raw(args[1])
        self.positions[result, "normalized"] = self.b.append(partial(_take, axis), (n, indices))
        self.positions[result, "log_scale"] = self.b.append(partial(_take_broadcast_scale, axis), (s, indices))
        source = self.scale_shapes[args[0]]
        scale_axis = normalize_axis(axis, len(source)) if source else 0
        if not source or source[scale_axis] == 1:
            self.scale_shapes[result] = source
        else:
            value_axis = normalize_axis(axis, len(self.value_shapes[result]))
            self.scale_shapes[result] = (*source[:scale_axis], self.value_shapes[result][value_axis], *source[scale_axis + 1 :])

    def _indexing(self, op: Any, call, scale_call, args: tuple[int, ...], result: int) -> None:
        """select / slice: raw stays raw, a pair is indexed with its scale (translate.py:570-585, 585-600)."""
        if (args[0], "raw") in self.positions:
            self.positions[result, "raw"] = self.b.append(call, (self._raw(args[0]),))
            return
        n, s = self._scaled(args[0])
        self.positions[result, "normalized"] = self.b.append(call, (n,))
        self.positions[result, "log_scale"] = self.b.append(scale_call, (s,))
        source = self.scale_shapes[args[0]]
        scale_axis = normalize_axis(op.axis, len(source)) if source else 0
        if op.name == "select":
            self.scale_shapes[result] = source if not source else (*source[:scale_axis], *source[scale_axis + 1 :])
        elif not source or source[scale_axis] == 1:
            self.scale_shapes[result] = source
        else:
            value_axis = normalize_axis(op.axis, len(self.value_shapes[result]))
            self.scale_shapes[result] = (*source[:scale_axis], self.value_shapes[result][value_axis], *source[scale_axis + 1 :])

    def _fused_log_einsum(self, format_string: str, args: tuple[int, ...], result: int) -> bool:
        """log(einsum(exp(x), exp(y))) as one log-space contraction (scaled_log_einsum), when both
        operands are exp results whose pairs nothing has needed yet and the einsum's only consumer is
        a log: the scaled pair of the product then never exists.  The value is the same function of
        the inputs; only its rounding differs from the pair-by-pair sequence."""
        if len(args) != 2 or any(a not in self.lazy_exp or (a, "normalized") in self.positions for a in args):
            return False
        if any(a in self.parameter_derived for a in args) or result == self.program.output_ssa:
            return False
        consumers = self.uses.get(result, [])
        if len(consumers) != 1:
            return False
        consumer = self.program.instructions[consumers[0] - self.program.n_inputs]
        if consumer.operator.name != "log" or not scaled_log_einsum_supported(format_string):
            return False
        if any(len(self.value_shapes[a]) != len(s) for a, s in zip(args, parse_format_string(format_string)[0])):
            return False
        self.fused_log[result] = self.b.append(partial(scaled_log_einsum, format_string),
                                               (self.lazy_exp[args[0]], self.lazy_exp[args[1]]))
        return True

    def _einsum(self, format_string: str, args: tuple[int, ...], result: int) -> None:
        """_append_scaled_einsum (translate.py:293-394)."""
        input_strings, output_string = parse_format_string(format_string)
        if len(input_strings) != len(args):
            raise ValueError(f"The einsum format string has {len(input_strings)} inputs, but the instruction has {len(args)} arguments.")
        b, pos = self.b, self.positions
        if result in self.parameter_derived:
            pos[result, "raw"] = b.append(partial(linear_einsum, format_string), tuple(self._raw(a) for a in args))
            return
        if self._fused_log_einsum(format_string, args, result):
            return

        operands: list[int] = []
        scales: list[tuple[int, Shape, bool, str, str]] = []
        for input_string, a in zip(input_strings, args, strict=True):
            if a in self.parameter_derived:
                operands.append(self._raw(a))
                continue
            n, s = self._scaled(a)
            scale_shape = self.scale_shapes[a]
            value_shape_is_known = len(self.value_shapes[a]) == len(input_string)
            scale_is_scalar = value_shape_is_known and not scale_shape
            scale_is_known = value_shape_is_known and (not scale_shape or len(scale_shape) == len(input_string))
            retained = "".join(label for label in output_string if label in input_string)
            reduction_axes = tuple(axis for axis, label in enumerate(input_string) if label not in output_string)
            if reduction_axes and not scale_is_scalar and (
                not scale_is_known or any(scale_shape[axis] != 1 for axis in reduction_axes)
            ):
                # one reference scale per contraction: the maximum over the reduced axes
                common = b.append(partial(ops.reduce, axes=reduction_axes, kind="max", keepdims=True), (s,))
                n = b.append(partial(ops.elementwise, "rescale"), (n, s, common))
                common_shape = tuple(1 if axis in reduction_axes else d for axis, d in enumerate(scale_shape))
            else:
                common, common_shape = s, scale_shape
            operands.append(n)
            scales.append((common, common_shape, scale_is_known, input_string, retained))

        if is_contraction_free_einsum(format_string) and all(known for _, _, known, _, _ in scales):
            # translate.py:350-370: keep the product normalised per operand, add the scales
            pos[result, "normalized"] = b.append(partial(linear_einsum, format_string), tuple(operands))
            result_scale: int | None = None
            result_shape: Shape = ()
            for scale, shape, _, input_string, _ in scales:
                if shape and input_string != output_string:
                    scale = b.append(partial(_broadcast_einsum_operand, input_string, output_string), (scale,))
                    shape = tuple(shape[input_string.index(label)] if label in input_string else 1 for label in output_string)
                if result_scale is None:
                    result_scale, result_shape = scale, shape
                else:
                    result_scale = b.append(partial(ops.elementwise, "add"), (result_scale, scale))
                    result_shape = _infer_binary_shape(result_shape, shape)
            if result_scale is None:
                raise ValueError("A contraction-free scaled einsum must have at least one non-parameter operand.")
            pos[result, "log_scale"] = result_scale
            self.scale_shapes[result] = result_shape
            return

        raw = b.append(partial(linear_einsum, format_string), tuple(operands))
        normalized, log_scale = self._pair(partial(ops.fiber_normalize, kind=self.norm), raw)
        pos[result, "normalized"] = normalized
        result_shape = _fiber_scale_shape(self.value_shapes[result])
        for scale, shape, known, input_string, retained in scales:
            broadcasts = known and len(shape) == len(output_string) and all(
                d == 1 or il == ol for d, il, ol in zip(shape, input_string, output_string, strict=True)
            )
            if (not known or shape) and not broadcasts:
                scale = b.append(partial(linear_einsum, f"{input_string}->{retained}"), (scale,))
            if retained and (not known or shape) and not broadcasts:
                scale = b.append(partial(_reshape_einsum_shift, retained, output_string), (scale,))
            if shape and not broadcasts:
                shape = tuple(shape[input_string.index(label)] if label in input_string else 1 for label in output_string) if retained else ()
            log_scale = b.append(partial(ops.elementwise, "add"), (log_scale, scale))
            result_shape = _infer_binary_shape(result_shape, shape)
        pos[result, "log_scale"] = log_scale
        self.scale_shapes[result] = result_shape
