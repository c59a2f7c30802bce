"""Expression front end for the stable-materialization path.

A host-side mirror of the parts of extended_einsum's public API that the
log-space hot path uses, with the same names, argument meaning and errors:

* operators and IR: language/rich_operators.py (OperatorExp ... OperatorEinsum),
  language/rich_instruction.py, language/rich_program.py:9-62
* expressions: interface/tensor_expression.py:44-265 (Parameter,
  TensorExpression, extract_program)
* builders: interface/functions.py:52-173 (array, exp, log, einsum, stack,
  take, slice, select, softmax)

It exists so that programs can be built and materialized where the reference
package is not installed (a GPU host).  The lowering in ``lowering.py`` only
looks at ``operator.name`` and the operator attributes, so it accepts both
these objects and the reference's own.
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass, field
from typing import Any, Literal

import numpy as np

StabilityMode = Literal["unstable", "scaled_min", "scaled_max", "scaled_sum", "logspace_min", "logspace_max"]
Shape = tuple[int, ...]


def parse_format_string(format_string: str) -> tuple[list[str], str]:
    """Splits 'ab,bc->ac' into (['ab', 'bc'], 'ac') (utils.py:9-30)."""
    arrow_split = format_string.split("->")
    if len(arrow_split) != 2:
        raise ValueError(f'"{format_string}" is not a valid einsum format string.')
    inputs, output = arrow_split
    return [part.strip() for part in inputs.split(",")], output.strip()


def is_contraction_free_einsum(format_string: str) -> bool:
    """Whether an einsum only broadcasts and multiplies operands (utils.py:33-42)."""
    input_strings, output_string = parse_format_string(format_string)
    output_labels = set(output_string)
    return (
        len(output_string) == len(output_labels)
        and all(len(s) == len(set(s)) and set(s) <= output_labels for s in input_strings)
        and set().union(*map(set, input_strings)) == output_labels
    )


def normalize_axis(axis: int, rank: int) -> int:
    if rank <= 0:
        raise ValueError("axis normalization requires a positive rank")
    normalized = axis + rank if axis < 0 else axis
    if normalized < 0 or normalized >= rank:
        raise ValueError(f"axis {axis} is out of bounds for rank {rank}")
    return normalized


# ---------------------------------------------------------------------------
# operators (rich_operators.py)


def _axis_sizes(index_strings: list[str], shapes: list[Shape]) -> dict[str, int]:
    sizes: dict[str, int] = {}
    for index_string, shape in zip(index_strings, shapes):
        for position, label in enumerate(index_string):
            if label not in sizes:
                sizes[label] = shape[position]
            elif sizes[label] != shape[position]:
                raise RuntimeError(f"Incompatible axis sizes for index {label}: {sizes[label]} and {shape[position]}.")
    return sizes


class _Unary:
    def check_inputs(self, operands: list[Any]) -> None:
        if len(operands) != 1:
            raise ValueError(f"The {self.name} operator takes exactly one argument, but {len(operands)} were given.")

    def propagate_shapes(self, input_shapes: list[Shape]) -> Shape:
        return tuple(input_shapes[0])


class _Binary:
    def check_inputs(self, operands: list[Any]) -> None:
        if len(operands) != 2:
            raise ValueError(f"The {self.name} operator takes exactly two arguments, but {len(operands)} were given.")

    def propagate_shapes(self, input_shapes: list[Shape]) -> Shape:
        return tuple(np.broadcast_shapes(input_shapes[0], input_shapes[1]))


@dataclass(frozen=True)
class OperatorExp(_Unary):
    name = "exp"


@dataclass(frozen=True)
class OperatorLog(_Unary):
    name = "log"


@dataclass(frozen=True)
class OperatorAdd(_Binary):
    name = "+"


@dataclass(frozen=True)
class OperatorSubtract(_Binary):
    name = "-"


@dataclass(frozen=True)
class OperatorMultiply(_Binary):
    name = "*"


@dataclass(frozen=True)
class OperatorDivide(_Binary):
    name = "/"


@dataclass(frozen=True)
class OperatorStack:
    axis: int
    name = "stack"

    def check_inputs(self, operands: list[Any]) -> None:
        if not operands:
            raise ValueError("The stack operator requires at least one argument.")
        if any(tuple(o.shape) != tuple(operands[0].shape) for o in operands[1:]):
            raise ValueError("The stack operator requires all arguments to have the same shape along the stack axis.")

    def propagate_shapes(self, input_shapes: list[Shape]) -> Shape:
        s = tuple(input_shapes[0])
        return (*s[: self.axis], len(input_shapes), *s[self.axis :])


@dataclass(frozen=True)
class OperatorConcat:
    axis: int
    name = "concat"

    def check_inputs(self, operands: list[Any]) -> None:
        if not operands:
            raise ValueError("The concat operator requires at least one argument.")

    def propagate_shapes(self, input_shapes: list[Shape]) -> Shape:
        s = list(input_shapes[0])
        s[self.axis] = sum(shape[self.axis] for shape in input_shapes)
        return tuple(s)


@dataclass(frozen=True)
class OperatorTake:
    axis: int
    name = "take"

    def check_inputs(self, operands: list[Any]) -> None:
        if len(operands) != 2:
            raise ValueError(f"The take operator takes exactly two arguments, but {len(operands)} were given.")

    def propagate_shapes(self, input_shapes: list[Shape]) -> Shape:
        s, idx = tuple(input_shapes[0]), tuple(input_shapes[1])
        if len(idx) != 1:
            raise ValueError("take requires an index with rank 1")
        return (*s[: self.axis], *idx, *s[self.axis + 1 :])


@dataclass(frozen=True)
class OperatorSlice:
    start: int
    stop: int
    axis: int
    name = "slice"

    def check_inputs(self, operands: list[Any]) -> None:
        if len(operands) != 1:
            raise ValueError(f"The slice operator takes exactly one argument, but {len(operands)} were given.")

    def propagate_shapes(self, input_shapes: list[Shape]) -> Shape:
        s = tuple(input_shapes[0])
        return (*s[: self.axis], self.stop - self.start, *s[self.axis + 1 :])


@dataclass(frozen=True)
class OperatorSelect:
    axis: int
    index: int
    name = "select"

    def check_inputs(self, operands: list[Any]) -> None:
        if len(operands) != 1:
            raise ValueError(f"The select operator takes exactly one argument, but {len(operands)} were given.")

    def propagate_shapes(self, input_shapes: list[Shape]) -> Shape:
        s = tuple(input_shapes[0])
        return (*s[: self.axis], *s[self.axis + 1 :])


@dataclass(frozen=True)
class OperatorSoftmax:
    axis: int | tuple[int, ...]
    name = "softmax"

    def check_inputs(self, operands: list[Any]) -> None:
        if len(operands) != 1:
            raise ValueError(f"The softmax operator takes exactly one argument, but {len(operands)} were given.")
        rank = len(operands[0].shape)
        if rank == 0:
            raise ValueError(f"The softmax operator takes a non-scalar as first arguments, but the first argument has shape {operands[0].shape}.")
        axes = (self.axis,) if isinstance(self.axis, int) else self.axis
        if not axes:
            raise ValueError("The softmax operator requires at least one axis.")
        if len(set(axes)) != len(axes):
            raise ValueError(f"The softmax operator axes must be unique, got {axes}.")
        if any(not 0 <= a < rank for a in axes):
            raise ValueError(f"The softmax operator wants to softmax axes {axes} but the operand only has {rank} axes.")

    def propagate_shapes(self, input_shapes: list[Shape]) -> Shape:
        return tuple(input_shapes[0])


@dataclass(frozen=True)
class OperatorEinsum:
    format_string: str
    name = "einsum"

    def __post_init__(self) -> None:
        index_strings, output_string = parse_format_string(self.format_string)
        if any(symbol not in set().union(*index_strings) for symbol in output_string):
            raise ValueError(f"Einsum format string error: an output symbol in {output_string} is not present in the input index strings.")

    def check_inputs(self, operands: list[Any]) -> None:
        index_strings, _ = parse_format_string(self.format_string)
        if len(index_strings) != len(operands):
            raise ValueError(f"The number of indices in the einsum format string ({len(index_strings)}) does not match the number of arguments ({len(operands)}).")
        if any(len(s) != len(o.shape) for s, o in zip(index_strings, operands)):
            raise ValueError(f"The einsum format string ({self.format_string}) has indices of different lengths than the order of the operands.")
        _axis_sizes(index_strings, [tuple(o.shape) for o in operands])

    def propagate_shapes(self, input_shapes: list[Shape]) -> Shape:
        index_strings, output_string = parse_format_string(self.format_string)
        sizes = _axis_sizes(index_strings, [tuple(s) for s in input_shapes])
        return tuple(sizes[label] for label in output_string)


# ---------------------------------------------------------------------------
# IR (rich_instruction.py, rich_program.py)


@dataclass(frozen=True)
class RichInstruction:
    operator: Any
    argument_ssa_ids: tuple[int, ...]


@dataclass(frozen=True)
class RichProgram:
    instructions: list[RichInstruction]
    n_inputs: int
    stability_mode: StabilityMode
    tensor_formats: list[str]
    shapes: list[Shape]
    parameter_indices: frozenset[int]
    arguments_of_ssa_id: dict[int, tuple[int, ...]] = field(init=False)
    consumers_of_ssa_id: dict[int, list[int]] = field(init=False)

    def __post_init__(self) -> None:
        n_ssa_ids = self.n_inputs + len(self.instructions)
        if len(self.shapes) != n_ssa_ids:
            raise ValueError(f"Number of shapes ({len(self.shapes)}) must match the expected number of SSA IDs ({self.n_inputs} inputs + {len(self.instructions)} instructions).")
        if len(self.tensor_formats) != n_ssa_ids:
            raise ValueError(f"Number of tensor formats ({len(self.tensor_formats)}) must match the expected number of SSA IDs ({self.n_inputs} inputs + {len(self.instructions)} instructions).")
        arguments: dict[int, tuple[int, ...]] = defaultdict(tuple)
        consumers: dict[int, list[int]] = defaultdict(list)
        for i, instruction in enumerate(self.instructions):
            arguments[self.n_inputs + i] = instruction.argument_ssa_ids
            for argument in instruction.argument_ssa_ids:
                consumers[argument].append(self.n_inputs + i)
        object.__setattr__(self, "arguments_of_ssa_id", arguments)
        object.__setattr__(self, "consumers_of_ssa_id", consumers)

    @property
    def output_ssa(self) -> int:
        return self.n_inputs + len(self.instructions) - 1


def dense_program(
    instructions: list[RichInstruction],
    n_inputs: int,
    stability_mode: StabilityMode,
    parameter_indices: frozenset[int] = frozenset(),
    shapes: list[Shape] | None = None,
) -> RichProgram:
    """A RichProgram with dense formats, as the reference's tests build them."""
    n = n_inputs + len(instructions)
    return RichProgram(
        instructions=list(instructions),
        n_inputs=n_inputs,
        stability_mode=stability_mode,
        tensor_formats=["dense"] * n,
        shapes=[()] * n if shapes is None else list(shapes),
        parameter_indices=frozenset(parameter_indices),
    )


# ---------------------------------------------------------------------------
# expressions (tensor_expression.py, functions.py)


@dataclass(frozen=True)
class BackendArrayWrapper:
    """A backend array with a tensor format (functions.py:23-41)."""

    backend_array: Any
    _format: str = "dense"

    @property
    def shape(self) -> Shape:
        return tuple(self.backend_array.shape)

    @property
    def backend(self) -> str:
        return "torch"

    @property
    def format(self) -> str:
        return self._format


def array(backend_array: Any, format: str = "dense") -> BackendArrayWrapper:
    return BackendArrayWrapper(backend_array, format)


@dataclass(frozen=True)
class Parameter:
    """Marks an input whose derived values stay linear in stable einsums."""

    array: Any

    @property
    def shape(self) -> Shape:
        return tuple(self.array.shape)

    @property
    def format(self) -> str:
        return getattr(self.array, "format", "dense")


class TensorExpression:
    def __init__(self, operator: Any, arguments: list[Any]) -> None:
        if len(arguments) == 0:
            raise ValueError("Tensor expression must have at least one argument.")
        self.operator = operator
        self.arguments = arguments
        operator.check_inputs(arguments)
        self._shape = tuple(operator.propagate_shapes([tuple(a.shape) for a in arguments]))
        self.format = "dense"

    @property
    def shape(self) -> Shape:
        return self._shape

    def materialize(self, stability_mode: StabilityMode = "unstable") -> BackendArrayWrapper:
        from .lowering import materialize

        return materialize(self, stability_mode)

    def __add__(self, other: Any) -> TensorExpression:
        return TensorExpression(OperatorAdd(), [self, other])

    def __sub__(self, other: Any) -> TensorExpression:
        return TensorExpression(OperatorSubtract(), [self, other])

    def __mul__(self, other: Any) -> TensorExpression:
        return TensorExpression(OperatorMultiply(), [self, other])

    def __truediv__(self, other: Any) -> TensorExpression:
        return TensorExpression(OperatorDivide(), [self, other])

    def __matmul__(self, other: Any) -> TensorExpression:
        return TensorExpression(OperatorEinsum("ik, kj -> ij"), [self, other])


def exp(a: Any) -> TensorExpression:
    return TensorExpression(OperatorExp(), [a])


def log(a: Any) -> TensorExpression:
    return TensorExpression(OperatorLog(), [a])


def einsum(format_string: str, *operands: Any) -> TensorExpression:
    index_strings, output_string = parse_format_string(format_string)
    if len(index_strings) != len(operands):
        raise ValueError(f"format string {format_string} has {len(index_strings)} indices, but {len(operands)} operands.")
    if any(symbol not in frozenset("".join(index_strings)) for symbol in output_string):
        raise ValueError(f"format string {format_string} contains output symbols that are not present in the operands.")
    return TensorExpression(OperatorEinsum(format_string), list(operands))


def stack(operands: list[Any], *, axis: int = 0) -> TensorExpression:
    if len(operands) == 0:
        raise ValueError("stack requires at least one argument")
    axis = normalize_axis(axis, len(operands[0].shape))
    return TensorExpression(OperatorStack(axis), list(operands))


def take(source: Any, index: Any, *, axis: int = 0) -> TensorExpression:
    if not source.shape:
        raise ValueError("The take operator requires an operand with a leading axis.")
    if not index.shape:
        raise ValueError("The take operator requires an index with a leading axis.")
    return TensorExpression(OperatorTake(normalize_axis(axis, len(source.shape))), [source, index])


def slice(source: Any, start: int, stop: int, *, axis: int = 0) -> TensorExpression:  # noqa: A001
    return TensorExpression(OperatorSlice(start, stop, normalize_axis(axis, len(source.shape))), [source])


def select(source: Any, index: int, *, axis: int = 0) -> TensorExpression:
    return TensorExpression(OperatorSelect(normalize_axis(axis, len(source.shape)), index), [source])


def softmax(a: Any, axis: int | tuple[int, ...] = 0) -> TensorExpression:
    """Applies the softmax function to the input tensor (functions.py:159-173)."""
    if not a.shape:
        raise ValueError("softmax requires an input tensor with at least one axis")
    axes = (axis,) if isinstance(axis, int) else axis
    if not axes:
        raise ValueError("softmax requires at least one axis")
    normalized = tuple(normalize_axis(item, len(a.shape)) for item in axes)
    return TensorExpression(OperatorSoftmax(normalized[0] if len(normalized) == 1 else normalized), [a])


def _is_expression(node: Any) -> bool:
    return hasattr(node, "operator") and hasattr(node, "arguments")


def _is_parameter(node: Any) -> bool:
    return type(node).__name__ == "Parameter" and hasattr(node, "array")


def input_tensor(node: Any) -> Any:
    """The backend array behind an input leaf (a wrapper, a Parameter, or a raw tensor)."""
    if _is_parameter(node):
        node = node.array
    return getattr(node, "backend_array", node)


def extract_program(expression: Any, stability_mode: StabilityMode) -> tuple[RichProgram, list[Any]]:
    """SSA program of an expression tree (tensor_expression.py:138-265).

    Inputs get SSA ids 0..n-1 in order of first appearance in a depth-first
    traversal, instructions follow in post-order; Parameter leaves are
    recorded in ``parameter_indices``.  Works on this module's expressions and
    on the reference's.
    """
    instructions: list[RichInstruction] = []
    ssa_ids: dict[int, int] = {}
    input_ids: dict[int, int] = {}
    inputs: list[Any] = []
    parameters: list[int] = []
    shapes: dict[int, Shape] = {}

    def visit(node: Any) -> int:
        key = id(node)
        if not _is_expression(node):
            if key in input_ids:
                return input_ids[key]
            input_ids[key] = -1 - len(input_ids)
            inputs.append(node.array if _is_parameter(node) else node)
            if _is_parameter(node):
                parameters.append(input_ids[key])
            shapes[input_ids[key]] = tuple(node.shape)
            return input_ids[key]
        if key in ssa_ids:
            return ssa_ids[key]
        arguments = tuple(visit(a) for a in node.arguments)
        ssa_ids[key] = len(ssa_ids)
        instructions.append(RichInstruction(node.operator, arguments))
        shapes[ssa_ids[key]] = tuple(node.shape)
        return ssa_ids[key]

    visit(expression)
    n_inputs = len(input_ids)

    def shift(old: int) -> int:
        return old + n_inputs if old >= 0 else -1 - old

    instructions = [RichInstruction(i.operator, tuple(map(shift, i.argument_ssa_ids))) for i in instructions]
    n = n_inputs + len(ssa_ids)
    shape_list: list[Shape] = [()] * n
    for key, shape in shapes.items():
        shape_list[shift(key)] = shape
    program = RichProgram(
        instructions=instructions,
        n_inputs=n_inputs,
        stability_mode=stability_mode,
        tensor_formats=["dense"] * n,
        shapes=shape_list,
        parameter_indices=frozenset(shift(p) for p in parameters),
    )
    return program, inputs
