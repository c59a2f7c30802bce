"""Lowering of a stable RichProgram onto the sm_100a kernels.

``lower(program)`` walks the program exactly like the reference's
``_translate_logspace`` (backend_translation/translate.py:604-810): every SSA
value lives in a raw and/or a log-space position, converted lazily and at
most once (translate.py:631-644); exp and log only move a value between the
two (translate.py:764-769); softmax is raw in / raw out (:770-773);
parameter-derived values stay linear inside einsums (:594-601, :723-725).
The difference is what each instruction emits: the reference appends 11-22
generic backend calls per stable einsum, this lowering appends one call into
libxe_b200.so (contraction.py), so a BackendProgram here is a short list of kernel
launches.

One pattern of the folded circuits is fused across instructions: a
Hadamard product of two log-domain values with identical labels (the folded
'cab,cab->cab' over the two slice halves of the previous level, or 'ab,ab->ab'
over two selects at the root; translate.py:706-718 lowers it to a log add)
whose only consumer is a two-operand contraction becomes the fused addend
(``a2``) of that contraction, so the product is never written to memory.
The arithmetic is unchanged: the kernel adds the two values in fp32 before
the row shift, as the separate log add would.

The result is a ``BackendProgram`` with the reference's structure
(backend.py:81-85) that ``run_program`` (runtime.py:9-21) executes.
"""

from __future__ import annotations

from collections import Counter
from collections.abc import Callable, Sequence
from dataclasses import dataclass, field
from functools import partial
from typing import Any

import torch

from . import contraction as _contraction
from . import ops
from .frontend import BackendArrayWrapper, extract_program, is_contraction_free_einsum, parse_format_string

LOGSPACE_SHIFTS = {"logspace_max": "max", "logspace_min": "min"}


@dataclass(frozen=True)
class BackendProgram:
    backend_calls: list[Callable[[Sequence[torch.Tensor]], torch.Tensor]]
    call_arguments: list[tuple[int, ...]]
    n_inputs: int


def run_program(program: BackendProgram, inputs: Sequence[torch.Tensor]) -> torch.Tensor:
    """Runs the calls in order and returns the last value (runtime.py:9-21)."""
    if len(inputs) != program.n_inputs:
        raise ValueError(f"The number of inputs ({len(inputs)}) does not match the number of inputs ({program.n_inputs}) in the program.")
    tensors: list[torch.Tensor] = list(inputs)
    for call, arguments in zip(program.backend_calls, program.call_arguments):
        tensors.append(call([tensors[a] for a in arguments]))
    return tensors[-1]


def _call(fn: Callable[..., torch.Tensor]) -> Callable[[Sequence[torch.Tensor]], torch.Tensor]:
    def backend_call(tensors: Sequence[torch.Tensor]) -> torch.Tensor:
        return fn(*tensors)

    backend_call.fn = fn  # type: ignore[attr-defined]
    return backend_call


@dataclass
class _Builder:
    n_inputs: int
    backend_calls: list[Callable[[Sequence[torch.Tensor]], torch.Tensor]] = field(default_factory=list)
    call_arguments: list[tuple[int, ...]] = field(default_factory=list)

    @property
    def last_position(self) -> int:
        return self.n_inputs + len(self.backend_calls) - 1

    def append(self, fn: Callable[..., torch.Tensor], arguments: tuple[int, ...]) -> int:
        self.backend_calls.append(_call(fn))
        self.call_arguments.append(arguments)
        return self.last_position

    def build(self) -> BackendProgram:
        return BackendProgram(self.backend_calls, self.call_arguments, self.n_inputs)


def parameter_derived_ssa_ids(program: Any) -> frozenset[int]:
    """SSA values whose complete dependency chain consists of parameters (translate.py:594-601)."""
    derived = set(program.parameter_indices)
    for index, instruction in enumerate(program.instructions):
        if instruction.argument_ssa_ids and all(a in derived for a in instruction.argument_ssa_ids):
            derived.add(program.n_inputs + index)
    return frozenset(derived)


def lower(program: Any) -> BackendProgram:
    """Lowers a RichProgram in a log-space or scaled stability mode onto the B200 kernels.

    Mode dispatch as in translate_to_backend_program (translate.py:32-41):
    logspace_max / logspace_min -> the log-space lowering below,
    scaled_sum / scaled_max / scaled_min -> scaled.py; anything else is
    NotImplementedError (the unstable mode has nothing to stabilise).
    """
    from .scaled import SCALED_NORMS, _ScaledLowering

    mode = program.stability_mode
    if mode in LOGSPACE_SHIFTS:
        return _LogspaceLowering(program, LOGSPACE_SHIFTS[mode]).run()
    if mode in SCALED_NORMS:
        return _ScaledLowering(program, SCALED_NORMS[mode], _Builder(program.n_inputs), parameter_derived_ssa_ids(program)).run()
    raise NotImplementedError(f"The B200 lowering is not implemented for stability mode {mode}.")


class _LogspaceLowering:
    def __init__(self, program: Any, shift: str) -> None:
        self.program = program
        self.shift = shift
        self.builder = _Builder(program.n_inputs)
        self.positions: dict[tuple[int, str], int] = {(i, "raw"): i for i in range(program.n_inputs)}
        self.parameter_derived = parameter_derived_ssa_ids(program)
        # Hadamard products held back to be fused into their consumer: ssa -> (log position, log position)
        self.deferred: dict[int, tuple[int, int]] = {}
        self.uses = Counter(a for instruction in program.instructions for a in instruction.argument_ssa_ids)
        self.uses[program.output_ssa] += 1
        self.consumer: dict[int, Any] = {}
        for instruction in program.instructions:
            for a in instruction.argument_ssa_ids:
                self.consumer[a] = instruction

    def run(self) -> BackendProgram:
        for index, instruction in enumerate(self.program.instructions):
            self._instruction(instruction, self.program.n_inputs + index)
        output = self._raw(self.program.output_ssa)
        if output != self.builder.last_position:
            raise ValueError("The raw value of the program's output must be the last computed tensor, because the runtime returns the last tensor.")
        return self.builder.build()

    # lazy domain conversion (translate.py:631-644)
    def _raw(self, ssa: int) -> int:
        if (ssa, "raw") not in self.positions:
            self.positions[ssa, "raw"] = self.builder.append(ops.exp, (self.positions[ssa, "logspace"],))
        return self.positions[ssa, "raw"]

    def _log(self, ssa: int) -> int:
        if (ssa, "logspace") not in self.positions:
            if ssa in self.deferred:
                # a held-back Hadamard product whose consumer could not take it fused
                self.positions[ssa, "logspace"] = self.builder.append(ops.log_add, self.deferred.pop(ssa))
            else:
                self.positions[ssa, "logspace"] = self.builder.append(ops.log, (self.positions[ssa, "raw"],))
        return self.positions[ssa, "logspace"]

    def _defer_hadamard(self, format_string: str, args: tuple[int, ...], result: int) -> bool:
        """Holds back a log-space Hadamard product whose single consumer is a binary contraction."""
        input_strings, output_string = parse_format_string(format_string)
        if len(args) != 2 or input_strings[0] != output_string or input_strings[1] != output_string:
            return False
        if any(a in self.parameter_derived for a in args) or result in self.parameter_derived:
            return False
        if self.uses[result] != 1 or result == self.program.output_ssa or result not in self.consumer:
            return False
        consumer = self.consumer[result]
        if consumer.operator.name != "einsum" or len(consumer.argument_ssa_ids) != 2 or consumer.argument_ssa_ids.count(result) != 1:
            return False
        if is_contraction_free_einsum(consumer.operator.format_string):
            return False
        self.deferred[result] = (self._log(args[0]), self._log(args[1]))
        return True

    def _instruction(self, instruction: Any, result: int) -> None:
        op = instruction.operator
        args = instruction.argument_ssa_ids
        name = op.name
        b = self.builder
        if name == "exp":
            self.positions[result, "logspace"] = self._raw(args[0])
        elif name == "log":
            self.positions[result, "raw"] = self._log(args[0])
        elif name == "softmax":
            self.positions[result, "raw"] = b.append(partial(ops.softmax, axis=op.axis), (self._raw(args[0]),))
        elif name in ("+", "-"):
            logs = tuple(self._log(a) for a in args)
            fn = partial(ops.log_add_exp, subtract=name == "-", shift=self.shift)
            self.positions[result, "logspace"] = b.append(fn, logs)
        elif name == "*":
            self.positions[result, "logspace"] = b.append(ops.log_add, tuple(self._log(a) for a in args))
        elif name == "/":
            fn = partial(ops.log_add, negate_b=True)
            self.positions[result, "logspace"] = b.append(fn, tuple(self._log(a) for a in args))
        elif name in ("stack", "concat", "select", "slice"):
            # indexing and concatenation commute with the elementwise log (translate.py:798-801)
            self.positions[result, "logspace"] = b.append(_structural(op), tuple(self._log(a) for a in args))
        elif name == "take":
            fn = partial(_take, axis=op.axis)
            self.positions[result, "logspace"] = b.append(fn, (self._log(args[0]), self._raw(args[1])))
        elif name == "einsum":
            if not self._defer_hadamard(op.format_string, args, result):
                self._einsum(op.format_string, args, result)
        else:
            raise NotImplementedError(f"The operator {name} has no logspace backend translation.")

    def _einsum(self, format_string: str, args: tuple[int, ...], result: int) -> None:
        input_strings, _ = parse_format_string(format_string)
        if len(input_strings) != len(args):
            raise ValueError(f"The einsum format string has {len(input_strings)} inputs, but the instruction has {len(args)} arguments.")
        linear = tuple(a in self.parameter_derived for a in args)
        if is_contraction_free_einsum(format_string) and not any(linear):
            fn = partial(_contraction.log_broadcast_product, format_string)
            self.positions[result, "logspace"] = self.builder.append(fn, tuple(self._log(a) for a in args))
            return
        fused = [i for i, a in enumerate(args) if a in self.deferred and not linear[i]]
        if len(args) == 2 and fused:
            # the held-back Hadamard product becomes the fused addend of this contraction's first operand
            i = fused[0]
            other = 1 - i
            b_position = self._raw(args[other]) if linear[other] else self._log(args[other])
            a_position, a2_position = self.deferred.pop(args[i])
            _, output_string = parse_format_string(format_string)
            fmt = f"{input_strings[i]},{input_strings[other]}->{output_string}"
            fn = partial(_contraction.logspace_einsum_hadamard, fmt, linear[other], self.shift)
            self.positions[result, "logspace"] = self.builder.append(fn, (a_position, a2_position, b_position))
            return
        positions = tuple(self._raw(a) if lin else self._log(a) for a, lin in zip(args, linear))
        fn = partial(_contraction.logspace_einsum, format_string, linear, self.shift)
        self.positions[result, "logspace"] = self.builder.append(fn, positions)


def _structural(op: Any) -> Callable[..., torch.Tensor]:
    name = op.name
    if name == "stack":
        return lambda *ts: torch.stack(ts, dim=op.axis)
    if name == "concat":
        return lambda *ts: torch.cat(ts, dim=op.axis)
    if name == "select":
        return lambda t: torch.select(t, op.axis, op.index)
    if name == "slice":
        return lambda t: t.narrow(op.axis if op.axis >= 0 else op.axis + t.dim(), op.start, op.stop - op.start)
    raise NotImplementedError(name)


def _take(source: torch.Tensor, indices: torch.Tensor, axis: int) -> torch.Tensor:
    return torch.index_select(source, axis, indices)


# ---------------------------------------------------------------------------
# compile / materialize (backend.py:88-93, tensor_expression.py:104-117)


class B200Compiler:
    """Compiles a lowered program into a callable (BackendCompiler protocol)."""

    @staticmethod
    def compile(program: BackendProgram, inputs: Sequence[torch.Tensor]) -> Callable[[Sequence[torch.Tensor]], torch.Tensor]:
        if len(inputs) != program.n_inputs:
            raise ValueError(f"The number of inputs ({len(inputs)}) does not match the number of inputs ({program.n_inputs}) in the program.")
        return partial(run_program, program)


def materialize(expression: Any, stability_mode: str) -> BackendArrayWrapper:
    """extract_program -> lower -> compile -> run, returning a wrapped result."""
    program, arguments = extract_program(expression, stability_mode)
    backend_program = lower(program)
    from .frontend import input_tensor

    tensors = [input_tensor(a) for a in arguments]
    code = B200Compiler.compile(backend_program, tensors)
    return BackendArrayWrapper(code(tensors), getattr(expression, "format", "dense"))
