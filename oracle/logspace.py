"""CPU oracle for the log-space path: a numpy restatement of extended_einsum's
stable log-space translation.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (the extended_einsum_b200
package) imports this module; it is used by tests/, __graft_entry__.smoke()
and bench.py's CPU baseline, as the checker.

Parity is pinned: tests/test_oracle_golden.py checks every function here
against golden vectors produced by running the reference itself
(tests/golden/make_golden.py) and against the reference's own known-answer
tests (tests/test_backend_translation.py of the reference).

Paths cited are relative to the extended_einsum project root.  Every array
operation follows the backend call the reference emits, in the same order, in
the dtype of the inputs (float32 mirrors the reference's torch fp32 path,
float64 is the ground truth).
"""

from __future__ import annotations

from typing import Any

import numpy as np


def parse_format_string(format_string: str) -> tuple[list[str], str]:
    """utils.py:9-30"""
    inputs, output = format_string.split("->")
    return [s.strip() for s in inputs.split(",")], output.strip()


def is_contraction_free_einsum(format_string: str) -> bool:
    """utils.py:33-42"""
    input_strings, output_string = parse_format_string(format_string)
    labels = set(output_string)
    return (
        len(output_string) == len(labels)
        and all(len(s) == len(set(s)) and set(s) <= labels for s in input_strings)
        and set().union(*map(set, input_strings)) == labels
    )


def _einsum(format_string: str, *operands: np.ndarray) -> np.ndarray:
    """TorchBackendFunctions.einsum (backends/torch.py:115-118); BLAS-backed for pairs."""
    dtype = np.result_type(*operands)
    return np.asarray(np.einsum(format_string.replace(" ", ""), *operands, optimize=True), dtype=dtype)


def _extreme(mode: str):
    return np.max if mode == "max" else np.min


def _reshape_shift(shift: np.ndarray, retained: str, output_string: str) -> np.ndarray:
    """_reshape_einsum_shift, translate.py:667-672"""
    dims = iter(shift.shape)
    return shift.reshape(tuple(next(dims) if label in retained else 1 for label in output_string))


def _broadcast_operand(operand: np.ndarray, input_string: str, output_string: str) -> np.ndarray:
    """_broadcast_einsum_operand, translate.py:675-683"""
    retained = "".join(label for label in output_string if label in input_string)
    if input_string != retained:
        operand = _einsum(f"{input_string}->{retained}", operand)
    dims = iter(operand.shape)
    return operand.reshape(tuple(next(dims) if label in retained else 1 for label in output_string))


def logspace_einsum(
    format_string: str, operands: list[np.ndarray], linear: list[bool], mode: str = "max"
) -> np.ndarray:
    """_append_logspace_einsum, translate.py:686-750.

    ``operands[i]`` is a log-space value, or the raw value when ``linear[i]``
    (parameter-derived, translate.py:723-725).  Returns the log-space result.
    """
    input_strings, output_string = parse_format_string(format_string)
    if is_contraction_free_einsum(format_string) and not any(linear):  # :706-718
        aligned = [
            x if s == output_string else _broadcast_operand(x, s, output_string) for s, x in zip(input_strings, operands)
        ]
        result = aligned[0]
        for x in aligned[1:]:
            result = result + x
        return result
    norm = _extreme(mode)
    raw_operands = []
    shifts = []
    for input_string, x, lin in zip(input_strings, operands, linear):
        if lin:
            raw_operands.append(x)
            continue
        retained = "".join(label for label in output_string if label in input_string)
        axes = tuple(a for a, label in enumerate(input_string) if label not in output_string)
        if not axes:
            shift = x
        elif retained:
            shift = norm(x, axis=axes, keepdims=True)  # :733
        else:
            shift = norm(x)  # :735
        raw_operands.append(np.exp(x - shift))  # :739-740
        shifts.append((shift, input_string, retained))
    result = np.log(_einsum(format_string, *raw_operands))  # :743-744
    for shift, input_string, retained in shifts:  # :745-749
        if retained:
            shift = _reshape_shift(_einsum(f"{input_string}->{retained}", shift), retained, output_string)
        result = result + shift
    return result


def softmax(x: np.ndarray, axis: int | tuple[int, ...]) -> np.ndarray:
    """TorchBackendFunctions.softmax, backends/torch.py:102-113 (exp(x - max) normalised by the sum)."""
    shifted = x - np.max(x, axis=axis, keepdims=True)
    e = np.exp(shifted)
    return e / np.sum(e, axis=axis, keepdims=True)


def log_add_exp(a: np.ndarray, b: np.ndarray, subtract: bool, mode: str = "max") -> np.ndarray:
    """Log-space + / - with the common scalar shift, translate.py:774-789 and _append_shifted :647-664."""
    norm = _extreme(mode)
    shift = norm(np.stack([norm(a), norm(b)], axis=0))
    ea, eb = np.exp(a - shift), np.exp(b - shift)
    return np.log(ea - eb if subtract else ea + eb) + shift


def parameter_derived_ssa_ids(program: Any) -> frozenset[int]:
    """translate.py:594-601"""
    derived = set(program.parameter_indices)
    for index, instruction in enumerate(program.instructions):
        if instruction.argument_ssa_ids and all(a in derived for a in instruction.argument_ssa_ids):
            derived.add(program.n_inputs + index)
    return frozenset(derived)


def run_logspace(program: Any, inputs: list[np.ndarray]) -> np.ndarray:
    """_translate_logspace (translate.py:604-628) + run_program, as one interpreter.

    Values are kept in a raw and/or a log-space form and converted lazily
    (translate.py:631-644), exactly as the translated backend program would.
    Works on the reference's RichProgram and on extended_einsum_b200's.
    """
    mode = {"logspace_max": "max", "logspace_min": "min"}[program.stability_mode]
    raw: dict[int, np.ndarray] = dict(enumerate(inputs))
    logs: dict[int, np.ndarray] = {}
    derived = parameter_derived_ssa_ids(program)

    def as_raw(ssa: int) -> np.ndarray:
        if ssa not in raw:
            raw[ssa] = np.exp(logs[ssa])
        return raw[ssa]

    def as_log(ssa: int) -> np.ndarray:
        if ssa not in logs:
            logs[ssa] = np.log(raw[ssa])
        return logs[ssa]

    for index, instruction in enumerate(program.instructions):
        result = program.n_inputs + index
        op = instruction.operator
        args = instruction.argument_ssa_ids
        name = op.name
        if name == "exp":  # :764-766
            logs[result] = as_raw(args[0])
        elif name == "log":  # :767-769
            raw[result] = as_log(args[0])
        elif name == "softmax":  # :770-773
            raw[result] = softmax(as_raw(args[0]), op.axis)
        elif name in ("+", "-"):  # :774-789
            logs[result] = log_add_exp(as_log(args[0]), as_log(args[1]), name == "-", mode)
        elif name == "*":  # :790-793
            logs[result] = as_log(args[0]) + as_log(args[1])
        elif name == "/":  # :794-797
            logs[result] = as_log(args[0]) - as_log(args[1])
        elif name == "stack":  # :798-801
            logs[result] = np.stack([as_log(a) for a in args], axis=op.axis)
        elif name == "concat":
            logs[result] = np.concatenate([as_log(a) for a in args], axis=op.axis)
        elif name == "select":
            logs[result] = np.take(as_log(args[0]), op.index, axis=op.axis)
        elif name == "slice":
            x = as_log(args[0])
            index = [slice(None)] * x.ndim
            index[op.axis] = slice(op.start, op.stop)
            logs[result] = x[tuple(index)]
        elif name == "take":  # :802-806
            logs[result] = np.take(as_log(args[0]), as_raw(args[1]).astype(np.int64), axis=op.axis)
        elif name == "einsum":  # :807-808
            linear = [a in derived for a in args]
            operands = [as_raw(a) if lin else as_log(a) for a, lin in zip(args, linear)]
            logs[result] = logspace_einsum(op.format_string, operands, linear, mode)
        else:
            raise NotImplementedError(f"The operator {name} has no logspace backend translation.")
    return as_raw(program.output_ssa)


# ---------------------------------------------------------------------------
# The hot-path patterns as direct functions (same arithmetic as run_logspace).


def logspace_matmul(a: np.ndarray, b: np.ndarray, mode: str = "max") -> np.ndarray:
    """log(einsum('...ik,...kj->...ij', exp(a), exp(b))) in logspace mode (translate.py:686-750)."""
    norm = _extreme(mode)
    sa = norm(a, axis=-1, keepdims=True)
    sb = norm(b, axis=-2, keepdims=True)
    return (np.log(np.matmul(np.exp(a - sa), np.exp(b - sb))) + sa) + sb


def logspace_cp_layer(x: np.ndarray, w: np.ndarray, mode: str = "max") -> np.ndarray:
    """Folded CP sum layer 'fbi,foi->fbo' with linear weights w (translate.py:686-750).

    x: (F, B, K) log-space, w: (F, O, K) linear.
    """
    norm = _extreme(mode)
    s = norm(x, axis=2, keepdims=True)
    return np.log(np.matmul(np.exp(x - s), np.swapaxes(w, 1, 2))) + s


def logspace_tucker(left: np.ndarray, right: np.ndarray, w: np.ndarray, mode: str = "max") -> np.ndarray:
    """Tucker layer 'bfi,bfj,foij->bfo' with linear weights (translate.py:686-750, preprocess.py:1095-1106)."""
    norm = _extreme(mode)
    sl = norm(left, axis=2, keepdims=True)
    sr = norm(right, axis=2, keepdims=True)
    raw = _einsum("bfi,bfj,foij->bfo", np.exp(left - sl), np.exp(right - sr), w)
    return (np.log(raw) + sl) + sr
