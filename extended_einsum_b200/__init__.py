"""B200 (sm_100a) kernels for extended_einsum's stable-materialization hot path.

Public surface:

* the expression API of the reference for this path (``array``, ``exp``,
  ``log``, ``einsum``, ``softmax``, ``stack``, ``take``, ``slice``,
  ``select``, ``Parameter``, ``extract_program``; ``materialize``), built on
  the same IR;
* ``lower(rich_program)`` -> BackendProgram of fused kernel calls, and
  ``run_program`` / ``B200Compiler`` to execute it;
* ``enable()`` routes the reference package's own
  ``TensorExpression.materialize`` (interface/tensor_expression.py:104-117)
  through ``lower`` for the log-space and scaled modes when every input is
  a CUDA tensor;
* ``ops`` — the torch-tensor entry points of libxe_b200.so;
* ``circuit`` — the folded quad-tree circuit driver.
"""

from __future__ import annotations

from . import ops
from .frontend import (
    BackendArrayWrapper,
    Parameter,
    RichInstruction,
    RichProgram,
    TensorExpression,
    array,
    dense_program,
    einsum,
    exp,
    extract_program,
    log,
    select,
    slice,
    softmax,
    stack,
    take,
)
from .lowering import B200Compiler, BackendProgram, lower, materialize, run_program

__all__ = [
    "B200Compiler",
    "BackendArrayWrapper",
    "BackendProgram",
    "Parameter",
    "RichInstruction",
    "RichProgram",
    "TensorExpression",
    "array",
    "dense_program",
    "einsum",
    "enable",
    "exp",
    "extract_program",
    "log",
    "lower",
    "materialize",
    "ops",
    "run_program",
    "select",
    "slice",
    "softmax",
    "stack",
    "take",
]

_ORIGINAL_MATERIALIZE = None
STABLE_MODES = ("logspace_max", "logspace_min", "scaled_sum", "scaled_max", "scaled_min")


def enable() -> None:
    """Routes the reference's TensorExpression.materialize through the B200 lowering.

    Applies to the log-space and scaled stability modes when every input of
    the expression is a CUDA float32 tensor; every other call goes to the reference's own
    implementation unchanged.  Requires the reference package (extended_einsum).
    """
    global _ORIGINAL_MATERIALIZE
    import torch
    from extended_einsum.interface import tensor_expression as reference

    if _ORIGINAL_MATERIALIZE is not None:
        return
    original = reference.TensorExpression.materialize

    def materialize_on_b200(self, stability_mode="unstable"):
        if stability_mode in STABLE_MODES:
            program, arguments = reference.extract_program(self, stability_mode)
            tensors = [a.backend_array for a in arguments]
            if all(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float32 for t in tensors):
                self._rich_program, self._input_arguments = program, arguments
                self._backend_program = lower(program)
                self._backend_code = B200Compiler.compile(self._backend_program, tensors)
                from extended_einsum.interface.functions import BackendArrayWrapper as ReferenceWrapper

                return ReferenceWrapper(self._backend_code(tensors), self.format)
        return original(self, stability_mode)

    reference.TensorExpression.materialize = materialize_on_b200
    _ORIGINAL_MATERIALIZE = original


def disable() -> None:
    """Restores the reference's own TensorExpression.materialize."""
    global _ORIGINAL_MATERIALIZE
    if _ORIGINAL_MATERIALIZE is None:
        return
    from extended_einsum.interface import tensor_expression as reference

    reference.TensorExpression.materialize = _ORIGINAL_MATERIALIZE
    _ORIGINAL_MATERIALIZE = None
