"""The drop-in hook on the host: enable() / disable() patch and restore the
reference package's own TensorExpression.materialize
(interface/tensor_expression.py:104-117), and inputs that are not CUDA
float32 tensors keep the reference's implementation.  Needs the reference
package installed in baseline/_ref; runs no kernel."""

from __future__ import annotations

import numpy as np

import extended_einsum_b200 as xb


def test_enable_patches_and_disable_restores(reference_xe):
    from extended_einsum.interface.tensor_expression import TensorExpression

    original = TensorExpression.materialize
    xb.enable()
    try:
        assert TensorExpression.materialize is not original
        xb.enable()  # idempotent
        assert xb._ORIGINAL_MATERIALIZE is original
    finally:
        xb.disable()
    assert TensorExpression.materialize is original
    xb.disable()  # idempotent
    assert TensorExpression.materialize is original


def test_non_cuda_inputs_keep_the_reference_path(reference_xe):
    """numpy inputs go to the reference's numpy executor unchanged, in every stable mode."""
    xe = reference_xe
    from extended_einsum.backend_translation.runtime import run_program
    from extended_einsum.backend_translation.translate import translate_to_backend_program
    from extended_einsum.backends.numpy import NumpyBackendFunctions

    rng = np.random.default_rng(0)
    a = np.log(rng.random((5, 7)))
    b = np.log(rng.random((7, 3)))
    xb.enable()
    try:
        for mode in xb.STABLE_MODES:
            expr = xe.log(xe.einsum("ik,kj->ij", xe.exp(xe.array(a)), xe.exp(xe.array(b))))
            got = expr.materialize(stability_mode=mode).backend_array
            program, arguments = xe.extract_program(expr, mode)
            expected = run_program(translate_to_backend_program(program, NumpyBackendFunctions()), [x.backend_array for x in arguments])
            np.testing.assert_array_equal(got, expected)
            assert not isinstance(expr._backend_program, xb.BackendProgram)
    finally:
        xb.disable()
