"""The drop-in path end to end on the GPU: the reference package's own public
API (xe.array / xe.einsum / xe.softmax / TensorExpression.materialize,
interface/tensor_expression.py:104-117) with CUDA inputs, routed by
extended_einsum_b200.enable() through lower() onto the sm_100a kernels, and the
reference's own folded circuit program (FoldSameShapedOperations +
OptimizeContractionPaths, as demo/cirkit.py:478-479 builds it) through
lower() / run_program.  Every result is compared with the reference's torch
executor (translate_to_backend_program + TorchBackendFunctions + run_program)
on the same inputs on the CPU, in fp32:

* log-domain outputs: |ours - reference| <= 1e-5 + 2.4e-7 |reference|
  (north star tolerance 1e-5 absolute, plus two fp32 ulps of the value);
* raw (softmax) outputs: relative 2e-5;
* circuit log-likelihoods, whose fp32 error grows with depth in the
  reference too: within the log-domain bound of the reference's fp32 output,
  or no further from the reference's fp64 output (same executor, double
  inputs) than twice the reference fp32 output's own error.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import extended_einsum_b200 as xb
from conftest import LOG_ATOL, LOG_RTOL, log_close
from extended_einsum_b200.circuit import demo_circuit_inputs, demo_circuit_program

pytestmark = pytest.mark.gpu

DEVICE = torch.device("cuda", 0)


def reference_cpu(xe, program, inputs):
    """The reference's own torch executor on CPU tensors, fp32."""
    from extended_einsum.backend_translation.runtime import run_program
    from extended_einsum.backend_translation.translate import translate_to_backend_program
    from extended_einsum.backends.torch import TorchBackendFunctions

    backend_program = translate_to_backend_program(program, TorchBackendFunctions())
    return run_program(backend_program, [t.cpu() for t in inputs]).numpy()


def circuit_close(xe, program, inputs, ours) -> None:
    expected32 = reference_cpu(xe, program, inputs)
    assert ours.shape == expected32.shape
    bound = LOG_ATOL + LOG_RTOL * np.abs(expected32)
    if np.all(np.abs(ours - expected32) <= bound):
        return
    expected64 = reference_cpu(xe, program, [t.double() for t in inputs])
    reference_error = np.abs(expected32.astype(np.float64) - expected64)
    our_error = np.abs(ours.astype(np.float64) - expected64)
    assert np.all(our_error <= np.maximum(2.0 * reference_error, bound)), (our_error.max(), reference_error.max())


def _cases(xe):
    from extended_einsum.interface.tensor_expression import Parameter

    def matmul(t):  # the 1024^2 log(U(0,1)) matrices of the CPU-runnable configuration, seed 0
        a, b = t["a"], t["b"]
        return xe.log(xe.einsum("ik,kj->ij", xe.exp(xe.array(a)), xe.exp(xe.array(b))))

    def batched(t):
        return xe.log(xe.einsum("bik,bkj->bij", xe.exp(xe.array(t["a"])), xe.exp(xe.array(t["b"]))))

    def cp_layer(t):
        w = xe.softmax(Parameter(xe.array(t["w"])), axis=2)
        return xe.log(xe.einsum("dac,dbc->dab", xe.exp(xe.array(t["x"])), w))

    def tucker(t):
        w = xe.softmax(Parameter(xe.array(t["w"])), axis=(2, 3))
        return xe.log(xe.einsum("bfi,bfj,foij->bfo", xe.exp(xe.array(t["l"])), xe.exp(xe.array(t["r"])), w))

    def mixing(t):
        stacked = xe.stack([xe.exp(xe.array(c)) for c in (t["c0"], t["c1"], t["c2"])], axis=1)
        return xe.log(xe.einsum("bhu,uh->bu", stacked, xe.softmax(Parameter(xe.array(t["w"])), axis=1)))

    def softmax(t):
        return xe.softmax(xe.array(t["x"]), axis=1)

    g = torch.Generator().manual_seed(0)
    cases = {
        "matmul_1024": (matmul, {"a": torch.log(torch.rand(1024, 1024, generator=g)), "b": torch.log(torch.rand(1024, 1024, generator=g))}, True),
        "batched_n64": (batched, {"a": 8.0 * torch.randn(4, 96, 160, generator=g), "b": 8.0 * torch.randn(4, 160, 72, generator=g)}, True),
        "cp_layer": (cp_layer, {"x": torch.randn(8, 512, 64, generator=g) - 2.0, "w": torch.randn(8, 64, 64, generator=g)}, True),
        "tucker": (tucker, {"l": torch.randn(256, 8, 32, generator=g) - 3.0, "r": torch.randn(256, 8, 32, generator=g) - 3.0,
                            "w": torch.randn(8, 32, 32, 32, generator=g)}, True),
        "mixing": (mixing, {"c0": torch.randn(300, 64, generator=g) - 3.0, "c1": torch.randn(300, 64, generator=g) - 3.0,
                            "c2": torch.randn(300, 64, generator=g) - 3.0, "w": torch.randn(64, 3, generator=g)}, True),
        "softmax": (softmax, {"x": 2.0 * torch.randn(64, 3000, generator=g)}, False),
    }
    return cases


@pytest.fixture(scope="module")
def enabled(reference_xe):
    xb.enable()
    yield reference_xe
    xb.disable()


@pytest.mark.parametrize("mode", xb.STABLE_MODES)
@pytest.mark.parametrize("case", ["matmul_1024", "batched_n64", "cp_layer", "tucker", "mixing", "softmax"])
def test_reference_materialize_runs_on_b200(enabled, case, mode):
    xe = enabled
    build, tensors, log_domain = _cases(xe)[case]
    expr = build({k: v.to(DEVICE) for k, v in tensors.items()})
    result = expr.materialize(stability_mode=mode)
    # the reference's materialize was routed through lower(): our program, our kernels
    assert isinstance(expr._backend_program, xb.BackendProgram)
    out = result.backend_array
    assert out.is_cuda
    program, arguments = xe.extract_program(expr, mode)
    expected = reference_cpu(xe, program, [a.backend_array for a in arguments])
    if log_domain:
        log_close(out.cpu().numpy(), expected)
    else:
        np.testing.assert_allclose(out.cpu().numpy(), expected, rtol=2e-5, atol=1e-7)


def test_matmul_materialize_is_one_kernel_call(enabled):
    xe = enabled
    a = torch.log(torch.rand(256, 128, device=DEVICE))
    b = torch.log(torch.rand(128, 64, device=DEVICE))
    expr = xe.log(xe.einsum("ik,kj->ij", xe.exp(xe.array(a)), xe.exp(xe.array(b))))
    expr.materialize(stability_mode="logspace_max")
    assert len(expr._backend_program.backend_calls) == 1


@pytest.mark.parametrize("layer,shape", [("cp", (4, 4, 8, 40)), ("cp", (8, 8, 16, 300)), ("cp", (8, 8, 64, 1024)),
                                         ("tucker", (4, 4, 32, 40)), ("tucker", (8, 8, 32, 300))])
@pytest.mark.parametrize("mode", ["logspace_max", "logspace_min"])
def test_reference_folded_circuit_through_lower(reference_xe, layer, shape, mode):
    """The reference's folded circuit program (its own folding passes) lowered with the Hadamard
    products fused into the sum layers (CP) or the fused Tucker layers on the Tucker kernel in their
    fold-major form, against the reference's torch executor of that program."""
    from extended_einsum_b200.contraction import logspace_einsum, logspace_einsum_hadamard

    xe = reference_xe
    h, w, units, batch = shape
    program, data_input = demo_circuit_program(xe, h, w, units, batch, stability_mode=mode, layer=layer)
    inputs = demo_circuit_inputs(program, data_input, torch.Generator().manual_seed(h * w + units))
    lowered = xb.lower(program)
    fused_kind = logspace_einsum_hadamard if layer == "cp" else logspace_einsum
    fused = [c for c in lowered.backend_calls if getattr(getattr(c, "fn", None), "func", None) is fused_kind]
    assert len(fused) == int(np.log2(h * w))
    ours = xb.run_program(lowered, [t.to(DEVICE) for t in inputs]).cpu().numpy()
    assert ours.shape == (batch, 1)
    circuit_close(xe, program, inputs, ours)


def test_reference_circuit_materialize_unfolded(enabled):
    """materialize() of the demo's circuit expression before folding (one small einsum per region)."""
    xe = enabled
    from extended_einsum.interface.tensor_expression import Parameter

    g = torch.Generator().manual_seed(11)
    units, batch = 8, 32
    data = torch.softmax(torch.randn(16, batch, units, generator=g), dim=-1).to(DEVICE)
    array = xe.array(data)
    weights = []

    def sum_layer(child, outputs=units):
        logits = torch.randn(outputs, units, generator=g).to(DEVICE)
        weights.append(logits)
        return xe.einsum("ab,cb->ac", child, xe.softmax(Parameter(xe.array(logits)), axis=1))

    level = [sum_layer(xe.select(array, v)) for v in range(16)]
    while len(level) > 2:
        half = len(level) // 2
        level = [sum_layer(xe.einsum("ab,ab->ab", level[i], level[i + half])) for i in range(half)]
    expr = xe.log(sum_layer(xe.einsum("ab,ab->ab", level[0], level[1]), outputs=1))
    out = expr.materialize(stability_mode="logspace_max").backend_array
    program, arguments = xe.extract_program(expr, "logspace_max")
    circuit_close(xe, program, [a.backend_array for a in arguments], out.cpu().numpy())


@pytest.mark.parametrize("layer,units", [("cp", 16), ("tucker", 32)])
def test_reference_folded_circuit_gradients_through_lower(reference_xe, layer, units):
    """Gradients of the summed log-likelihood with respect to every input of the reference's folded
    circuit program (data and packed parameters) through the lowered program, against the
    reference's torch executor of the same program in fp64 (shifts detached as it detaches them)."""
    from extended_einsum.backend_translation.runtime import run_program as reference_run
    from extended_einsum.backend_translation.translate import translate_to_backend_program
    from extended_einsum.backends.torch import TorchBackendFunctions

    program, data_input = demo_circuit_program(reference_xe, 4, 4, units, 50, layer=layer)
    inputs = demo_circuit_inputs(program, data_input, torch.Generator().manual_seed(17))
    ours = [t.to(DEVICE).requires_grad_(True) for t in inputs]
    xb.run_program(xb.lower(program), ours).sum().backward()
    ref = [t.double().requires_grad_(True) for t in inputs]
    reference_run(translate_to_backend_program(program, TorchBackendFunctions()), ref).sum().backward()
    for mine, theirs in zip(ours, ref):
        expected = theirs.grad.numpy()
        scale = max(float(np.abs(expected).max()), 1.0)
        np.testing.assert_allclose(mine.grad.double().cpu().numpy(), expected, rtol=1e-4, atol=1e-5 * scale)
