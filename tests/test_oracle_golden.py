"""The oracle against golden vectors of the reference (no GPU).

Pins oracle/ before it is trusted as the checker of the B200 path: every
golden program is re-run through the oracle's restatement of the log-space
translation and compared with the reference's own outputs.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import build_program, golden_inputs, log_close
from oracle import circuit as oracle_circuit
from oracle import logspace as oracle


def _cast(inputs, dtype):
    return [x.astype(dtype) if x.dtype.kind == "f" else x for x in inputs]


def test_golden_fixture_is_complete(golden, golden_programs):
    assert len(golden_programs) >= 30
    for name, spec in golden_programs.items():
        for mode in spec["modes"]:
            assert f"{name}/{mode}/f32" in golden
            assert f"{name}/{mode}/f64" in golden


@pytest.mark.parametrize("mode", ["logspace_max", "logspace_min"])
def test_oracle_matches_reference_fp64(golden, golden_programs, mode):
    """fp64 oracle == fp64 reference (numpy executor) to rounding."""
    for name, spec in golden_programs.items():
        program = build_program(spec, mode)
        out = oracle.run_logspace(program, _cast(golden_inputs(golden, name, spec), np.float64))
        np.testing.assert_allclose(out, golden[f"{name}/{mode}/f64"], rtol=1e-9, atol=1e-12, equal_nan=True, err_msg=name)


@pytest.mark.parametrize("mode", ["logspace_max", "logspace_min"])
def test_oracle_matches_reference_fp32(golden, golden_programs, mode):
    """fp32 oracle (numpy) vs fp32 reference (torch executor): same algorithm, different libm/BLAS."""
    for name, spec in golden_programs.items():
        if name.startswith("huge_chain") or name.startswith("agreement_normalized"):
            # raw outputs of 1e30-scale chains: compared relatively below
            continue
        program = build_program(spec, mode)
        out = oracle.run_logspace(program, _cast(golden_inputs(golden, name, spec), np.float32))
        ref = golden[f"{name}/{mode}/f32"]
        log_close(out, ref, atol=2e-5, rtol=1e-6)


def test_oracle_pattern_functions(golden, golden_programs):
    a, b = golden["matmul_logu/in0"].astype(np.float64), golden["matmul_logu/in1"].astype(np.float64)
    np.testing.assert_allclose(oracle.logspace_matmul(a, b), golden["matmul_logu/logspace_max/f64"], rtol=1e-12)
    np.testing.assert_allclose(oracle.logspace_matmul(a, b, "min"), golden["matmul_logu/logspace_min/f64"], rtol=1e-12)
    a, b = golden["batched_n64/in0"].astype(np.float64), golden["batched_n64/in1"].astype(np.float64)
    np.testing.assert_allclose(oracle.logspace_matmul(a, b), golden["batched_n64/logspace_max/f64"], rtol=1e-12)
    x, wl = golden["cp_layer/in0"].astype(np.float64), golden["cp_layer/in1"].astype(np.float64)
    w = oracle.softmax(wl, 2)
    np.testing.assert_allclose(oracle.logspace_cp_layer(x, w), golden["cp_layer/logspace_max/f64"], rtol=1e-12)
    l, r, wl = (golden[f"tucker/in{i}"].astype(np.float64) for i in range(3))
    w = oracle.softmax(wl, (2, 3))
    np.testing.assert_allclose(oracle.logspace_tucker(l, r, w), golden["tucker/logspace_max/f64"], rtol=1e-12)


@pytest.mark.parametrize("name", ["circuit_4x4", "circuit_8x8"])
def test_oracle_circuit_matches_reference(golden, golden_programs, name):
    spec = golden_programs[name]
    levels = len([i for i in spec["instructions"] if i[0] == "einsum" and i[1]["format_string"] == "dac,dbc->dab"])
    level_logits = [golden[f"{name}/in{1 + l}"].astype(np.float64) for l in range(levels)]
    root = golden[f"{name}/in{1 + levels}"].astype(np.float64)
    out = oracle_circuit.circuit_log_likelihood(
        golden[f"{name}/categorical_logits"].astype(np.float64),
        golden[f"{name}/pixels"],
        golden[f"{name}/var_of_fold"],
        level_logits,
        root,
    )
    # the reference's data input is the fp32 softmax (computed in torch, demo/cirkit.py:525-527);
    # the oracle recomputes it in fp64 from the logits, hence rtol 1e-7 instead of rounding level
    np.testing.assert_allclose(out, golden[f"{name}/logspace_max/f64"], rtol=1e-7)


def test_reference_known_answers_hold_in_golden(golden):
    """Closed forms asserted by the reference's own tests (test_backend_translation.py:516-536, 581-601)."""
    log_values = np.array([[0.0, -1.0], [-1000.0, -1001.0]])
    weights = np.array([[1.0, 2.0], [3.0, 4.0]])
    m = log_values.max(axis=1, keepdims=True)
    expected = m + np.log(np.exp(log_values - m) @ weights)
    np.testing.assert_allclose(golden["row_shift_minus1000/logspace_max/f64"], expected, rtol=1e-9)
    log_values = np.array([[0.0, -1000.0], [-1.0, -1001.0]])
    m = log_values.max(axis=0, keepdims=True)
    expected = m.T + np.log(np.einsum("ib,io->bo", np.exp(log_values - m), weights))
    np.testing.assert_allclose(golden["axis_reorder_minus1000/logspace_max/f64"], expected, rtol=1e-9)


@pytest.mark.parametrize("norm", ["sum", "max", "min"])
def test_scaled_oracle_pattern_functions(golden, norm):
    """oracle/scaled.py == the reference's fp64 scaled-mode outputs (translate.py:293-394, 436-449)."""
    from oracle import scaled as oracle_scaled

    mode = f"scaled_{norm}"
    f64 = lambda key: golden[key].astype(np.float64)  # noqa: E731
    np.testing.assert_allclose(
        oracle_scaled.scaled_matmul(f64("matmul_logu/in0"), f64("matmul_logu/in1"), norm), golden[f"matmul_logu/{mode}/f64"], rtol=1e-12
    )
    np.testing.assert_allclose(
        oracle_scaled.scaled_matmul(f64("batched_n64/in0"), f64("batched_n64/in1"), norm), golden[f"batched_n64/{mode}/f64"], rtol=1e-12
    )
    w = oracle.softmax(f64("cp_layer/in1"), 2)
    np.testing.assert_allclose(oracle_scaled.scaled_cp_layer(f64("cp_layer/in0"), w, norm), golden[f"cp_layer/{mode}/f64"], rtol=1e-12)
    w = oracle.softmax(f64("tucker/in2"), (2, 3))
    np.testing.assert_allclose(
        oracle_scaled.scaled_tucker(f64("tucker/in0"), f64("tucker/in1"), w, norm), golden[f"tucker/{mode}/f64"], rtol=1e-12
    )


def test_golden_records_every_stable_mode(golden_programs):
    """The reference accepts every golden program in all five stable modes."""
    for name, spec in golden_programs.items():
        assert set(spec["modes"]) == {"logspace_max", "logspace_min", "scaled_sum", "scaled_max", "scaled_min"}, name


def test_reference_gradients_are_the_exact_function_gradients(golden):
    """The recorded reference gradients (shifts detached, translate.py:727-740) equal the
    autograd gradients of the exact log-sum-exp function, so the GPU backward can be
    checked against either."""
    import torch

    a = torch.from_numpy(golden["matmul_logu/in0"].astype(np.float64)).requires_grad_(True)
    b = torch.from_numpy(golden["matmul_logu/in1"].astype(np.float64)).requires_grad_(True)
    w = torch.from_numpy(golden["matmul_logu/logspace_max/grad_weights"].astype(np.float64))
    (torch.logsumexp(a[:, :, None] + b[None, :, :], dim=1) * w).sum().backward()
    np.testing.assert_allclose(a.grad.numpy(), golden["matmul_logu/logspace_max/grad0"], rtol=1e-10, atol=1e-14)
    np.testing.assert_allclose(b.grad.numpy(), golden["matmul_logu/logspace_max/grad1"], rtol=1e-10, atol=1e-14)
