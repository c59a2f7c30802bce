"""Host-side lowering (no GPU): program structure, error behaviour, and
agreement of the front end with the reference's IR where it is importable."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

import extended_einsum_b200 as xb
from conftest import build_program
from extended_einsum_b200 import frontend as fe
from extended_einsum_b200.circuit import QuadTreeCircuit, quad_tree_leaf_order


def _fns(program):
    return [getattr(call, "fn", call) for call in program.backend_calls]


def test_logspace_matmul_lowers_to_one_call():
    a = xb.array(torch.zeros(4, 3))
    b = xb.array(torch.zeros(3, 5))
    program, inputs = xb.extract_program(xb.log(xb.einsum("ik,kj->ij", xb.exp(a), xb.exp(b))), "logspace_max")
    lowered = xb.lower(program)
    # the reference's translation emits 16 calls for this expression (max, detach, subtract,
    # exp for each operand, einsum, log, and a reduce + reshape + add per shift)
    assert len(lowered.backend_calls) == 1
    assert lowered.call_arguments == [(0, 1)]


def test_exp_log_roundtrip_is_free():
    program = fe.dense_program([fe.RichInstruction(fe.OperatorExp(), (0,)), fe.RichInstruction(fe.OperatorLog(), (1,))], 1, "logspace_max")
    assert len(xb.lower(program).backend_calls) == 0


def test_softmax_parameters_stay_linear():
    instructions = [
        fe.RichInstruction(fe.OperatorSoftmax(axis=0), (1,)),
        fe.RichInstruction(fe.OperatorExp(), (0,)),
        fe.RichInstruction(fe.OperatorEinsum("bi, io -> bo"), (3, 2)),
        fe.RichInstruction(fe.OperatorLog(), (4,)),
    ]
    program = fe.dense_program(instructions, 2, "logspace_max", parameter_indices=frozenset({1}))
    lowered = xb.lower(program)
    # softmax + one fused einsum (the reference needs 10 calls)
    assert len(lowered.backend_calls) == 2
    einsum_call = lowered.backend_calls[1].fn
    assert einsum_call.args[1] == (False, True)  # data operand log-space, weights linear


def test_unsupported_mode_and_operator_raise_like_the_reference():
    program = fe.dense_program([fe.RichInstruction(fe.OperatorExp(), (0,))], 1, "unstable")
    with pytest.raises(NotImplementedError):
        xb.lower(program)

    class OperatorSin:
        name = "sin"

    program = fe.dense_program([fe.RichInstruction(OperatorSin(), (0,))], 1, "logspace_max")
    with pytest.raises(NotImplementedError, match="has no logspace backend translation"):
        xb.lower(program)


def test_run_program_checks_input_count():
    program = xb.BackendProgram([], [], 2)
    with pytest.raises(ValueError):
        xb.run_program(program, [torch.zeros(1)])


def test_circuit_program_lowering(golden_programs):
    from extended_einsum_b200.contraction import logspace_einsum_hadamard

    program = build_program(golden_programs["circuit_4x4"], "logspace_max")
    lowered = xb.lower(program)
    # one log of the raw categorical data input; level 0: softmax + CP einsum; each level >= 1:
    # softmax, 2 slice views and one CP einsum with the Hadamard product of the halves fused
    # as its addend; top: 2 select views, softmax and the root einsum with the root product
    # fused.  The reference's translation of the same program has 63 calls.
    levels = 4
    assert len(lowered.backend_calls) == 1 + 2 + 4 * (levels - 1) + 4
    names = [getattr(f, "func", f) for f in _fns(lowered)]
    assert names.count(xb.ops.log) == 1 and xb.ops.exp not in names
    assert xb.ops.log_add not in names
    assert names.count(logspace_einsum_hadamard) == levels  # levels 1..3 and the root


def test_hadamard_with_two_consumers_is_not_fused():
    """A product read twice is computed once (as the reference computes it) and not fused."""
    from extended_einsum_b200.contraction import log_broadcast_product, logspace_einsum_hadamard

    instructions = [
        fe.RichInstruction(fe.OperatorEinsum("ab,ab->ab"), (0, 1)),
        fe.RichInstruction(fe.OperatorEinsum("ab,cb->ac"), (3, 2)),
        fe.RichInstruction(fe.OperatorEinsum("ab,ac->bc"), (3, 4)),
    ]
    program = fe.dense_program(instructions, 3, "logspace_max")
    names = [getattr(f, "func", f) for f in _fns(xb.lower(program))]
    assert logspace_einsum_hadamard not in names and names.count(log_broadcast_product) == 1


def test_quad_tree_leaf_order_is_a_permutation():
    for h, w in ((2, 2), (4, 4), (8, 4), (32, 32)):
        order = quad_tree_leaf_order(h, w)
        assert sorted(order) == list(range(h * w))


def test_quad_tree_regions_are_rectangles():
    h = w = 8
    order = quad_tree_leaf_order(h, w)
    f = h * w
    regions = [{order[i]} for i in range(f)]
    while f > 1:
        f //= 2
        regions = [regions[i] | regions[i + f] for i in range(f)]
        for region in regions:
            rows = {v // w for v in region}
            cols = {v % w for v in region}
            assert len(rows) * len(cols) == len(region)


def test_circuit_cost_model():
    c = QuadTreeCircuit(32, 32, 64, 256)
    assert c.fold_counts == [1024 >> l for l in range(10)]
    assert c.flops_per_sample() == 2 * 64 * 64 * 2046 + 2 * 64
    assert c.hbm_bytes_per_sample() == 4 * 64 * (1024 + 3 * (512 + 256 + 128 + 64 + 32 + 16 + 8 + 4 + 2)) + 4 * (2 * 64 + 1) + 1024


def test_front_end_matches_reference_extract_program(reference_xe):
    ref = reference_xe
    from extended_einsum.interface.tensor_expression import Parameter as RefParameter

    x = torch.zeros(4, 6, 8)
    w = torch.zeros(4, 5, 8)
    ours, _ = xb.extract_program(xb.log(xb.einsum("dac,dbc->dab", xb.exp(xb.array(x)), xb.softmax(xb.Parameter(xb.array(w)), axis=2))), "logspace_max")
    theirs, _ = ref.extract_program(ref.log(ref.einsum("dac,dbc->dab", ref.exp(ref.array(x)), ref.softmax(RefParameter(ref.array(w)), axis=2))), "logspace_max")
    assert ours.n_inputs == theirs.n_inputs
    assert ours.parameter_indices == theirs.parameter_indices
    assert list(map(tuple, ours.shapes)) == list(map(tuple, theirs.shapes))
    assert [(i.operator.name, i.argument_ssa_ids) for i in ours.instructions] == [(i.operator.name, i.argument_ssa_ids) for i in theirs.instructions]
    # the lowering accepts the reference's own program object
    assert len(xb.lower(theirs).backend_calls) == len(xb.lower(ours).backend_calls) == 2


@pytest.mark.parametrize("mode", ["scaled_sum", "scaled_max", "scaled_min"])
def test_scaled_modes_lower_every_golden_program(golden_programs, mode):
    """The scaled lowering (translate.py:115-585) accepts every golden program; nothing runs."""
    for name, spec in golden_programs.items():
        lowered = xb.lower(build_program(spec, mode))
        assert lowered.n_inputs == spec["n_inputs"]
        assert len(lowered.backend_calls) == len(lowered.call_arguments)


@pytest.mark.parametrize("mode", ["scaled_sum", "scaled_max", "scaled_min"])
def test_scaled_log_matmul_is_one_fused_contraction(mode):
    """log(einsum(exp(A), exp(B))): the pairs of the exp results and of the product are never
    formed, the whole expression is one log-space contraction with the exp rule's shifts."""
    from extended_einsum_b200.contraction import scaled_log_einsum

    a = xb.array(torch.zeros(4, 3))
    b = xb.array(torch.zeros(3, 5))
    program, _ = xb.extract_program(xb.log(xb.einsum("ik,kj->ij", xb.exp(a), xb.exp(b))), mode)
    fns = _fns(xb.lower(program))
    assert len(fns) == 1 and getattr(fns[0], "func", None) is scaled_log_einsum


def test_scaled_matmul_without_log_uses_one_tensor_core_contraction():
    """Without the log the product's pair is the output: the pair-by-pair sequence, one contraction."""
    from extended_einsum_b200.contraction import linear_einsum

    a = xb.array(torch.zeros(4, 3))
    b = xb.array(torch.zeros(3, 5))
    program, _ = xb.extract_program(xb.einsum("ik,kj->ij", xb.exp(a), xb.exp(b)), "scaled_sum")
    fns = _fns(xb.lower(program))
    einsums = [f for f in fns if getattr(f, "func", None) is linear_einsum]
    assert len(einsums) == 1 and einsums[0].args == ("ik,kj->ij",)


def test_unknown_stability_mode_is_not_implemented():
    program = fe.dense_program([fe.RichInstruction(fe.OperatorExp(), (0,))], 1, "unstable")
    with pytest.raises(NotImplementedError):
        xb.lower(program)


@pytest.mark.parametrize("layer", ["cp", "tucker"])
def test_reference_folded_circuits_lower_without_generic_glue(reference_xe, layer):
    """The reference's own folded circuit programs (its folding passes) lower to one kernel call per
    layer: no log add for the Hadamard products, and the fused Tucker layers in their fold-major
    form ('acde,abd,abe->abc') and the root's form ('bcd,ac,ad->ab') on the Tucker kernel."""
    from extended_einsum_b200.circuit import demo_circuit_program
    from extended_einsum_b200.contraction import log_broadcast_product, logspace_einsum, logspace_einsum_hadamard

    program, data_input = demo_circuit_program(reference_xe, 8, 8, 32, 7, layer=layer)
    lowered = xb.lower(program)
    names = [getattr(f, "func", f) for f in _fns(lowered)]
    assert log_broadcast_product not in names and xb.ops.log_add not in names
    levels = 6
    if layer == "cp":
        assert names.count(logspace_einsum_hadamard) == levels
    else:
        formats = [f.args[0] for f in _fns(lowered) if getattr(f, "func", None) is logspace_einsum]
        assert len(formats) == levels
        assert all(f.replace(" ", "") in ("acde,abd,abe->abc", "bcd,ac,ad->ab") for f in formats), formats
