"""Backward passes on the GPU against torch autograd of the same formulas in
fp64 (and, through materialize, against the reference's own gradients in the
golden fixtures).  Shifts are constants in both (stop_gradient in the
reference), so the gradients are those of the exact function."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import extended_einsum_b200 as xb
from conftest import build_program
from extended_einsum_b200 import ops

pytestmark = pytest.mark.gpu

GRAD_RTOL, GRAD_ATOL = 2e-5, 1e-6


def _close(ours: torch.Tensor, ref: torch.Tensor, rtol=GRAD_RTOL, atol=GRAD_ATOL):
    ref = ref.detach().double().cpu()
    scale = float(ref.abs().max())
    np.testing.assert_allclose(ours.detach().double().cpu().numpy(), ref.numpy(), rtol=rtol, atol=atol * max(scale, 1.0))


def _leaf(t: torch.Tensor, device="cpu") -> torch.Tensor:
    return t.detach().to(device).requires_grad_(True)


@pytest.mark.parametrize("linear", [(False, False), (False, True), (True, False)], ids=["log-log", "log-lin", "lin-log"])
@pytest.mark.parametrize("shift", ["max", "min"])
@pytest.mark.parametrize("addend", [False, True])
def test_logspace_gemm_backward(linear, shift, addend):
    if addend and linear[0]:
        pytest.skip("the fused addend belongs to a log-domain A")
    g = torch.Generator().manual_seed(7)
    batch, m, k, n = 2, 70, 96, 40
    a = torch.randn(batch, m, k, generator=g) * 3 if not linear[0] else torch.rand(batch, m, k, generator=g) + 0.05
    a2 = torch.randn(batch, m, k, generator=g) * 2 if addend else None
    b = torch.randn(batch, k, n, generator=g) * 3 if not linear[1] else torch.rand(batch, k, n, generator=g) + 0.05
    up = torch.randn(batch, m, n, generator=g)
    ad, bd = _leaf(a, "cuda"), _leaf(b, "cuda")
    a2d = _leaf(a2, "cuda") if addend else None
    c = ops.logspace_gemm(ad, bd, a2=a2d, a_linear=linear[0], b_linear=linear[1], shift=shift)
    (c * up.cuda()).sum().backward()
    ar, br = _leaf(a.double()), _leaf(b.double())
    a2r = _leaf(a2.double()) if addend else None
    la = torch.log(ar) if linear[0] else (ar + a2r if addend else ar)
    lb = torch.log(br) if linear[1] else br
    cr = torch.logsumexp(la[:, :, :, None] + lb[:, None, :, :], dim=2)
    (cr * up.double()).sum().backward()
    _close(ad.grad, ar.grad)
    _close(bd.grad, br.grad)
    if addend:
        _close(a2d.grad, a2r.grad)


@pytest.mark.parametrize("shape,axis,log_output", [((6, 50), 1, False), ((4, 7, 9), (1, 2), False), ((5, 40), 1, True), ((8, 6, 6), 2, False)])
def test_softmax_backward(shape, axis, log_output):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(shape, generator=g) * 2
    up = torch.randn(shape, generator=g)
    xd = _leaf(x, "cuda")
    (ops.softmax(xd, axis, log_output=log_output) * up.cuda()).sum().backward()
    xr = _leaf(x.double())
    axes = (axis,) if isinstance(axis, int) else axis
    lse = torch.logsumexp(xr, dim=axes, keepdim=True)
    yr = xr - lse if log_output else torch.exp(xr - lse)
    (yr * up.double()).sum().backward()
    _close(xd.grad, xr.grad)


def test_log_add_exp_log_backward():
    g = torch.Generator().manual_seed(5)
    a = torch.randn(6, 1, 8, generator=g)
    b = torch.randn(5, 8, generator=g)
    up = torch.randn(6, 5, 8, generator=g)
    ad, bd = _leaf(a, "cuda"), _leaf(b, "cuda")
    y = ops.log(ops.exp(ops.log_add(ad, bd, negate_b=True)))
    (y * up.cuda()).sum().backward()
    ar, br = _leaf(a.double()), _leaf(b.double())
    (torch.log(torch.exp(ar - br)) * up.double()).sum().backward()
    _close(ad.grad, ar.grad)
    _close(bd.grad, br.grad)


def test_logspace_reduce_backward():
    g = torch.Generator().manual_seed(8)
    x = torch.randn(3, 9, 20, generator=g) * 4
    up = torch.randn(3, 9, generator=g)
    xd = _leaf(x, "cuda")
    (ops.logspace_reduce(xd) * up.cuda()).sum().backward()
    xr = _leaf(x.double())
    (torch.logsumexp(xr, dim=2) * up.double()).sum().backward()
    _close(xd.grad, xr.grad)


def test_no_backward_is_loud():
    """The scaled modes' glue has no backward on this path."""
    a = torch.rand(2, 4, 8, device="cuda", requires_grad=True)
    with pytest.raises(NotImplementedError):
        ops.scaled_gemm(a, a.transpose(1, 2))


@pytest.mark.parametrize("shape", [(200, 3, 32, 32, 32), (50, 2, 8, 32, 5)], ids=["tucker-kernel", "general-kernel"])
@pytest.mark.parametrize("shift", ["max", "min"])
def test_logspace_tucker_backward(shape, shift):
    """y = log sum_ij exp(l_i + r_j) w_oij, with the shifts detached (translate.py:727-740)."""
    b, f, i, j, o = shape
    g = torch.Generator().manual_seed(9)
    left = torch.randn(b, f, i, generator=g) - 3.0
    right = torch.randn(b, f, j, generator=g) - 3.0
    w = torch.softmax(torch.randn(f, o, i * j, generator=g), dim=2).reshape(f, o, i, j)
    up = torch.randn(b, f, o, generator=g)
    ld, rd, wd = _leaf(left, "cuda"), _leaf(right, "cuda"), _leaf(w, "cuda")
    (ops.logspace_tucker(ld, rd, wd, shift=shift) * up.cuda()).sum().backward()
    lr, rr, wr = _leaf(left.double()), _leaf(right.double()), _leaf(w.double())
    yr = torch.logsumexp((lr[:, :, None, :, None] + rr[:, :, None, None, :] + torch.log(wr)[None]).flatten(3), dim=3)
    (yr * up.double()).sum().backward()
    _close(ld.grad, lr.grad)
    _close(rd.grad, rr.grad)
    _close(wd.grad, wr.grad)


@pytest.mark.parametrize("subtract", [False, True])
@pytest.mark.parametrize("shift", ["max", "min"])
def test_log_add_exp_backward(subtract, shift):
    """y = log(exp(a) +/- exp(b)) with a scalar shift m detached (translate.py:647-664, 774-789)."""
    g = torch.Generator().manual_seed(12)
    b = torch.randn(5, 8, generator=g)
    a = torch.randn(6, 1, 8, generator=g)
    if subtract:  # every broadcast pair with a > b, so that the difference is positive
        a = a.abs() + b.max() + 0.5
    up = torch.randn(6, 5, 8, generator=g)
    ad, bd = _leaf(a, "cuda"), _leaf(b, "cuda")
    (ops.log_add_exp(ad, bd, subtract=subtract, shift=shift) * up.cuda()).sum().backward()
    ar, br = _leaf(a.double()), _leaf(b.double())
    yr = torch.log(torch.exp(ar) - torch.exp(br)) if subtract else torch.logaddexp(ar, br)
    (yr * up.double()).sum().backward()
    _close(ad.grad, ar.grad)
    _close(bd.grad, br.grad)


def _gather_inputs(folds, states, units, batch, variables, seed):
    g = torch.Generator().manual_seed(seed)
    table = torch.log_softmax(torch.randn(folds, states, units, generator=g), dim=1)
    pixels = torch.randint(states, (batch, variables), generator=g, dtype=torch.uint8)
    var = torch.randperm(variables, generator=g)[:folds].to(torch.int32)
    return table, pixels, var


def _gather_ref(table, pixels, var):
    return table[torch.arange(table.shape[0])[:, None], pixels[:, var.long()].T.long()]


def test_categorical_gather_backward():
    table, pixels, var = _gather_inputs(6, 20, 16, 50, 8, 13)
    up = torch.randn(6, 50, 16)
    td = _leaf(table, "cuda")
    (ops.categorical_gather(td, pixels.cuda(), var.cuda()) * up.cuda()).sum().backward()
    tr = _leaf(table.double())
    (_gather_ref(tr, pixels, var) * up.double()).sum().backward()
    _close(td.grad, tr.grad)


@pytest.mark.parametrize("pair", [False, True], ids=["gather", "state-table-pair"])
@pytest.mark.parametrize("batch", [300, 1030])
def test_fused_gather_layer_backward(pair, batch):
    """The first circuit layers with the gather fused, against the gather, the Hadamard sum and
    the log-space contraction written out in fp64."""
    folds, states, units = 4, 32, 64
    table, pixels, var = _gather_inputs(2 * folds if pair else folds, states, units, batch, 16, 21 + pair)
    g = torch.Generator().manual_seed(3)
    w = torch.softmax(torch.randn(folds, units, units, generator=g), dim=2)  # (F, O, K)
    up = torch.randn(folds, batch, units, generator=g)
    td, wd = _leaf(table, "cuda"), _leaf(w, "cuda")
    fused = ops.logspace_gemm_gather_pair if pair else ops.logspace_gemm_gather
    (fused(td, pixels.cuda(), var.cuda(), wd.permute(0, 2, 1), b_linear=True) * up.cuda()).sum().backward()
    tr, wr = _leaf(table.double()), _leaf(w.double())
    rows = _gather_ref(tr, pixels, var)
    a = rows[:folds] + rows[folds:] if pair else rows
    yr = torch.logsumexp(a[:, :, None, :] + torch.log(wr)[:, None, :, :], dim=3)
    (yr * up.double()).sum().backward()
    _close(td.grad, tr.grad, rtol=5e-5, atol=2e-6)
    _close(wd.grad, wr.grad, rtol=5e-5, atol=2e-6)
    assert ops.device_status() == 0


@pytest.mark.parametrize("name", ["matmul_logu", "batched_n64", "cp_layer", "softmax_rows", "tucker", "tucker_two_levels",
                                  "mixing_layer", "agreement_add", "circuit_4x4"])
def test_materialize_gradients_match_reference(golden, golden_programs, name):
    spec = golden_programs[name]
    if f"{name}/logspace_max/grad0" not in golden:
        pytest.skip("no reference gradients recorded for this program")
    program = build_program(spec, "logspace_max")
    lowered = xb.lower(program)
    inputs = [_leaf(torch.from_numpy(golden[f"{name}/in{i}"]), "cuda") for i in range(spec["n_inputs"])]
    out = xb.run_program(lowered, inputs)
    weights = torch.from_numpy(golden[f"{name}/logspace_max/grad_weights"]).cuda()
    (out * weights).sum().backward()
    for i in range(spec["n_inputs"]):
        key = f"{name}/logspace_max/grad{i}"
        if key in golden:
            _close(inputs[i].grad, torch.from_numpy(golden[key]), rtol=5e-5, atol=5e-6)


def _torch_circuit_ll(cat_logits, pixels, var_of_fold, level_logits, root_logits):
    """The folded circuit in fp64 torch (the formulas of oracle/circuit.py), differentiable."""
    table = torch.log_softmax(cat_logits, dim=1)
    f_idx = torch.arange(table.shape[0])[:, None]
    x = table[f_idx, pixels[:, var_of_fold].T.long()]  # (F0, B, K)
    y = None
    for level, logits in enumerate(level_logits):
        logw = torch.log_softmax(logits, dim=2)  # (F, O, K)
        if level > 0:
            half = y.shape[0] // 2
            x = y[:half] + y[half:]
        y = torch.logsumexp(x[:, :, None, :] + logw[:, None, :, :], dim=3)  # (F, B, O)
    h = y[0] + y[1]
    logw_root = torch.log_softmax(root_logits, dim=1)  # (1, K)
    return torch.logsumexp(h[:, None, :] + logw_root[None, :, :], dim=2)  # (B, 1)


@pytest.mark.parametrize("batch_from", ["golden", "per-sample"])
def test_circuit_gradients(golden, golden_programs, batch_from):
    """Every parameter of the circuit, the categorical logits included, through the fused first
    layers (state table + gathered pairs for the golden batch; the fused per-sample gather for a
    batch below half the states)."""
    from extended_einsum_b200.circuit import CircuitForward, QuadTreeCircuit

    name = "circuit_4x4"
    spec = golden_programs[name]
    c = spec["circuit"]
    levels = len([i for i in spec["instructions"] if i[0] == "einsum" and i[1]["format_string"] == "dac,dbc->dab"])
    cat = torch.from_numpy(golden[f"{name}/categorical_logits"])
    lv = [torch.from_numpy(golden[f"{name}/in{1 + l}"]) for l in range(levels)]
    root = torch.from_numpy(golden[f"{name}/in{1 + levels}"])
    pixels = torch.from_numpy(golden[f"{name}/pixels"])
    if batch_from == "per-sample":
        pixels = pixels[:5]
    var = torch.from_numpy(golden[f"{name}/var_of_fold"])
    circuit = QuadTreeCircuit(c["height"], c["width"], c["units"], c["states"])
    assert circuit.uses_state_table(pixels.shape[0]) == (batch_from == "golden")
    cat_d = _leaf(cat, "cuda")
    lv_d = [_leaf(t, "cuda") for t in lv]
    root_d = _leaf(root, "cuda")
    forward = CircuitForward(circuit, {"categorical": cat_d, "levels": lv_d, "root": root_d, "var_of_fold": var.cuda()})
    forward(pixels.cuda()).sum().backward()
    cat_r = _leaf(cat.double())
    lv_r = [_leaf(t.double()) for t in lv]
    root_r = _leaf(root.double())
    _torch_circuit_ll(cat_r, pixels, var.long(), lv_r, root_r).sum().backward()
    _close(cat_d.grad, cat_r.grad, rtol=1e-4, atol=1e-5)
    for ours, ref in zip(lv_d, lv_r):
        _close(ours.grad, ref.grad, rtol=1e-4, atol=1e-5)
    _close(root_d.grad, root_r.grad, rtol=1e-4, atol=1e-5)
    assert ops.device_status() == 0
