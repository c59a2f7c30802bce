"""The CP sum-layer kernel (K = N = 64, cp_layer.cuh) against the general
contraction kernel and the oracle: both kernels run the same arithmetic in the
same order, so their outputs are compared bit for bit; the oracle bounds both."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import log_close
from extended_einsum_b200 import ops
from oracle import logspace as oracle

pytestmark = pytest.mark.gpu


def _layer(folds, rows, pair, seed, minus_inf=False):
    g = torch.Generator().manual_seed(seed)
    y = 3.0 * torch.randn(2 * folds if pair else folds, rows, 64, generator=g) - 5.0
    if minus_inf:
        y[0, :7, :] = -float("inf")  # whole rows of the first fold
        y[-1, 3, 5] = -float("inf")
    w = torch.softmax(torch.randn(folds, 64, 64, generator=g), dim=2)
    return y.cuda(), w.cuda()


def _run(y, w, folds, pair, mode, monkeypatch, general):
    if general:
        monkeypatch.setenv("XE_GEMM_NO_CP_LAYER", "1")
    else:
        monkeypatch.delenv("XE_GEMM_NO_CP_LAYER", raising=False)
    b = w.permute(0, 2, 1)  # (F, K, N), k contiguous
    if pair:
        out = ops.logspace_gemm(y[:folds], b, a2=y[folds:], b_linear=True, shift=mode)
    else:
        out = ops.logspace_gemm(y, b, b_linear=True, shift=mode)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize(
    "folds,rows,pair,mode",
    [(1, 512, True, "max"), (3, 1000, True, "max"), (7, 513, False, "max"), (2, 600, True, "min"),
     (300, 512, True, "max"), (5, 777, False, "min"), (149, 520, False, "max")],
)
def test_cp_layer_equals_general_kernel(folds, rows, pair, mode, monkeypatch):
    y, w = _layer(folds, rows, pair, seed=folds * 31 + rows)
    ours = _run(y, w, folds, pair, mode, monkeypatch, general=False).cpu().numpy()
    general = _run(y, w, folds, pair, mode, monkeypatch, general=True).cpu().numpy()
    assert np.array_equal(ours, general, equal_nan=True)
    assert ops.device_status() == 0


def test_cp_layer_matches_oracle_with_minus_inf_rows(monkeypatch):
    folds, rows = 4, 700
    y, w = _layer(folds, rows, True, seed=5, minus_inf=True)
    ours = _run(y, w, folds, True, "max", monkeypatch, general=False).cpu().numpy()
    general = _run(y, w, folds, True, "max", monkeypatch, general=True).cpu().numpy()
    assert np.array_equal(ours, general, equal_nan=True)
    a = (y[:folds] + y[folds:]).cpu().double().numpy()
    b = w.permute(0, 2, 1).cpu().double().numpy()
    with np.errstate(invalid="ignore", divide="ignore"):
        ref = oracle.logspace_einsum("bmk,bkn->bmn", [a, b], [False, True], "max")
    log_close(ours, ref, atol=1e-5, rtol=1e-6)
    assert ops.device_status() == 0


def test_cp_layer_strided_output_falls_back(monkeypatch):
    """An output view whose rows are not 16-byte aligned takes the general kernel, same values."""
    folds, rows = 2, 600
    y, w = _layer(folds, rows, True, seed=9)
    b = w.permute(0, 2, 1)
    full = torch.empty(folds, rows, 65, device="cuda")
    out = full[:, :, :64]
    ops.logspace_gemm(y[:folds], b, a2=y[folds:], b_linear=True, out=out)
    ref = _run(y, w, folds, True, "max", monkeypatch, general=False)
    assert torch.equal(out, ref)


def _pair_inputs(folds, states, batch, seed):
    g = torch.Generator().manual_seed(seed)
    variables = 2 * folds + 3
    table = (torch.randn(2 * folds, states, 64, generator=g) - 4.0).cuda()
    pixels = torch.randint(states, (batch, variables), generator=g, dtype=torch.uint8).cuda()
    var = torch.randperm(variables, generator=g)[: 2 * folds].to(torch.int32).cuda()
    w = torch.softmax(torch.randn(folds, 64, 64, generator=g), dim=2).cuda()
    return table, pixels, var, w.permute(0, 2, 1)


@pytest.mark.parametrize(
    "folds,states,batch,mode",
    [(16, 256, 1000, "max"), (5, 7, 600, "max"), (300, 256, 512, "max"), (3, 100, 2049, "min"), (1, 256, 8192, "max")],
)
def test_slab_pair_layer_equals_general_kernel(folds, states, batch, mode, monkeypatch):
    """The state-table pair layer with the slabs in shared memory == the gathered general kernel, bit for bit."""
    table, pixels, var, b = _pair_inputs(folds, states, batch, seed=folds + states + batch)
    monkeypatch.delenv("XE_GEMM_NO_CP_LAYER", raising=False)
    ours = ops.logspace_gemm_gather_pair(table, pixels, var, b, b_linear=True, shift=mode).cpu().numpy()
    monkeypatch.setenv("XE_GEMM_NO_CP_LAYER", "1")
    general = ops.logspace_gemm_gather_pair(table, pixels, var, b, b_linear=True, shift=mode).cpu().numpy()
    assert np.array_equal(ours, general, equal_nan=True)
    assert ops.device_status() == 0


def test_slab_pair_layer_reports_out_of_range_pixels(monkeypatch):
    monkeypatch.delenv("XE_GEMM_NO_CP_LAYER", raising=False)
    table, pixels, var, b = _pair_inputs(4, 10, 600, seed=3)
    pixels[17, int(var[2])] = 250  # no such state
    assert ops.device_status() == 0
    ops.logspace_gemm_gather_pair(table, pixels, var, b, b_linear=True)
    status = ops.device_status(clear=True)
    assert status >> 16 == 1 and status & 0xFFFF == 33  # XE_ERR_INVALID_ARGUMENT, the gathered-row site
    assert ops.device_status() == 0
