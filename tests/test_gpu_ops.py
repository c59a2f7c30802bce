"""Softmax, log-space elementwise kernels, reductions and the categorical
gather on the GPU against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import log_close
from extended_einsum_b200 import ops
from oracle import logspace as oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(
    "shape,axis",
    [((5, 37), 1), ((300, 1000), 1), ((7, 4096), 1), ((3, 20000), 1), ((2, 40000), 1), ((2, 70000), 1), ((4, 9, 5), 1),
     ((3, 5, 7), (1, 2)), ((2, 3, 4, 5), (1, 3)), ((64, 64, 64), 2), ((6, 128), 0), ((1, 1), 1), ((9, 33), -1),
     # rows of at most 64 (lane groups), and middle axes staged per slice in shared memory
     ((1000, 64), 1), ((50, 20), 1), ((7, 4), 1), ((300, 256, 64), 1), ((5, 256, 4), 1), ((3, 100, 8), 1),
     ((2, 96, 256), 1)],
)
def test_softmax(shape, axis):
    gen = torch.Generator().manual_seed(len(shape) * 100 + shape[0])
    x = 2.0 * torch.randn(*shape, generator=gen)
    y = ops.softmax(x.cuda(), axis).cpu().numpy()
    expected = oracle.softmax(x.double().numpy(), axis if isinstance(axis, int) else tuple(axis))
    np.testing.assert_allclose(y, expected, rtol=2e-6, atol=1e-9)
    logy = ops.softmax(x.cuda(), axis, log_output=True).cpu().numpy()
    log_close(logy, np.log(expected))


def test_softmax_wide_rows_configuration():
    """Row softmax at the width of the large configuration (32768 columns), a slab of rows."""
    gen = torch.Generator().manual_seed(4)
    x = 2.0 * torch.randn(64, 32768, generator=gen)
    y = ops.softmax(x.cuda(), 1).cpu().numpy()
    np.testing.assert_allclose(y, oracle.softmax(x.double().numpy(), 1), rtol=2e-6, atol=1e-12)
    np.testing.assert_allclose(y.sum(axis=1), 1.0, rtol=1e-5)


@pytest.mark.parametrize("rows,cols", [(300, 20000), (1000, 32768), (3, 16388)])
def test_prefetching_row_softmax_equals_register_softmax(rows, cols, monkeypatch):
    """Rows of 16K-32K columns take the kernel that streams the next row into shared memory;
    it runs the register-resident kernel's arithmetic, so both agree bit for bit, with -inf
    and NaN rows included."""
    gen = torch.Generator().manual_seed(rows + cols)
    x = 2.0 * torch.randn(rows, cols, generator=gen)
    x[1, :] = -float("inf")
    x[2, 7] = float("nan")
    x = x.cuda()
    for log_output in (False, True):
        monkeypatch.delenv("XE_SOFTMAX_NO_PREFETCH", raising=False)
        ours = ops.softmax(x, 1, log_output=log_output).cpu().numpy()
        monkeypatch.setenv("XE_SOFTMAX_NO_PREFETCH", "1")
        reg = ops.softmax(x, 1, log_output=log_output).cpu().numpy()
        assert np.array_equal(ours, reg, equal_nan=True)
    monkeypatch.delenv("XE_SOFTMAX_NO_PREFETCH", raising=False)
    assert ops.device_status() == 0


def test_log_add_broadcast_and_quotient():
    gen = torch.Generator().manual_seed(3)
    a = torch.randn(4, 1, 6, generator=gen)
    b = torch.randn(5, 1, generator=gen)
    y = ops.log_add(a.cuda(), b.cuda()).cpu().numpy()
    np.testing.assert_array_equal(y, (a + b).numpy())
    y = ops.log_add(a.cuda(), b.cuda(), negate_b=True).cpu().numpy()
    np.testing.assert_array_equal(y, (a - b).numpy())
    big = torch.randn(1000, 64, generator=gen)
    y = ops.log_add(big.cuda(), big.cuda()).cpu().numpy()
    np.testing.assert_array_equal(y, (big + big).numpy())


@pytest.mark.parametrize("subtract", [False, True])
@pytest.mark.parametrize("mode", ["max", "min"])
def test_log_add_exp(subtract, mode):
    gen = torch.Generator().manual_seed(5)
    a = torch.randn(3, 4, generator=gen) + 2.0
    b = torch.randn(3, 4, generator=gen) - 2.0
    y = ops.log_add_exp(a.cuda(), b.cuda(), subtract=subtract, shift=mode).cpu().numpy()
    expected = oracle.log_add_exp(a.double().numpy(), b.double().numpy(), subtract, mode)
    log_close(y, expected)


@pytest.mark.parametrize("shape,reduced", [((7, 300), (1,)), ((300, 7), (0,)), ((5, 6, 7), (0, 2)), ((3, 4), (0, 1))])
def test_logspace_reduce_via_einsum(shape, reduced):
    from extended_einsum_b200.contraction import logspace_einsum

    labels = "abc"[: len(shape)]
    out = "".join(l for i, l in enumerate(labels) if i not in reduced)
    gen = torch.Generator().manual_seed(6)
    x = 3.0 * torch.randn(*shape, generator=gen)
    y = logspace_einsum(f"{labels}->{out}", [False], "max", x.cuda()).cpu().numpy()
    expected = oracle.logspace_einsum(f"{labels}->{out}", [x.double().numpy()], [False])
    log_close(y, expected)


def test_unary_conversions():
    x = torch.rand(1001) + 0.01
    np.testing.assert_allclose(ops.log(x.cuda()).cpu().numpy(), np.log(x.double().numpy()), rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(ops.exp(x.cuda()).cpu().numpy(), np.exp(x.double().numpy()), rtol=1e-6)


def test_categorical_gather():
    gen = torch.Generator().manual_seed(8)
    table = torch.randn(6, 256, 12, generator=gen)
    pixels = torch.randint(256, (9, 10), generator=gen, dtype=torch.uint8)
    var = torch.tensor([3, 1, 0, 9, 4, 5], dtype=torch.int32)
    y = ops.categorical_gather(table.cuda(), pixels.cuda(), var.cuda()).cpu()
    expected = table[torch.arange(6)[:, None], pixels[:, var.long()].T.long()]
    assert torch.equal(y, expected)
    table = torch.randn(4, 16, 5, generator=gen)  # units not a multiple of 4: scalar path
    pixels = torch.randint(16, (3, 4), generator=gen, dtype=torch.uint8)
    y = ops.categorical_gather(table.cuda(), pixels.cuda()).cpu()
    assert torch.equal(y, table[torch.arange(4)[:, None], pixels.T.long()])


def test_cpu_tensors_are_rejected():
    with pytest.raises(ValueError, match="CUDA"):
        ops.logspace_gemm(torch.zeros(1, 2, 2), torch.zeros(1, 2, 2))


def test_no_device_wait_timed_out():
    assert ops.device_status() == 0


@pytest.mark.parametrize("shape", [(6, 256, 64), (40, 64)])
def test_softmax_minus_inf_and_nan_fibres(shape):
    """A fibre that is all -inf gives NaN and a NaN propagates through its fibre, as torch does."""
    gen = torch.Generator().manual_seed(17)
    x = 2.0 * torch.randn(*shape, generator=gen)
    if len(shape) == 3:
        x[0, :, 3] = -float("inf")
        x[1, 5, 9] = float("nan")
        axis = 1
    else:
        x[0, :] = -float("inf")
        x[1, 5] = float("nan")
        axis = 1
    for log_output in (False, True):
        ours = ops.softmax(x.cuda(), axis, log_output=log_output).cpu()
        ref = torch.log_softmax(x.double(), axis) if log_output else torch.softmax(x.double(), axis)
        assert torch.equal(torch.isnan(ours), torch.isnan(ref))
        ok = ~torch.isnan(ref)
        np.testing.assert_allclose(ours[ok].numpy(), ref[ok].numpy(), rtol=2e-6, atol=1e-6 if log_output else 1e-9)


@pytest.mark.parametrize("shape,axes", [((8192, 64), (0,)), ((1024, 256, 64), (1,)), ((300, 7), (0,)),
                                        ((5, 70, 3, 9), (1, 2)), ((64, 100), (0,)), ((3, 40, 300), (1,))])
@pytest.mark.parametrize("kind", ["sum", "max", "min"])
def test_reduce_leading_and_middle_axes(shape, axes, kind):
    """xe_reduce over a leading or middle block of axes (contiguous outputs: the column kernel when
    the reduced length reaches 64 and at most 256 outputs per entry) against torch fp64."""
    g = torch.Generator().manual_seed(len(shape) + sum(shape))
    x = torch.randn(*shape, generator=g)
    if kind == "max":
        x.view(-1)[17] = float("nan")
    y = ops.reduce(x.cuda(), axes, kind).cpu()
    xd = x.double()
    ref = xd.sum(dim=axes) if kind == "sum" else (xd.amax(dim=axes) if kind == "max" else xd.amin(dim=axes))
    if kind == "max":
        # a NaN input propagates to its output (the reference's torch max does the same)
        nan_out = torch.isnan(ref)
        assert torch.equal(torch.isnan(y), nan_out)
        y, ref = y[~nan_out], ref[~nan_out]
    np.testing.assert_allclose(y.double().numpy(), ref.numpy(), rtol=1e-5, atol=1e-4)
    assert ops.device_status() == 0
