"""xe_logspace_gemm against the oracle (fp64) on the GPU: every staging layout,
ragged extents, linear operands, both shift modes, the fused log-space
addend, every tile width, and the full-size batched configuration."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import log_close
from extended_einsum_b200 import ops
from oracle import logspace as oracle

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1, 1, 1), (1, 5, 7, 3), (2, 130, 70, 33), (1, 128, 256, 64), (3, 200, 300, 100), (1, 64, 513, 96), (2, 257, 129, 257)]
LAYOUTS = [("k", "mn"), ("k", "k"), ("mn", "mn"), ("mn", "k")]


def _operand(rows: int, cols: int, batch: int, layout: str, linear: bool, gen: torch.Generator, contiguous_dim: str):
    """(batch, rows, cols) fp32 on the GPU; `layout` 'k' = cols contiguous... see callers."""
    if linear:
        values = torch.rand(batch, rows, cols, generator=gen) + 0.05
    else:
        values = 2.0 * torch.randn(batch, rows, cols, generator=gen)
    if layout == contiguous_dim:
        dev = values.cuda()
    else:
        dev = values.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    return values.double().numpy(), dev


def _expected(a64, b64, a_lin, b_lin, mode):
    return oracle.logspace_einsum("bmk,bkn->bmn", [a64, b64], [a_lin, b_lin], mode)


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{b}x{m}x{n}x{k}" for b, m, n, k in SHAPES])
@pytest.mark.parametrize("layout", LAYOUTS, ids=[f"A{a}-B{b}" for a, b in LAYOUTS])
@pytest.mark.parametrize("linear", [(False, False), (False, True), (True, False)], ids=["log-log", "log-lin", "lin-log"])
@pytest.mark.parametrize("mode", ["max", "min"])
@pytest.mark.parametrize("tma", ["1", "0"], ids=["tma", "ldg"])
def test_gemm_matches_oracle(shape, layout, linear, mode, tma, monkeypatch):
    # A rows come from a TMA-filled staging ring when A is k-contiguous; the
    # global-load path is forced here for the other half of the sweep
    monkeypatch.setenv("XE_GEMM_NO_TMA", "0" if tma == "1" else "1")
    batch, m, n, k = shape
    gen = torch.Generator().manual_seed(hash((shape, layout, linear, mode)) % 2**31)
    # A is (batch, M, K): layout 'k' -> k contiguous, 'mn' -> m contiguous
    a64, a = _operand(m, k, batch, layout[0], linear[0], gen, contiguous_dim="k")
    # B is (batch, K, N): layout 'mn' -> n contiguous, 'k' -> k contiguous
    b64, b = _operand(k, n, batch, layout[1], linear[1], gen, contiguous_dim="mn")
    if layout[0] == "mn":
        assert a.stride(1) == 1
    if layout[1] == "k":
        assert b.stride(1) == 1
    out = ops.logspace_gemm(a, b, a_linear=linear[0], b_linear=linear[1], shift=mode)
    torch.cuda.synchronize()
    log_close(out.cpu().numpy(), _expected(a64, b64, *linear, mode))


@pytest.mark.parametrize("bn", ["32", "64", "128"])
def test_gemm_tile_widths(bn, monkeypatch):
    monkeypatch.setenv("XE_GEMM_BN", bn)
    gen = torch.Generator().manual_seed(7)
    a = 3.0 * torch.randn(2, 300, 200, generator=gen)
    b = 3.0 * torch.randn(2, 200, 333, generator=gen)
    out = ops.logspace_gemm(a.cuda(), b.cuda())
    log_close(out.cpu().numpy(), oracle.logspace_matmul(a.double().numpy(), b.double().numpy()))


def test_gemm_fused_addend_and_unaligned_operands():
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(3, 2, 77, 45, generator=gen) - 1.0  # two halves of a folded level
    w = torch.rand(3, 45, 19, generator=gen) + 0.1
    xd = x.cuda()
    left, right = xd[:, 0], xd[:, 1]
    out = ops.logspace_gemm(left, w.cuda(), a2=right, b_linear=True)
    expected = oracle.logspace_einsum("bmk,bkn->bmn", [(x[:, 0] + x[:, 1]).double().numpy(), w.double().numpy()], [False, True])
    log_close(out.cpu().numpy(), expected)
    # an operand that starts one element past a 16-byte boundary takes the scalar path
    flat = torch.randn(1 + 2 * 64 * 48, generator=gen)
    a = flat[1:].view(2, 64, 48)
    b = torch.randn(2, 48, 40, generator=gen)
    out = ops.logspace_gemm(flat.cuda()[1:].view(2, 64, 48), b.cuda())
    log_close(out.cpu().numpy(), oracle.logspace_matmul(a.double().numpy(), b.double().numpy()))


def test_gemm_strided_output_and_broadcast_batch():
    gen = torch.Generator().manual_seed(12)
    a = torch.randn(4, 70, 50, generator=gen)
    b = torch.randn(1, 50, 60, generator=gen)
    out_full = torch.full((4, 60, 70), float("nan"), device="cuda")
    out = out_full.transpose(1, 2)  # (4, 70, 60) with n-stride 70
    ops.logspace_gemm(a.cuda(), b.cuda().expand(4, 50, 60), out=out)
    expected = oracle.logspace_matmul(a.double().numpy(), np.broadcast_to(b.double().numpy(), (4, 50, 60)))
    log_close(out.cpu().numpy(), expected)


def test_gemm_minus_inf_rows_and_underflow():
    """-inf entries contribute 0; an all -inf row gives NaN (as torch: -inf - (-inf)); like the reference."""
    a = torch.randn(1, 40, 64)
    a[0, 3, :] = float("-inf")
    a[0, 5, 10:] = float("-inf")
    a[0, 7, :] = -1000.0
    b = torch.randn(1, 64, 48)
    out = ops.logspace_gemm(a.cuda(), b.cuda()).cpu().numpy()
    with np.errstate(invalid="ignore"):
        expected = oracle.logspace_matmul(a.double().numpy(), b.double().numpy())
    assert np.isnan(out[0, 3]).all() and np.isnan(expected[0, 3]).all()
    log_close(np.delete(out, 3, axis=1), np.delete(expected, 3, axis=1), rtol=1e-6)


@pytest.mark.parametrize("seed,scale,k", [(0, None, 1024), (1, 8.0, 512)], ids=["logU-1024cube", "N64-batched"])
def test_gemm_benchmark_configurations(seed, scale, k):
    """The log-space matmul configurations at full size (1024^3 and 128 x 512^3), checked
    against the fp64 oracle on every row of a sample of batches."""
    torch.manual_seed(seed)
    if scale is None:
        a = torch.log(torch.rand(1, 1024, 1024))
        b = torch.log(torch.rand(1, 1024, 1024))
    else:
        a = scale * torch.randn(128, 512, 512)
        b = scale * torch.randn(128, 512, 512)
    out = ops.logspace_gemm(a.cuda(), b.cuda()).cpu()
    sample = [0] if a.shape[0] == 1 else [0, 1, 63, 127]
    expected = oracle.logspace_matmul(a[sample].double().numpy(), b[sample].double().numpy())
    assert torch.isfinite(out).all()
    log_close(out[sample].numpy(), expected)


def test_no_device_wait_timed_out():
    assert ops.device_status() == 0


@pytest.mark.parametrize("k", [4096, 32768])
def test_gemm_long_contraction_has_no_accumulation_bias(k):
    """The tensor core accumulates with truncation; the chunked accumulation keeps the
    error at the level of a single chunk for any K (the mean error would otherwise grow
    linearly with K, to ~-2.4e-4 at K = 32768)."""
    gen = torch.Generator().manual_seed(k)
    a = 0.5 * torch.randn(1, 128, k, generator=gen)
    b = 0.5 * torch.randn(1, k, 96, generator=gen)
    out = ops.logspace_gemm(a.cuda(), b.cuda()).cpu().double().numpy()
    expected = oracle.logspace_matmul(a.double().numpy(), b.double().numpy())
    err = out - expected
    assert abs(err.mean()) < 2e-6, err.mean()
    log_close(out, expected)


@pytest.mark.parametrize("shape", [(1, 4096, 4096, 2048), (64, 512, 64, 64)], ids=["4096x4096x2048", "cp-layer"])
def test_gemm_is_deterministic(shape):
    """Repeated launches give bit-identical results (every TMEM access is warp-converged)."""
    batch, m, n, k = shape
    g = torch.Generator().manual_seed(9)
    a = torch.log(torch.rand(batch, m, k, generator=g)).cuda()
    b = torch.log(torch.rand(batch, k, n, generator=g)).cuda()
    first = ops.logspace_gemm(a, b)
    for _ in range(4):
        assert torch.equal(ops.logspace_gemm(a, b), first)
