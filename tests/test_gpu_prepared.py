"""The prepared B operand (xe_logspace_b_prepare, xe_logspace_gemm_prepared).

The contraction with B prepared once (exp'd, split into TF32 hi / lo, laid out as
the kernel's shared-memory stages) computes the same values in the same order
as the in-kernel B transform, so every result must equal the
XE_GEMM_NO_PLANES=1 path bit for bit; one case per layout is also checked
against the oracle (fp64)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import log_close
from extended_einsum_b200 import _lib, ops
from oracle import logspace as oracle

pytestmark = pytest.mark.gpu

# (batch, m, n, k): tails in n and k, one and several 128-column tiles, many k-blocks
SHAPES = [(2, 300, 200, 160), (1, 257, 132, 100), (3, 256, 512, 512), (1, 130, 1000, 1028)]


def _same(x: torch.Tensor, y: torch.Tensor) -> bool:
    return bool(torch.equal(torch.nan_to_num(x, nan=123.0), torch.nan_to_num(y, nan=123.0)) and
                torch.equal(torch.isnan(x), torch.isnan(y)))


def _operands(shape, b_layout: str, linear: tuple[bool, bool], gen: torch.Generator):
    batch, m, n, k = shape
    a = (torch.rand(batch, m, k, generator=gen) + 0.05) if linear[0] else 4.0 * torch.randn(batch, m, k, generator=gen)
    b = (torch.rand(batch, k, n, generator=gen) + 0.05) if linear[1] else 4.0 * torch.randn(batch, k, n, generator=gen)
    bd = b.cuda() if b_layout == "n" else b.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    return a, b, a.cuda(), bd


def _uses_planes(m, n, k):
    lib = _lib.load()
    return lib.xe_logspace_gemm_workspace_size_prepared(1, m, n, k, 0, 0) > lib.xe_logspace_gemm_workspace_size(1, m, n, k, 0, 0)


def test_planes_follow_the_row_tile_threshold(monkeypatch):
    """xe_logspace_gemm prepares B by itself from 8 row tiles of A (1024 rows) up, or from 2 with
    XE_GEMM_PLANES=1, and never with XE_GEMM_NO_PLANES=1."""
    assert not _uses_planes(512, 512, 512) and _uses_planes(1024, 512, 512)
    monkeypatch.setenv("XE_GEMM_PLANES", "1")
    assert _uses_planes(256, 512, 512) and not _uses_planes(128, 512, 512)
    monkeypatch.setenv("XE_GEMM_NO_PLANES", "1")
    assert not _uses_planes(8192, 512, 512)


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{b}x{m}x{n}x{k}" for b, m, n, k in SHAPES])
@pytest.mark.parametrize("b_layout", ["n", "k"], ids=["B-n-contiguous", "B-k-contiguous"])
@pytest.mark.parametrize("linear", [(False, False), (False, True), (True, False)], ids=["log-log", "log-lin", "lin-log"])
@pytest.mark.parametrize("mode", ["max", "min"])
def test_prepared_b_is_bit_identical_to_the_in_kernel_transform(shape, b_layout, linear, mode, monkeypatch):
    batch, m, n, k = shape
    gen = torch.Generator().manual_seed(hash((shape, b_layout, linear, mode)) % 2**31)
    _, _, a, b = _operands(shape, b_layout, linear, gen)
    monkeypatch.setenv("XE_GEMM_NO_PLANES", "1")
    plain = ops.logspace_gemm(a, b, a_linear=linear[0], b_linear=linear[1], shift=mode)
    monkeypatch.setenv("XE_GEMM_NO_PLANES", "0")
    monkeypatch.setenv("XE_GEMM_PLANES", "1")
    assert _uses_planes(m, n, k)
    planes = ops.logspace_gemm(a, b, a_linear=linear[0], b_linear=linear[1], shift=mode)
    # the explicit two-call form: B prepared once, then contracted
    prep = ops.PreparedB(b, linear=linear[1], shift=mode)
    shift_a = None if linear[0] else ops.logspace_shift(a, shift=mode)
    explicit = ops.logspace_gemm_prepared(a, prep, shift_a)
    torch.cuda.synchronize()
    assert _same(plain, planes)
    assert _same(plain, explicit)


@pytest.mark.parametrize("b_layout", ["n", "k"])
def test_prepared_b_matches_oracle(b_layout, monkeypatch):
    monkeypatch.setenv("XE_GEMM_PLANES", "1")
    gen = torch.Generator().manual_seed(5)
    shape = (2, 300, 200, 160)
    a_h, b_h, a, b = _operands(shape, b_layout, (False, False), gen)
    out = ops.logspace_gemm(a, b)
    log_close(out.cpu().numpy(), oracle.logspace_matmul(a_h.double().numpy(), b_h.double().numpy()))


def test_prepared_b_fused_addend_and_minus_inf():
    """The folded Hadamard addend, a column of B that is all -inf (NaN, as the reference) and rows
    of A that are -inf at some k."""
    gen = torch.Generator().manual_seed(9)
    a = 2.0 * torch.randn(2, 260, 200, generator=gen)
    a2 = 2.0 * torch.randn(2, 260, 200, generator=gen)
    b = 2.0 * torch.randn(2, 200, 136, generator=gen)
    b[0, :, 7] = -float("inf")
    a[1, 3, :50] = -float("inf")
    ad, a2d, bd = a.cuda(), a2.cuda(), b.cuda()
    import os

    os.environ["XE_GEMM_NO_PLANES"] = "1"
    try:
        plain = ops.logspace_gemm(ad, bd, a2=a2d)
    finally:
        os.environ.pop("XE_GEMM_NO_PLANES")
    os.environ["XE_GEMM_PLANES"] = "1"
    try:
        planes = ops.logspace_gemm(ad, bd, a2=a2d)
    finally:
        os.environ.pop("XE_GEMM_PLANES")
    torch.cuda.synchronize()
    assert _same(plain, planes)
    assert torch.isnan(planes[0, :, 7]).all()
    expected = oracle.logspace_matmul((a + a2).double().numpy()[1], b.double().numpy()[1])
    log_close(planes[1].cpu().numpy(), expected)


def test_one_prepared_b_against_row_blocks_of_a():
    """A row-sharded contraction: B prepared once, each row block of A contracted with it; the
    blocks are the unsharded result's rows bit for bit."""
    gen = torch.Generator().manual_seed(13)
    a = torch.log(torch.rand(1, 1024, 768, generator=gen)).cuda()
    b = torch.log(torch.rand(1, 768, 640, generator=gen)).cuda()
    full = ops.logspace_gemm(a, b)
    prep = ops.PreparedB(b)
    for lo, hi in ((0, 384), (384, 1024)):
        block = a[:, lo:hi]
        part = ops.logspace_gemm_prepared(block, prep, ops.logspace_shift(block))
        assert _same(part, full[:, lo:hi])


def test_prepare_rejects_bad_arguments():
    lib = _lib.load()
    b = torch.zeros(1, 64, 130, device="cuda")  # n % 4 != 0 with n contiguous and k not contiguous
    buf = torch.empty(lib.xe_logspace_b_prepared_size(1, 130, 64), device="cuda", dtype=torch.uint8)
    sb = torch.empty(130, device="cuda")
    st = lib.xe_logspace_b_prepare(b.data_ptr(), b.stride(0), b.stride(1), b.stride(2), 0, 1, 130, 64, 0,
                                   buf.data_ptr(), buf.numel(), sb.data_ptr(), None)
    assert st == _lib.XE_ERR_NOT_SUPPORTED
    b = torch.zeros(1, 64, 128, device="cuda")
    st = lib.xe_logspace_b_prepare(b.data_ptr(), b.stride(0), b.stride(1), b.stride(2), 0, 1, 128, 64, 0,
                                   buf.data_ptr(), 1024, sb.data_ptr(), None)
    assert st == _lib.XE_ERR_INVALID_ARGUMENT and "needed" in _lib.last_error()
    assert ops.device_status() == 0
    # stages (batch x 128-column tiles x 32-k blocks of 32 KB) + the partial column extremes
    np.testing.assert_equal(lib.xe_logspace_b_prepared_size(2, 129, 33), 2 * 2 * 2 * 32768 + 2 * 256 * 4)
