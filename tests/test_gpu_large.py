"""The large configurations at full size (one GPU): the 32768^3 log-space
matmul with A row-sharded as over four ranks, and the 65536 x 32768 row
softmax.  Inputs are drawn by seeded CPU generators.  Full-size checks are
size-independent properties (shards reproduce the unsharded rows bit for bit;
softmax rows sum to one) plus sampled entries against the oracle in fp64
(oracle.logspace.logspace_matmul / softmax: a row's and a column's entries
need only that row of A and that column of B)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import log_close
from extended_einsum_b200 import ops
from extended_einsum_b200.distributed import shard_bounds
from oracle import logspace as oracle

pytestmark = pytest.mark.gpu

N = 32768


@pytest.fixture(scope="module")
def operands():
    g = torch.Generator().manual_seed(4)
    a = torch.log(torch.rand(N, N, generator=g)).cuda()
    b = torch.log(torch.rand(N, N, generator=g)).cuda()
    return a, b


def test_row_sharded_32768_cube_matches_unsharded_and_fp64(operands):
    a, b = operands
    full = ops.logspace_gemm(a.unsqueeze(0), b.unsqueeze(0))[0]
    world = 4
    for rank in range(world):
        lo, hi = shard_bounds(N, rank, world)
        shard = ops.logspace_gemm(a[lo:hi].unsqueeze(0), b.unsqueeze(0))[0]
        assert torch.equal(shard, full[lo:hi]), f"shard {rank} differs from the unsharded rows"
        del shard
    rows = torch.tensor([0, 1, 12345, N - 1], device="cuda")
    cols = torch.tensor([0, 7, 4096, 20000, N - 2, N - 1], device="cuda")
    expected = oracle.logspace_matmul(a[rows].double().cpu().numpy(), b[:, cols].double().cpu().numpy())
    log_close(full[rows][:, cols].cpu().numpy(), expected)
    assert ops.device_status() == 0


def test_row_softmax_65536_by_32768():
    g = torch.Generator().manual_seed(4)
    x = (2.0 * torch.randn(65536, 32768, generator=g)).cuda()
    y = ops.softmax(x, 1)
    sums = y.sum(dim=1, dtype=torch.float64)
    assert torch.all((sums - 1.0).abs() < 1e-5)
    rows = torch.tensor([0, 777, 65535], device="cuda")
    expected = oracle.softmax(x[rows].double().cpu().numpy(), 1)
    np.testing.assert_allclose(y[rows].double().cpu().numpy(), expected, rtol=2e-6, atol=1e-12)
