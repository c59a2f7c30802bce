"""Multi-rank host logic on CPU: world_size-2 gloo process groups.

The sharding plan, the broadcast of B, the gathers and the row-sharded
contraction run as real torch.distributed ranks; the per-rank contraction is
the oracle's (CPU), the GPU kernels being covered by the -m gpu tests.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from extended_einsum_b200.distributed import shard_bounds

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_contract(a_rows: torch.Tensor, b: torch.Tensor, shift: str) -> torch.Tensor:
    from oracle import logspace as oracle

    return torch.from_numpy(oracle.logspace_matmul(a_rows.double().numpy(), b.double().numpy(), shift))


def _worker(rank: int, world_size: int, port: int, case: str, out_dir: str) -> None:
    sys.path.insert(0, str(REPO))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world_size, timeout=datetime.timedelta(seconds=60))
    try:
        from extended_einsum_b200 import distributed as xd

        if case == "matmul":
            total, k, n = 37, 24, 19
            g = torch.Generator().manual_seed(11)
            a = torch.log(torch.rand(total, k, generator=g))
            b = torch.log(torch.rand(k, n, generator=g))
            lo, hi = xd.shard_bounds(total, rank, world_size)
            mm = xd.RowShardedMatmul(shift="max", contract=_oracle_contract)
            mm.set_b(b if rank == 0 else None, (k, n))
            full = mm(a[lo:hi], total, gather=True)
            torch.save(full, Path(out_dir) / f"matmul_{rank}.pt")
        elif case == "circuit":
            total = 29
            g = torch.Generator().manual_seed(5)
            pixels = torch.randint(256, (total, 6), generator=g, dtype=torch.uint8)
            lo, hi = xd.shard_bounds(total, rank, world_size)
            # a per-sample function stands in for the circuit forward: rows must come back in order
            forward = lambda p: p.float().sum(dim=1, keepdim=True)  # noqa: E731
            ll = xd.sharded_circuit_log_likelihood(forward, pixels[lo:hi], total)
            torch.save(ll, Path(out_dir) / f"circuit_{rank}.pt")
        elif case == "bad_shard":
            try:
                xd.gather_rows(torch.zeros(3, 2), 10)
            except ValueError:
                torch.save(torch.tensor([1]), Path(out_dir) / f"bad_{rank}.pt")
    finally:
        dist.destroy_process_group()


def _spawn(case: str, tmp_path: Path, world_size: int = 2) -> None:
    mp.start_processes(_worker, args=(world_size, _free_port(), case, str(tmp_path)), nprocs=world_size,
                       start_method="spawn", join=True)


@pytest.mark.parametrize("total,world_size", [(0, 2), (1, 2), (7, 2), (8, 4), (37, 3), (8192, 8), (5, 8)])
def test_shard_bounds_partition_the_items(total, world_size):
    bounds = [shard_bounds(total, r, world_size) for r in range(world_size)]
    assert bounds[0][0] == 0 and bounds[-1][1] == total
    for (lo, hi), (lo2, _) in zip(bounds, bounds[1:]):
        assert hi == lo2 and hi >= lo
    sizes = [hi - lo for lo, hi in bounds]
    assert max(sizes) - min(sizes) <= 1


def test_shard_bounds_rejects_bad_ranks():
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)
    with pytest.raises(ValueError):
        shard_bounds(-1, 0, 2)


def test_row_sharded_matmul_gathers_the_unsharded_result(tmp_path):
    _spawn("matmul", tmp_path)
    g = torch.Generator().manual_seed(11)
    a = torch.log(torch.rand(37, 24, generator=g))
    b = torch.log(torch.rand(24, 19, generator=g))
    expected = _oracle_contract(a, b, "max")
    for rank in range(2):
        full = torch.load(tmp_path / f"matmul_{rank}.pt")
        # fp64 BLAS may block a shard's rows differently from the whole: rounding-level differences
        np.testing.assert_allclose(full.numpy(), expected.numpy(), rtol=1e-14, atol=0)


def test_sharded_circuit_gather_keeps_sample_order(tmp_path):
    _spawn("circuit", tmp_path)
    g = torch.Generator().manual_seed(5)
    pixels = torch.randint(256, (29, 6), generator=g, dtype=torch.uint8)
    expected = pixels.float().sum(dim=1, keepdim=True)
    for rank in range(2):
        np.testing.assert_array_equal(torch.load(tmp_path / f"circuit_{rank}.pt").numpy(), expected.numpy())


def test_gather_rejects_a_shard_of_the_wrong_size(tmp_path):
    _spawn("bad_shard", tmp_path)
    assert (tmp_path / "bad_0.pt").exists() and (tmp_path / "bad_1.pt").exists()
