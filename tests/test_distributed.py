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

    timeout = 5 if case == "peer_vanishes" else 60
    dist.init_process_group("gloo", rank=rank, world_size=world_size, timeout=datetime.timedelta(seconds=timeout))
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
        elif case == "peer_raises":
            # rank 1 fails in its step before the collective; rank 0 learns of it through the
            # store before it launches the collective, instead of waiting in it
            monitor = xd.PeerMonitor()
            dist.barrier()
            if rank == 1:
                try:
                    with monitor.guard():
                        raise ValueError("bad input on rank 1")
                except ValueError:
                    pass
                dist.barrier()  # the report is in the store before rank 0 checks
            else:
                dist.barrier()
                try:
                    monitor.check()
                    dist.all_reduce(torch.ones(4))
                except xd.PeerFailure as exc:
                    (Path(out_dir) / "peer_failure.txt").write_text(f"{exc.rank}|{exc.reason}")
        elif case == "peer_vanishes":
            # rank 1 leaves between steps without a word; rank 0's next collective ends with an
            # error after the process group's short timeout instead of hanging
            dist.barrier()
            if rank == 0:
                import time

                t0 = time.monotonic()
                try:
                    dist.all_reduce(torch.ones(4))
                    outcome = "completed"
                except Exception as exc:  # noqa: BLE001 - gloo raises RuntimeError subclasses
                    outcome = type(exc).__name__
                (Path(out_dir) / "vanished.txt").write_text(f"{outcome}|{time.monotonic() - t0:.1f}")
            return  # no destroy: the peer is gone
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001 - a group whose peer left may not shut down cleanly
                pass


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


def test_a_rank_that_raises_is_reported_before_the_next_collective(tmp_path):
    _spawn("peer_raises", tmp_path)
    rank, reason = (tmp_path / "peer_failure.txt").read_text().split("|", 1)
    assert rank == "1" and "bad input on rank 1" in reason


def test_a_rank_that_vanishes_ends_the_next_collective_with_an_error(tmp_path):
    _spawn("peer_vanishes", tmp_path)
    outcome, seconds = (tmp_path / "vanished.txt").read_text().split("|")
    assert outcome != "completed"
    assert float(seconds) < 30.0


def test_init_distributed_builds_nonblocking_nccl_options(monkeypatch):
    """The NCCL options init_distributed passes (no GPU: the call to torch is intercepted)."""
    from extended_einsum_b200 import distributed as xd

    seen = {}
    monkeypatch.setattr(dist, "init_process_group", lambda backend, **kw: seen.update(backend=backend, **kw))
    xd.init_distributed("nccl", timeout_s=7.0)
    assert seen["backend"] == "nccl" and seen["pg_options"].config.blocking == 0
    assert seen["timeout"].total_seconds() == 7.0
    seen.clear()
    xd.init_distributed("gloo", timeout_s=3.0)
    assert "pg_options" not in seen
