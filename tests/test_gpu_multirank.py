"""Two ranks on two GPUs over NCCL (skipped with fewer GPUs).

* The row-sharded contraction: B broadcast from rank 0 over NCCL, each rank
  contracting its rows of A; the gathered rows equal the unsharded result bit
  for bit (every rank computes the same column shifts of its full B).
* Failure between steps: rank 1 fails before the step's collective and reports
  it through the store; rank 0 learns of it on the host before it launches the
  collective, and aborts its non-blocking NCCL communicator.  No GPU fault, no
  hang: the failure is a host exception, and neither rank has a kernel or a
  collective in flight when it leaves.  NVLS is off (NCCL_NVLS_ENABLE=0).
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs"),
]

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world_size: int, port: int, case: str, out_dir: str) -> None:
    sys.path.insert(0, str(REPO))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world_size),
                      NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from extended_einsum_b200 import distributed as xd
    from extended_einsum_b200 import ops

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    xd.init_distributed("nccl", timeout_s=60.0, device=device, nonblocking=True)
    aborted = False
    try:
        if case == "rowshard":
            m, k, n = 2048, 1024, 768
            g = torch.Generator(device=device).manual_seed(7)
            a = torch.log(torch.rand(m, k, device=device, generator=g))
            b = torch.log(torch.rand(k, n, device=device, generator=g))  # the same on both ranks (same seed)
            lo, hi = xd.shard_bounds(m, rank, world_size)
            mm = xd.RowShardedMatmul(shift="max")
            mm.set_b(b if rank == 0 else None, (k, n), device=device)
            full = mm(a[lo:hi].contiguous(), m, gather=True)
            if rank == 0:
                ref = ops.logspace_gemm(a.unsqueeze(0), b.unsqueeze(0))[0]
                same = bool(torch.equal(full, ref))
                (Path(out_dir) / "rowshard.txt").write_text(f"{same}|{(full - ref).abs().max().item()}")
        elif case == "peer_fails":
            monitor = xd.PeerMonitor()
            dist.barrier()
            if rank == 1:
                try:
                    with monitor.guard():
                        raise RuntimeError("rank 1 input check failed")
                except RuntimeError:
                    pass
                dist.barrier()
            else:
                dist.barrier()
                try:
                    monitor.check()
                    dist.all_reduce(torch.ones(8, device=device))
                    outcome = "no failure seen"
                except xd.PeerFailure as exc:
                    outcome = f"PeerFailure|{exc.rank}|{exc.reason}"
                (Path(out_dir) / "peer.txt").write_text(outcome)
            torch.cuda.synchronize()
            xd.abort_process_group()
            aborted = True
    finally:
        if not aborted and dist.is_initialized():
            dist.destroy_process_group()


def _spawn(case: str, tmp_path: Path) -> None:
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(2, _free_port(), case, str(tmp_path)), nprocs=2, start_method="spawn", join=True)


def test_row_sharded_contraction_over_nccl_is_the_unsharded_result(tmp_path):
    _spawn("rowshard", tmp_path)
    same, diff = (tmp_path / "rowshard.txt").read_text().split("|")
    assert same == "True", f"max difference {diff}"


def test_a_failed_rank_is_seen_before_the_collective_and_nccl_is_aborted(tmp_path):
    _spawn("peer_fails", tmp_path)
    outcome = (tmp_path / "peer.txt").read_text().split("|")
    assert outcome[0] == "PeerFailure" and outcome[1] == "1" and "input check failed" in outcome[2]
