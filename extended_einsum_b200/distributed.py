"""Multi-GPU execution of the hot path: one process per GPU, torch.distributed
over NCCL (gloo on CPU for the host-logic tests).

The path shards without any exchange inside the math:

* batched contractions and the folded circuit: every rank owns a contiguous
  slice of the batch (``shard_bounds``) and runs the same kernels on it;
  the circuit's per-sample log-likelihoods are gathered once at the end
  (``gather_rows``), the only collective of a forward pass;
* the large log-space matmul 'ik,kj->ij': A is row-sharded, B is broadcast
  once from its owner (``broadcast_operand``) and every rank computes the
  same column shifts of its full copy of B, so the shards of C are exactly
  the rows the unsharded contraction would produce; C is gathered only when
  the caller asks for the full result;
* softmax over rows: row-sharded, no communication.

Collectives are issued in the same order on every rank.  The kernels used
per rank are the single-GPU entry points (``ops``); ``RowShardedMatmul``
takes the contraction as a parameter so that the plumbing can be tested on
CPU ranks.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist


def world() -> tuple[int, int]:
    """(rank, world size) of the default process group, (0, 1) without one."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def shard_bounds(total: int, rank: int, world_size: int) -> tuple[int, int]:
    """Contiguous, balanced [lo, hi) slice of ``total`` items owned by ``rank``.

    The first ``total % world_size`` ranks own one item more; every item is
    owned by exactly one rank and the slices appear in rank order.
    """
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} is not in a world of {world_size}")
    if total < 0:
        raise ValueError("the number of items must be non-negative")
    base, extra = divmod(total, world_size)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def broadcast_operand(t: torch.Tensor | None, shape: tuple[int, ...], src: int = 0, group=None,
                      device: torch.device | None = None) -> torch.Tensor:
    """The operand ``t`` of rank ``src`` on every rank (ranks other than src pass None)."""
    rank, _ = world()
    if rank == src:
        if t is None or tuple(t.shape) != tuple(shape):
            raise ValueError(f"the source rank must pass the operand of shape {shape}")
        buf = t.contiguous()
    else:
        buf = torch.empty(shape, dtype=torch.float32, device=device)
    dist.broadcast(buf, src=src, group=group)
    return buf


def gather_rows(local: torch.Tensor, total_rows: int, group=None) -> torch.Tensor:
    """Concatenation over ranks (in rank order) of the row shards ``local``.

    Shards follow ``shard_bounds``; uneven shards are padded to the largest
    one for the collective and trimmed afterwards.
    """
    rank, world_size = world()
    lo, hi = shard_bounds(total_rows, rank, world_size)
    if local.shape[0] != hi - lo:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its shard is {hi - lo}")
    if world_size == 1:
        return local
    width = (total_rows + world_size - 1) // world_size
    padded = torch.zeros((width, *local.shape[1:]), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    out = torch.empty((world_size * width, *local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, padded, group=group)
    pieces = []
    for r in range(world_size):
        r_lo, r_hi = shard_bounds(total_rows, r, world_size)
        pieces.append(out[r * width : r * width + (r_hi - r_lo)])
    return torch.cat(pieces, dim=0)


def _gpu_logspace_matmul(a: torch.Tensor, b: torch.Tensor, shift: str) -> torch.Tensor:
    from . import ops

    return ops.logspace_gemm(a.unsqueeze(0), b.unsqueeze(0), shift=shift)[0]


class RowShardedMatmul:
    """log(exp(A) @ exp(B)) with A row-sharded over the ranks and B broadcast once.

    ``contract(a_rows, b, shift)`` computes one rank's rows (default: the
    sm_100a log-space contraction).  Each rank's rows depend only on its A
    rows and the full B, so the gathered result equals the unsharded one.
    """

    def __init__(self, shift: str = "max", group=None,
                 contract: Callable[[torch.Tensor, torch.Tensor, str], torch.Tensor] | None = None) -> None:
        self.shift = shift
        self.group = group
        self.contract = contract or _gpu_logspace_matmul
        self.b: torch.Tensor | None = None

    def set_b(self, b: torch.Tensor | None, shape: tuple[int, int], src: int = 0, device=None) -> None:
        """Broadcasts B (held by rank ``src``) to every rank; done once per operand."""
        self.b = broadcast_operand(b, shape, src=src, group=self.group, device=device)

    def __call__(self, a_rows: torch.Tensor, total_rows: int, gather: bool = False) -> torch.Tensor:
        if self.b is None:
            raise ValueError("set_b() must run before the contraction")
        rank, world_size = world()
        lo, hi = shard_bounds(total_rows, rank, world_size)
        if a_rows.shape[0] != hi - lo:
            raise ValueError(f"rank {rank} holds {a_rows.shape[0]} rows of A, its shard is {hi - lo}")
        c_rows = self.contract(a_rows, self.b, self.shift)
        return gather_rows(c_rows, total_rows, self.group) if gather else c_rows


def sharded_circuit_log_likelihood(forward: Callable[[torch.Tensor], torch.Tensor], pixels_local: torch.Tensor,
                                   total_batch: int, group=None) -> torch.Tensor:
    """Log-likelihoods (total_batch, 1) of a batch-sharded circuit: local forward + one gather."""
    return gather_rows(forward(pixels_local), total_batch, group)
