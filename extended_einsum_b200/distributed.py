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

import contextlib
import datetime
from collections.abc import Callable, Iterator

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
    rank, world_size = world()
    if world_size == 1:
        if t is None or tuple(t.shape) != tuple(shape):
            raise ValueError(f"the source rank must pass the operand of shape {shape}")
        return t.contiguous()
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


# ---------------------------------------------------------------------------
# failure detection between steps


def init_distributed(backend: str, timeout_s: float = 60.0, device: torch.device | None = None,
                     nonblocking: bool = True) -> None:
    """The default process group, with a short collective timeout.

    For NCCL the communicators are created non-blocking (ncclConfig.blocking = 0):
    their calls return at once and report errors asynchronously, so that a
    collective stuck on a dead peer can be aborted from the host
    (``abort_process_group``) instead of blocking the thread.  NVLS stays as the
    environment sets it (NCCL_NVLS_ENABLE).  Rendezvous through MASTER_ADDR /
    MASTER_PORT / RANK / WORLD_SIZE.
    """
    options = None
    if backend == "nccl" and nonblocking:
        from torch._C._distributed_c10d import ProcessGroupNCCL

        options = ProcessGroupNCCL.Options()
        options.config.blocking = 0
    kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None:
        kwargs["device_id"] = device
    if options is not None:
        kwargs["pg_options"] = options
    dist.init_process_group(backend, **kwargs)


def abort_process_group(group=None) -> None:
    """Ends the process group without waiting for peers: NCCL communicators are aborted
    (ncclCommAbort through ProcessGroupNCCL), other backends destroyed."""
    if not (dist.is_available() and dist.is_initialized()):
        return
    if dist.get_backend(group) == "nccl":
        from torch.distributed import distributed_c10d as c10d

        c10d._abort_process_group(group)
    else:
        dist.destroy_process_group(group)


class PeerFailure(RuntimeError):
    """Another rank reported a failure (or stopped answering) before this rank's next collective."""

    def __init__(self, rank: int, reason: str) -> None:
        super().__init__(f"rank {rank} failed: {reason}")
        self.rank = rank
        self.reason = reason


class PeerMonitor:
    """Host-side failure detection between steps, through the process group's store.

    A rank that fails inside ``guard()`` records the failure under its rank in
    the store before the exception propagates; every rank calls ``check()``
    before it launches the step's kernels and collectives, so the others learn
    of the failure on the host and leave between steps, with none of their
    kernels or collectives in flight.  A rank that dies without reporting is
    caught by the process group's timeout on the next collective instead.
    """

    def __init__(self, store=None, prefix: str = "xe-peer") -> None:
        if store is None:
            from torch.distributed import distributed_c10d as c10d

            store = c10d._get_default_store()
        self.store = store
        self.prefix = prefix
        self.rank, self.world_size = world()

    def _key(self, rank: int) -> str:
        return f"{self.prefix}/failed/{rank}"

    def report_failure(self, reason: str) -> None:
        self.store.set(self._key(self.rank), reason[:512])

    def check(self) -> None:
        """Raises PeerFailure for the first other rank that reported a failure."""
        for r in range(self.world_size):
            if r != self.rank and self.store.check([self._key(r)]):
                raise PeerFailure(r, self.store.get(self._key(r)).decode(errors="replace"))

    @contextlib.contextmanager
    def guard(self) -> Iterator[None]:
        """Reports any exception of the block to the peers, then re-raises it."""
        try:
            yield
        except BaseException as exc:
            self.report_failure(f"{type(exc).__name__}: {exc}")
            raise
