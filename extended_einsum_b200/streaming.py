"""Materialization of batched expressions whose operands live in host memory.

A stable expression over operands that share a leading batch axis (the
batched contractions and the batch-sharded circuit layers of this path) is
independent per batch element.  ``materialize_streamed`` splits the batch into
chunks and overlaps, on three CUDA streams, the host-to-device copy of chunk
i + 1, the kernels of chunk i and the device-to-host copy of chunk i - 1, so
that the PCIe transfers, not their sum with the kernels, bound the call.  Each
distinct chunk shape is lowered once (``lowering.lower``); the kernels are the
same as for device-resident operands.

The host operands and the output should be pinned (``tensor.pin_memory()``) for
the copies to be asynchronous.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from typing import Any

import torch

from .frontend import extract_program, input_tensor
from .lowering import lower, run_program


_COPY_STREAMS: dict[int, tuple[torch.cuda.Stream, torch.cuda.Stream]] = {}


def _copy_streams(device: torch.device) -> tuple[torch.cuda.Stream, torch.cuda.Stream]:
    """The host-to-device and device-to-host copy streams of a device, created once."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    if index not in _COPY_STREAMS:
        _COPY_STREAMS[index] = (torch.cuda.Stream(index), torch.cuda.Stream(index))
    return _COPY_STREAMS[index]


def materialize_streamed(
    build: Callable[..., Any],
    host_operands: Sequence[torch.Tensor],
    out: torch.Tensor,
    stability_mode: str,
    chunks: int = 8,
    device: torch.device | None = None,
) -> torch.Tensor:
    """Writes build(*operands).materialize(stability_mode) into the host tensor ``out``.

    ``build`` maps device operands to an expression (e.g. ``lambda a, b:
    xe.log(xe.einsum('bik,bkj->bij', xe.exp(xe.array(a)), xe.exp(xe.array(b))))``).
    Every operand and the result have the batch as their leading axis, and
    the result of a batch slice is the same slice of the result.  Returns
    ``out`` after the last copy has completed.
    """
    if not host_operands:
        raise ValueError("materialize_streamed needs at least one operand")
    batch = host_operands[0].shape[0]
    if any(t.dim() == 0 or t.shape[0] != batch for t in host_operands) or out.shape[0] != batch:
        raise ValueError("every operand and the output must share the leading batch axis")
    if any(t.device.type != "cpu" for t in (*host_operands, out)):
        raise ValueError("materialize_streamed takes host operands and a host output")
    device = device or torch.device("cuda", torch.cuda.current_device())
    chunks = max(1, min(chunks, batch))
    bounds = [(batch * i // chunks, batch * (i + 1) // chunks) for i in range(chunks)]

    compute = torch.cuda.current_stream(device)
    copy_in, copy_out = _copy_streams(device)
    lowered: dict[tuple, tuple[Any, list[int]]] = {}
    # two device buffers per operand: chunk i + 1 is copied in while chunk i computes
    buffers = [[torch.empty((bounds[0][1] - bounds[0][0] + 1, *t.shape[1:]), dtype=t.dtype, device=device)
                for t in host_operands] for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    for e in in_free:
        e.record(compute)
    done = torch.cuda.Event()

    def stage(i: int) -> list[torch.Tensor]:
        lo, hi = bounds[i]
        slot = i % 2
        copy_in.wait_event(in_free[slot])
        views = []
        with torch.cuda.stream(copy_in):
            for buf, host in zip(buffers[slot], host_operands):
                view = buf[: hi - lo]
                view.copy_(host[lo:hi], non_blocking=True)
                views.append(view)
        in_ready[slot].record(copy_in)
        return views

    # Each chunk's result stays referenced here until the last copy has completed, so no block is
    # handed to another stream (record_stream would keep the caching allocator from reusing the
    # blocks of one call in the next, and it then allocates fresh ones for every chunk).
    results: list[torch.Tensor] = []
    pending = stage(0)
    for i, (lo, hi) in enumerate(bounds):
        views = pending
        if i + 1 < chunks:
            pending = stage(i + 1)
        compute.wait_event(in_ready[i % 2])
        key = tuple(tuple(v.shape) for v in views)
        if key not in lowered:
            program, arguments = extract_program(build(*views), stability_mode)
            order = []
            for argument in arguments:
                tensor = input_tensor(argument)
                order.append(next(j for j, v in enumerate(views) if v is tensor))
            lowered[key] = (lower(program), order)
        backend_program, order = lowered[key]
        result = run_program(backend_program, [views[j] for j in order])
        in_free[i % 2].record(compute)
        done.record(compute)
        copy_out.wait_event(done)
        results.append(result)
        with torch.cuda.stream(copy_out):
            out[lo:hi].copy_(result.reshape(out[lo:hi].shape), non_blocking=True)
    copy_out.synchronize()
    results.clear()
    return out
