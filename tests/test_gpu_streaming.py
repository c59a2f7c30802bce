"""Host-operand materialization: the chunked H2D / kernels / D2H pipeline gives
exactly the result of materializing the device-resident operands."""

from __future__ import annotations

import pytest
import torch

import extended_einsum_b200 as xb
from extended_einsum_b200.streaming import materialize_streamed


def _build(a, b):
    return xb.log(xb.einsum("bik,bkj->bij", xb.exp(xb.array(a)), xb.exp(xb.array(b))))


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["logspace_max", "scaled_sum"])
@pytest.mark.parametrize("batch,chunks", [(13, 4), (8, 8), (3, 8), (1, 1)])
def test_streamed_equals_device_materialize(mode, batch, chunks):
    g = torch.Generator().manual_seed(batch * 7 + chunks)
    a = (8.0 * torch.randn(batch, 70, 96, generator=g)).pin_memory()
    b = (8.0 * torch.randn(batch, 96, 130, generator=g)).pin_memory()
    out = torch.empty(batch, 70, 130).pin_memory()
    materialize_streamed(_build, [a, b], out, mode, chunks=chunks)
    expected = _build(a.cuda(), b.cuda()).materialize(mode).backend_array.cpu()
    assert torch.equal(out, expected)


def test_streamed_rejects_mismatched_batches():
    a = torch.zeros(4, 2, 3)
    b = torch.zeros(5, 3, 2)
    with pytest.raises(ValueError):
        materialize_streamed(_build, [a, b], torch.zeros(4, 2, 2), "logspace_max")
    with pytest.raises(ValueError):
        materialize_streamed(_build, [a, a], torch.zeros(3, 2, 2), "logspace_max")
