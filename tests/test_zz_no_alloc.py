"""The allocation-free contraction entry point (xe_logspace_gemm_noalloc).

Some callers cannot allocate device memory (an embedding runtime that owns all
of it, code that must not synchronise or allocate inside a stream-ordered
region).  For them the library keeps the contraction's scratch, the per-row and
per-column shift vectors, in a static device array of fixed size.  This test
calls that entry point through the C ABI, twice in a row, and compares each
result with the allocating entry point's on the same inputs.  It lives in a
file of its own that is collected last.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import log_close
from extended_einsum_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _call_noalloc(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> int:
    batch, m, k = a.shape
    n = b.shape[2]
    return _lib.load().xe_logspace_gemm_noalloc(
        a.data_ptr(), None, a.stride(0), a.stride(1), a.stride(2), 0,
        b.data_ptr(), b.stride(0), b.stride(1), b.stride(2), 0,
        out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
        batch, m, n, k, _lib.XE_SHIFT_MAX, torch.cuda.current_stream().cuda_stream,
    )


def test_noalloc_matches_the_allocating_entry_point_on_two_calls():
    gen = torch.Generator().manual_seed(21)
    shapes = [(3, 200, 150, 300), (2, 96, 130, 64)]
    for batch, m, n, k in shapes:
        a = (2.0 * torch.randn(batch, m, k, generator=gen)).cuda()
        b = (2.0 * torch.randn(batch, k, n, generator=gen)).cuda()
        expected = ops.logspace_gemm(a, b).cpu().numpy()
        out = torch.full((batch, m, n), float("nan"), device="cuda")
        status = _call_noalloc(a, b, out)
        _lib.check(status, "xe_logspace_gemm_noalloc")
        torch.cuda.synchronize()
        log_close(out.cpu().numpy(), expected)
        assert np.isfinite(out.cpu().numpy()).all()


def test_noalloc_rejects_problems_above_the_static_scratch():
    a = torch.zeros(1, 4, 4, device="cuda")
    b = torch.zeros(1, 4, 4, device="cuda")
    out = torch.empty(1, 4, 4, device="cuda")
    lib = _lib.load()
    huge = 1 << 21  # batch * (m + n) floats beyond the 4 MiB array
    status = lib.xe_logspace_gemm_noalloc(
        a.data_ptr(), None, 0, 4, 1, 0, b.data_ptr(), 0, 4, 1, 0, out.data_ptr(), 0, 4, 1,
        huge, 1, 1, 4, _lib.XE_SHIFT_MAX, None,
    )
    assert status == _lib.XE_ERR_INVALID_ARGUMENT
    assert "static scratch" in _lib.last_error()
