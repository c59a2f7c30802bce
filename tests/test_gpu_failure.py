"""Failure detection on the GPU without a GPU fault: bounded device waits that
run out.  Every kernel wait is bounded; one that runs out records
(XE_ERR_DEVICE_TIMEOUT << 16) | site in the device status word, the CTA winds
down (waiting, with a fixed limit, for its own tensor-core work and bulk copies
still in flight, then freeing its TMEM) and the kernel returns, so the context
stays usable.

* xe_wait_probe waits on a barrier that nothing completes: the wait must run
  out after the configured limit, report its site, and leave the device clean
  for the next call.
* The production kernels (contraction, CP layer, Tucker layer, prefetching
  softmax) run under a 2 us limit, at which their ordinary waits run out at
  arbitrary points: each call must return, report either nothing or a timeout
  code, and the same call under the default limit must then give the results
  it gave before, bit for bit.
"""

from __future__ import annotations

import time

import pytest
import torch

from extended_einsum_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TIMEOUT_CODE = _lib.XE_ERR_DEVICE_TIMEOUT << 16
PROBE_SITE = 17


@pytest.fixture()
def default_limit_after():
    ops.device_status(clear=True)
    yield
    ops.set_wait_timeout_ns(0)
    ops.device_status(clear=True)


def _probe(complete: int) -> None:
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.load().xe_wait_probe(complete, stream), "xe_wait_probe")


def test_wait_that_nothing_completes_runs_out_and_reports_its_site(default_limit_after):
    ops.set_wait_timeout_ns(5_000_000)  # 5 ms
    t0 = time.perf_counter()
    _probe(0)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert ops.device_status(clear=True) == TIMEOUT_CODE | PROBE_SITE
    assert elapsed < 1.0  # the 5 ms limit, not the 2 s default
    # the status word was cleared, and the next launches run normally
    assert ops.device_status(clear=False) == 0
    _probe(1)
    torch.cuda.synchronize()
    assert ops.device_status(clear=True) == 0


def test_default_limit_is_restored(default_limit_after):
    ops.set_wait_timeout_ns(2_000_000)
    ops.set_wait_timeout_ns(0)
    _probe(1)
    torch.cuda.synchronize()
    assert ops.device_status() == 0


def _workloads():
    g = torch.Generator(device="cuda").manual_seed(5)
    a = 8.0 * torch.randn(8, 512, 512, device="cuda", generator=g)
    b = 8.0 * torch.randn(8, 512, 512, device="cuda", generator=g)
    x = torch.randn(64, 1024, 64, device="cuda", generator=g) - 2.0
    x2 = torch.randn(64, 1024, 64, device="cuda", generator=g) - 2.0
    w = ops.softmax(torch.randn(64, 64, 64, device="cuda", generator=g), 2).permute(0, 2, 1)
    left = torch.randn(512, 64, 32, device="cuda", generator=g) - 3.0
    right = torch.randn(512, 64, 32, device="cuda", generator=g) - 3.0
    tw = ops.softmax(torch.randn(64, 32, 32, 32, device="cuda", generator=g), (2, 3))
    s = 2.0 * torch.randn(296, 32768, device="cuda", generator=g)
    return {
        "contraction": lambda: ops.logspace_gemm(a, b),
        "cp_layer": lambda: ops.logspace_gemm(x, w, a2=x2, b_linear=True),
        "tucker_layer": lambda: ops.logspace_tucker(left, right, tw),
        "softmax_prefetch": lambda: ops.softmax(s, 1),
    }


@pytest.mark.parametrize("name", ["contraction", "cp_layer", "tucker_layer", "softmax_prefetch"])
def test_kernels_wind_down_when_their_waits_run_out(default_limit_after, name):
    run = _workloads()[name]
    expected = run()
    torch.cuda.synchronize()
    assert ops.device_status(clear=True) == 0
    ops.set_wait_timeout_ns(2_000)  # 2 us: ordinary waits run out at arbitrary points
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    status = ops.device_status(clear=True)
    assert status == 0 or status >> 16 == _lib.XE_ERR_DEVICE_TIMEOUT, hex(status)
    ops.set_wait_timeout_ns(0)
    again = run()
    torch.cuda.synchronize()
    assert ops.device_status(clear=True) == 0
    assert torch.equal(again, expected)
