"""The fused log-space Tucker layer 'bfi,bfj,foij->bfo' on the GPU against the
oracle (fp64), including the full configuration (b=512, f=2048, i=j=o=32)
checked on a sample of folds (folds are independent)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import log_close
from extended_einsum_b200 import ops
from oracle import logspace as oracle

pytestmark = pytest.mark.gpu


def _inputs(b, f, i, j, o, seed):
    gen = torch.Generator().manual_seed(seed)
    left = torch.randn(b, f, i, generator=gen) - 3.0
    right = torch.randn(b, f, j, generator=gen) - 3.0
    logits = torch.randn(f, o, i, j, generator=gen)
    w = torch.softmax(logits.reshape(f, o, i * j), dim=2).reshape(f, o, i, j)
    return left, right, w


@pytest.mark.parametrize("shape", [(20, 3, 32, 32, 8), (130, 5, 32, 32, 32), (64, 3, 16, 64, 20), (257, 2, 8, 32, 70), (1, 1, 32, 32, 1)])
@pytest.mark.parametrize("mode", ["max", "min"])
def test_tucker_matches_oracle(shape, mode):
    left, right, w = _inputs(*shape, seed=sum(shape))
    y = ops.logspace_tucker(left.cuda(), right.cuda(), w.cuda(), shift=mode).cpu().numpy()
    expected = oracle.logspace_tucker(left.double().numpy(), right.double().numpy(), w.double().numpy(), mode)
    log_close(y, expected)


def test_tucker_full_configuration_sample():
    torch.manual_seed(2)
    b, f, i, j, o = 512, 2048, 32, 32, 32
    left = torch.randn(b, f, i) - 3.0
    right = torch.randn(b, f, j) - 3.0
    w = torch.softmax(torch.randn(f, o, i * j), dim=2).reshape(f, o, i, j)
    y = ops.logspace_tucker(left.cuda(), right.cuda(), w.cuda()).cpu()
    assert torch.isfinite(y).all()
    sample = [0, 1, 777, 2047]
    expected = oracle.logspace_tucker(left[:, sample].double().numpy(), right[:, sample].double().numpy(), w[sample].double().numpy())
    log_close(y[:, sample].numpy(), expected)


def test_tucker_rejects_unsupported_shapes():
    left = torch.zeros(4, 2, 12, device="cuda")
    right = torch.zeros(4, 2, 48, device="cuda")
    w = torch.zeros(2, 3, 12, 48, device="cuda")
    with pytest.raises(NotImplementedError):
        ops.logspace_tucker(left, right, w)


def test_no_device_wait_timed_out():
    assert ops.device_status() == 0


@pytest.mark.parametrize("b,f,mode", [(300, 7, "max"), (128, 150, "min"), (1000, 3, "max")])
def test_tucker_layer_kernel_matches_general_kernel(b, f, mode, monkeypatch):
    """I = J = O = 32 runs the two-stage kernel (j contracted first on the tensor cores, i in
    the epilogue); the general kernel contracts (i, j) at once.  Both against each other
    and the oracle, with a row of -inf and rows past a 128-row tile."""
    left, right, w = _inputs(b, f, 32, 32, 32, seed=b + f)
    left[5, 1] = -float("inf")
    monkeypatch.delenv("XE_GEMM_NO_CP_LAYER", raising=False)
    ours = ops.logspace_tucker(left.cuda(), right.cuda(), w.cuda(), shift=mode).cpu().numpy()
    monkeypatch.setenv("XE_GEMM_NO_CP_LAYER", "1")
    general = ops.logspace_tucker(left.cuda(), right.cuda(), w.cuda(), shift=mode).cpu().numpy()
    with np.errstate(invalid="ignore", divide="ignore"):
        expected = oracle.logspace_tucker(left.double().numpy(), right.double().numpy(), w.double().numpy(), mode)
    log_close(ours, expected)
    log_close(ours, general)
    assert ops.device_status() == 0
