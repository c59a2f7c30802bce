"""The scaled stability modes on the GPU: the kernels one by one against numpy,
and the lowered hot-path patterns against oracle/scaled.py (pinned to the
reference's own outputs) at sizes beyond the golden fixtures.

Tolerances: log-domain results 1e-5 absolute (the fp32 log-domain bound of
the path); linear fp32 results relative to the fp64 value."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import extended_einsum_b200 as xb
from conftest import log_close
from extended_einsum_b200 import ops
from extended_einsum_b200.contraction import linear_einsum
from oracle import logspace as oracle_logspace
from oracle import scaled as oracle

pytestmark = pytest.mark.gpu


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


@pytest.mark.parametrize(
    "batch,m,n,k",
    [(1, 128, 128, 64), (3, 100, 70, 45), (2, 257, 129, 300), (1, 64, 32, 1), (5, 33, 200, 1000), (1, 512, 512, 4096)],
)
@pytest.mark.parametrize("layout", ["rowmajor", "transposed"])
def test_scaled_gemm_matches_fp64(batch, m, n, k, layout):
    g = _gen(batch * 1000 + m + n + k)
    a = torch.rand(batch, m, k, generator=g)
    b = torch.rand(batch, k, n, generator=g)
    if layout == "transposed":
        a_dev = a.transpose(1, 2).contiguous().cuda().transpose(1, 2)
        b_dev = b.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    else:
        a_dev, b_dev = a.cuda(), b.cuda()
    out = ops.scaled_gemm(a_dev, b_dev).cpu().double()
    expected = torch.bmm(a.double(), b.double())
    # all terms positive: the split-TF32 sum is fp32-accurate relative to the value
    np.testing.assert_allclose(out.numpy(), expected.numpy(), rtol=3e-6, atol=0)


def test_scaled_gemm_zero_k_is_zero():
    a = torch.rand(2, 3, 0, device="cuda")
    b = torch.rand(2, 0, 4, device="cuda")
    assert torch.equal(ops.scaled_gemm(a, b).cpu(), torch.zeros(2, 3, 4))


@pytest.mark.parametrize("kind", ["sum", "max", "min", "exp", "lse"])
@pytest.mark.parametrize("shape,permute", [((37,), None), ((6, 5, 70), None), ((9, 1500), None), ((8, 12, 3), (2, 0, 1)), ((), None)])
def test_fiber_normalize(kind, shape, permute):
    g = _gen(len(shape) * 7 + len(kind))
    x = torch.rand(shape, generator=g) + 0.05 if kind in ("sum", "max", "min") else 3.0 * torch.randn(shape, generator=g)
    x_dev = x.cuda()
    if permute is not None:
        x = x.permute(permute)
        x_dev = x_dev.permute(permute)
    n, s = ops.fiber_normalize(x_dev, kind)
    xd = x.double().numpy()
    if kind in ("sum", "max", "min"):
        t = {"sum": np.sum, "max": np.max, "min": np.min}[kind](xd, axis=-1, keepdims=True)
        en, es = xd / t, np.log(t)
    elif kind == "exp":
        es = np.max(xd, axis=-1, keepdims=True)
        en = np.exp(xd - es)
    else:
        m = np.max(xd, axis=-1, keepdims=True)
        es = m + np.log(np.sum(np.exp(xd - m), axis=-1, keepdims=True))
        en = np.exp(xd - es)
    if not shape:
        en, es = en.reshape(()), es.reshape(())
    assert tuple(n.shape) == tuple(x.shape) and tuple(s.shape) == es.shape
    np.testing.assert_allclose(n.cpu().numpy(), en, rtol=2e-6, atol=1e-30)
    np.testing.assert_allclose(s.cpu().numpy(), es, rtol=1e-6, atol=2e-6)


def test_fiber_normalize_non_finite_rows():
    x = torch.tensor([[-np.inf, -np.inf, -np.inf], [0.0, np.nan, 1.0], [0.0, -np.inf, 0.0]], device="cuda")
    n, s = ops.fiber_normalize(x, "exp")
    ref = torch.exp(x.cpu() - torch.amax(x.cpu(), dim=-1, keepdim=True))
    np.testing.assert_array_equal(torch.isnan(n).cpu().numpy(), torch.isnan(ref).numpy())
    assert s[0, 0].item() == -np.inf and np.isnan(s[1, 0].item()) and s[2, 0].item() == 0.0


@pytest.mark.parametrize("kind", ["sum", "max", "min"])
@pytest.mark.parametrize("shape,axes", [((5, 7, 9), (1,)), ((5, 7, 9), (0, 2)), ((300,), None), ((4, 1, 6), (1,))])
def test_reduce(kind, shape, axes):
    x = torch.randn(shape, generator=_gen(11))
    y = ops.reduce(x.cuda(), axes, kind, keepdims=True).cpu()
    dims = tuple(range(len(shape))) if axes is None else axes
    ref = {"sum": torch.sum, "max": torch.amax, "min": torch.amin}[kind](x.double(), dim=dims, keepdim=True)
    np.testing.assert_allclose(y.numpy(), ref.numpy(), rtol=1e-6, atol=1e-5)


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "max", "min", "mul_exp", "log_add", "rescale"])
@pytest.mark.parametrize("shapes", [((64,), (64,), (64,)), ((4, 5, 6), (4, 1, 6), (1, 5, 1)), ((3, 1), (1, 7), ()), ((), (), ())])
def test_elementwise_broadcast(op, shapes):
    g = _gen(sum(len(s) for s in shapes))
    a = torch.rand(shapes[0], generator=g) + 0.1
    b = torch.randn(shapes[1], generator=g)
    c = torch.randn(shapes[2], generator=g) if op == "rescale" else None
    y = ops.elementwise(op, a.cuda(), b.cuda(), c.cuda() if c is not None else None).cpu()
    ref = {
        "add": lambda: a + b, "sub": lambda: a - b, "mul": lambda: a * b, "div": lambda: a / b,
        "max": lambda: torch.maximum(a, b), "min": lambda: torch.minimum(a, b),
        "mul_exp": lambda: a * torch.exp(b), "log_add": lambda: torch.log(a) + b,
        "rescale": lambda: a * torch.exp(b - c),
    }[op]()
    if op in ("add", "sub", "mul", "div", "max", "min"):
        assert torch.equal(y, ref)  # correctly rounded fp32 ops: bit-exact
    else:
        np.testing.assert_allclose(y.numpy(), ref.numpy(), rtol=1e-6, atol=1e-6)


def test_elementwise_max_propagates_nan():
    a = torch.tensor([np.nan, 1.0, 2.0], device="cuda")
    b = torch.tensor([0.0, np.nan, 1.0], device="cuda")
    y = ops.elementwise("max", a, b).cpu()
    assert np.isnan(y[0]) and np.isnan(y[1]) and y[2] == 2.0


@pytest.mark.parametrize(
    "fmt,shapes",
    [
        ("ij->i", [(7, 9)]),
        ("ij->ji", [(7, 9)]),
        ("ijk->", [(3, 4, 5)]),
        ("ij,j->ij", [(6, 5), (5,)]),
        ("bi,bj->bij", [(4, 3), (4, 5)]),
        ("ik,kj->ij", [(33, 70), (70, 19)]),
        ("ki,kj->ji", [(40, 12), (40, 30)]),
        ("bik,bkj->bji", [(3, 20, 30), (3, 30, 10)]),
        ("ikp,kj->ij", [(12, 16, 3), (16, 9)]),
        ("dac,dbc->dab", [(4, 50, 16), (4, 16, 16)]),
        ("bfi,bfj,foij->bfo", [(6, 3, 32), (6, 3, 32), (3, 5, 32, 32)]),
    ],
)
def test_linear_einsum_matches_torch(fmt, shapes):
    g = _gen(len(fmt))
    operands = [torch.rand(s, generator=g) + 0.01 for s in shapes]
    out = linear_einsum(fmt, *[o.cuda() for o in operands]).cpu()
    ref = torch.einsum(fmt, *[o.double() for o in operands])
    assert out.shape == ref.shape
    np.testing.assert_allclose(out.numpy(), ref.numpy(), rtol=5e-6, atol=0)


def _lowered(expr, mode):
    return expr.materialize(mode).backend_array.cpu().numpy()


@pytest.mark.parametrize("norm", ["sum", "max", "min"])
@pytest.mark.parametrize("m,k,n", [(256, 384, 320), (1024, 1024, 1024)])
def test_scaled_matmul_against_oracle(norm, m, k, n):
    g = _gen(m + k + n)
    a = torch.log(torch.rand(m, k, generator=g))
    b = torch.log(torch.rand(k, n, generator=g))
    out = _lowered(xb.log(xb.einsum("ik,kj->ij", xb.exp(xb.array(a.cuda())), xb.exp(xb.array(b.cuda())))), f"scaled_{norm}")
    expected = oracle.scaled_matmul(a.double().numpy(), b.double().numpy(), norm)
    log_close(out, expected)


@pytest.mark.parametrize("norm", ["sum", "max"])
def test_scaled_batched_n64_against_oracle(norm):
    g = _gen(1)
    a = 8.0 * torch.randn(8, 128, 96, generator=g)
    b = 8.0 * torch.randn(8, 96, 200, generator=g)
    out = _lowered(xb.log(xb.einsum("bik,bkj->bij", xb.exp(xb.array(a.cuda())), xb.exp(xb.array(b.cuda())))), f"scaled_{norm}")
    log_close(out, oracle.scaled_matmul(a.double().numpy(), b.double().numpy(), norm))


@pytest.mark.parametrize("norm", ["sum", "min"])
def test_scaled_cp_layer_against_oracle(norm):
    g = _gen(3)
    x = torch.randn(16, 512, 64, generator=g) - 2.0
    w_logits = torch.randn(16, 64, 64, generator=g)
    expr = xb.log(xb.einsum("dac,dbc->dab", xb.exp(xb.array(x.cuda())), xb.softmax(xb.Parameter(xb.array(w_logits.cuda())), axis=2)))
    out = _lowered(expr, f"scaled_{norm}")
    w = oracle_logspace.softmax(w_logits.double().numpy(), 2)
    log_close(out, oracle.scaled_cp_layer(x.double().numpy(), w, norm))


def test_scaled_tucker_against_oracle():
    g = _gen(2)
    left = torch.randn(64, 8, 32, generator=g) - 3.0
    right = torch.randn(64, 8, 32, generator=g) - 3.0
    w_logits = torch.randn(8, 32, 32, 32, generator=g)
    expr = xb.log(
        xb.einsum(
            "bfi,bfj,foij->bfo",
            xb.exp(xb.array(left.cuda())),
            xb.exp(xb.array(right.cuda())),
            xb.softmax(xb.Parameter(xb.array(w_logits.cuda())), axis=(2, 3)),
        )
    )
    out = _lowered(expr, "scaled_sum")
    w = oracle_logspace.softmax(w_logits.double().numpy(), (2, 3))
    log_close(out, oracle.scaled_tucker(left.double().numpy(), right.double().numpy(), w, "sum"))
