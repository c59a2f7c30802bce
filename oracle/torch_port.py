"""The reference's CPU executor for the log-space path, as torch-CPU calls —
TEST AND BASELINE INFRASTRUCTURE ONLY (bench.py's CPU baseline and
``--impl reference`` arm time it on the host cores).

Each function issues the same torch calls, in the same order, that
TorchBackendFunctions (backends/torch.py:12-138) executes for the backend
program _append_logspace_einsum (backend_translation/translate.py:686-750)
emits: amax over the contracted axis, detach, subtract, exp per log operand,
einsum, log, and per shift an einsum reduction + reshape + add.
"""

from __future__ import annotations

import torch


def logspace_bmm(a: torch.Tensor, b: torch.Tensor, fmt: str = "bik,bkj->bij") -> torch.Tensor:
    """log(einsum(exp a, exp b)) in logspace_max for 'bik,bkj->bij' (16 backend calls in the reference)."""
    sa = torch.amax(a, dim=(2,), keepdim=True).detach()
    ea = torch.exp(a - sa)
    sb = torch.amax(b, dim=(1,), keepdim=True).detach()
    eb = torch.exp(b - sb)
    c = torch.log(torch.einsum(fmt, ea, eb))
    c = c + torch.reshape(torch.einsum("bik->bi", sa), (a.shape[0], a.shape[1], 1))
    c = c + torch.reshape(torch.einsum("bkj->bj", sb), (b.shape[0], 1, b.shape[2]))
    return c


def logspace_cp_layer(x: torch.Tensor, w_logits: torch.Tensor) -> torch.Tensor:
    """Folded CP sum layer 'dac,dbc->dab' with softmax(Parameter) weights (11 backend calls)."""
    w = torch.softmax(w_logits, dim=2)
    s = torch.amax(x, dim=(2,), keepdim=True).detach()
    c = torch.log(torch.einsum("dac,dbc->dab", torch.exp(x - s), w))
    return c + torch.reshape(torch.einsum("dac->da", s), (x.shape[0], x.shape[1], 1))


def circuit_log_likelihood(categorical_logits, pixels, var_of_fold, level_logits, root_logits) -> torch.Tensor:
    """The folded quad-tree circuit as the reference's torch executor runs it (demo/cirkit.py:428-446, 525-527)."""
    probs = torch.softmax(categorical_logits, dim=1)
    f_idx = torch.arange(probs.shape[0])[:, None]
    x = torch.log(probs[f_idx, pixels[:, var_of_fold.long()].T.long()])
    y = None
    for level, logits in enumerate(level_logits):
        if level > 0:
            half = y.shape[0] // 2
            x = y[:half] + y[half:]
        y = logspace_cp_layer(x, logits)
    h = y[0] + y[1]
    w = torch.softmax(root_logits, dim=1)
    s = torch.amax(h, dim=(1,), keepdim=True).detach()
    return torch.log(torch.einsum("ab,cb->ac", torch.exp(h - s), w)) + s
