"""CPU oracle for the scaled stability modes (scaled_sum / scaled_max /
scaled_min): numpy restatements of what extended_einsum's scaled translation
computes for the hot-path patterns.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (the extended_einsum_b200
package) imports this module; tests/ use it as the checker at sizes beyond
the golden fixtures.

Parity is pinned: tests/test_oracle_golden.py checks each function against
the golden vectors of the reference's own runs (tests/golden/make_golden.py),
in fp64 to rounding.

The representation (backend_translation/translate.py:119-126): a value is
n * exp(s) with one log scale s per last-axis fibre.  The steps below follow
the backend calls of the reference for an expression
log(einsum(fmt, exp(A), exp(B))) with optional linear (parameter-derived)
operands, in order:

  exp(X)           s = max over the last axis (keepdims), n = exp(X - s)      translate.py:436-444
  einsum operand   if s varies along a contracted axis: c = max of s over the
                   contracted axes (keepdims), n = n * exp(s - c); else c = s  translate.py:323-342
  einsum           raw = einsum(fmt, n_A, n_B); t = norm of raw over its last
                   axis (keepdims); n = raw / t; s = log(t) + each operand's c
                   summed over its dropped (size-1) labels and reshaped onto
                   the output labels                                          translate.py:372-394
  log(n * e^s)     log(n) + s                                                 translate.py:445-449
"""

from __future__ import annotations

import numpy as np

from .logspace import parse_format_string

NORMS = {"sum": np.sum, "max": np.max, "min": np.min}


def _exp_pair(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    s = np.max(x, axis=-1, keepdims=True)
    return np.exp(x - s), s


def _contraction_scale(n: np.ndarray, s: np.ndarray, labels: str, output: str) -> tuple[np.ndarray, np.ndarray]:
    reduced = tuple(axis for axis, label in enumerate(labels) if label not in output)
    if reduced and any(s.shape[axis] != 1 for axis in reduced):
        c = np.max(s, axis=reduced, keepdims=True)
        return n * np.exp(s - c), c
    return n, s


def _onto_output(c: np.ndarray, labels: str, output: str) -> np.ndarray:
    retained = "".join(label for label in output if label in labels)
    squeezed = np.einsum(f"{labels}->{retained}", c)
    dims = iter(squeezed.shape)
    return squeezed.reshape(tuple(next(dims) if label in retained else 1 for label in output))


def scaled_log_einsum(format_string: str, operands: list[np.ndarray], linear: list[bool], norm: str = "sum") -> np.ndarray:
    """log(einsum(fmt, ...)) in a scaled mode, each operand exp(X) (log-domain X) or a linear value."""
    input_strings, output = parse_format_string(format_string)
    normalized, scales = [], []
    for x, labels, lin in zip(operands, input_strings, linear, strict=True):
        if lin:
            normalized.append(x)
            continue
        n, s = _exp_pair(x)
        n, c = _contraction_scale(n, s, labels, output)
        normalized.append(n)
        scales.append(_onto_output(c, labels, output))
    raw = np.einsum(format_string, *normalized, optimize=True)
    total = NORMS[norm](raw, axis=-1, keepdims=True)
    log_scale = np.log(total)
    for c in scales:
        log_scale = log_scale + c
    return np.log(raw / total) + log_scale


def scaled_matmul(a: np.ndarray, b: np.ndarray, norm: str = "sum") -> np.ndarray:
    """log(einsum('...ik,...kj->...ij', exp(a), exp(b))) in the scaled mode with `norm`."""
    fmt = "ik,kj->ij" if a.ndim == 2 else "bik,bkj->bij"
    return scaled_log_einsum(fmt, [a, b], [False, False], norm)


def scaled_cp_layer(x: np.ndarray, w: np.ndarray, norm: str = "sum") -> np.ndarray:
    """log(einsum('dac,dbc->dab', exp(x), w)) with linear weights w (F, O, K)."""
    return scaled_log_einsum("dac,dbc->dab", [x, w], [False, True], norm)


def scaled_tucker(left: np.ndarray, right: np.ndarray, w: np.ndarray, norm: str = "sum") -> np.ndarray:
    """log(einsum('bfi,bfj,foij->bfo', exp(l), exp(r), w)) with linear weights w."""
    return scaled_log_einsum("bfi,bfj,foij->bfo", [left, right, w], [False, False, True], norm)
