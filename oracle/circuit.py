"""CPU oracle for the folded quad-tree CP circuit — TEST INFRASTRUCTURE ONLY.

Restates what the reference computes for the circuit that demo/cirkit.py
builds (to_xe_expression, demo/cirkit.py:131-187; categorical inputs,
demo/cirkit.py:525-527) after FoldSameShapedOperations
(preprocess.py:1310-1393) and the log-space translation
(backend_translation/translate.py:604-810):

  data  = softmax(categorical_logits, axis=1)[f, pixels[b, var_of_fold[f]], :]   (F0, B, K)
  level 0:   y = log einsum('dac,dbc->dab', data, softmax(logits_0, axis=2))
  level l:   x = y[:F] + y[F:]                      (folded Hadamard 'cab,cab->cab' of the two halves)
             y = log einsum('dac,dbc->dab', exp(x), softmax(logits_l, axis=2))
  root:      h = y[0] + y[1];  ll = log einsum('ab,cb->ac', exp(h), softmax(root_logits, axis=1))

The reference computes the categorical probabilities in torch and the
log-space translation takes their log; tests/golden/make_golden.py runs the
reference on this exact structure to pin this restatement.
"""

from __future__ import annotations

import numpy as np

from . import logspace


def circuit_log_likelihood(
    categorical_logits: np.ndarray,
    pixels: np.ndarray,
    var_of_fold: np.ndarray,
    level_logits: list[np.ndarray],
    root_logits: np.ndarray,
    mode: str = "max",
) -> np.ndarray:
    """Per-sample log-likelihoods (B, 1) of the folded circuit, in the inputs' dtype."""
    probs = logspace.softmax(categorical_logits, axis=1)  # (F0, S, K)
    f_idx = np.arange(probs.shape[0])[:, None]
    data = probs[f_idx, pixels[:, var_of_fold].T]  # (F0, B, K)
    x = np.log(data)
    y = None
    for level, logits in enumerate(level_logits):
        w = logspace.softmax(logits, axis=2)  # (F, O, K)
        if level > 0:
            half = y.shape[0] // 2
            x = y[:half] + y[half:]
        y = logspace.logspace_einsum("dac,dbc->dab", [x, w], [False, True], mode)
    h = y[0] + y[1]
    w_root = logspace.softmax(root_logits, axis=1)
    return logspace.logspace_einsum("ab,cb->ac", [h, w_root], [False, True], mode)
