"""CPU oracle for the lm_head argmax.  TEST INFRASTRUCTURE ONLY.

Restates k_argmax (engine/faie2fn.cu:1910-1935): each thread scans its strided elements keeping (v, idx) with a strict
`l[i] > v` starting from (-inf, 0), then warps and the block merge with "larger value, or equal value and lower
index". The resulting rule, written out here element by element in index order:
  * the winner is the lowest index holding the largest value;
  * NaN never compares greater, so it never wins;
  * -0.0 == +0.0 under `>` / `==`, so the two zeros tie and the lower index wins;
  * when no element exceeds -inf (all -inf and/or NaN) nothing replaces the initial (-inf, 0): the result is 0.
"""

from __future__ import annotations

import numpy as np


def argmax_ref(logits: np.ndarray) -> np.ndarray:
    """argmax [nt] of logits [nt][n] (or [n]) by the rule above; a plain loop, for small rows."""
    lg = np.atleast_2d(np.asarray(logits, np.float32))
    out = np.zeros(lg.shape[0], np.int64)
    for t, row in enumerate(lg):
        v, idx = -np.inf, 0
        for i, x in enumerate(row.tolist()):
            if x > v:
                v, idx = x, i
        out[t] = idx
    return out


def argmax_fast(logits: np.ndarray) -> np.ndarray:
    """The same rule vectorised (checked against argmax_ref in the CPU suite): NaN -> -inf, then the first index of
    the maximum (numpy's argmax returns the first occurrence, and -0.0 == 0.0 there too)."""
    lg = np.atleast_2d(np.asarray(logits, np.float32))
    clean = np.where(np.isnan(lg), -np.inf, lg)
    idx = np.argmax(clean, axis=1)
    # rows whose maximum is -inf (every element -inf or NaN): index 0
    return np.where(clean[np.arange(lg.shape[0]), idx] > -np.inf, idx, 0).astype(np.int64)
