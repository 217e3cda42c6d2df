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


def amax_key(v: np.ndarray, rows: np.ndarray) -> np.ndarray:
    """The ordering key of (value, global row) the B200 kernels combine by max: the order-preserving bits of v (with
    -0 as +0) above (2^32 - 1 - row); 0 for NaN and -inf (never a winner). Restated here so that the partition logic
    can be checked on the CPU: max over keys == argmax_ref of the concatenated rows."""
    v = np.asarray(v, np.float32).copy()
    v[v == 0] = 0.0
    u = v.view(np.uint32).astype(np.uint64)
    o = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000).astype(np.uint64)
    k = (o << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.asarray(rows, np.uint64))
    return np.where(np.asarray(v) > -np.inf, k, np.uint64(0)).astype(np.uint64)


def slice_key(logits_slice: np.ndarray, row0: int) -> np.ndarray:
    """Max key per token [nt] of one rank's logit slice [nt][r] whose first row is global row row0."""
    lg = np.atleast_2d(np.asarray(logits_slice, np.float32))
    rows = row0 + np.arange(lg.shape[1], dtype=np.uint64)
    return np.array([amax_key(r, rows).max(initial=np.uint64(0)) for r in lg], np.uint64)
