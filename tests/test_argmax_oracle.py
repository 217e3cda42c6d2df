"""CPU checks of the argmax oracle (k_argmax, engine/faie2fn.cu:1910-1935): the loop restatement on hand-made edge
cases, and the vectorised form against the loop on seeded rows with planted ties, NaN, infinities and signed zeros."""

import numpy as np

from oracle.argmax import argmax_fast, argmax_ref

NAN, INF = np.float32("nan"), np.float32("inf")


def test_edge_cases_loop():
    cases = [
        ([1.0, 3.0, 3.0, 2.0], 1),          # tie: lower index
        ([NAN, 1.0, 2.0], 2),               # NaN never wins
        ([2.0, NAN, 2.0], 0),
        ([-INF, -INF, -INF], 0),            # nothing exceeds -inf
        ([NAN, NAN], 0),
        ([NAN, -INF, -5.0], 2),
        ([-1.0, -0.0, 0.0, -2.0], 1),       # -0 ties +0: lower index
        ([-1.0, 0.0, -0.0], 1),
        ([INF, 1.0, INF], 0),
        ([-3.0, -2.0, -7.0], 1),
    ]
    for row, want in cases:
        assert argmax_ref(np.array(row, np.float32))[0] == want, row
        assert argmax_fast(np.array(row, np.float32))[0] == want, row


def test_fast_matches_loop_on_seeded_rows():
    rng = np.random.default_rng(0)
    rows = []
    for case in range(40):
        n = int(rng.integers(1, 3000))
        r = rng.standard_normal(n).astype(np.float32)
        kind = case % 5
        if kind == 1:  # planted ties of the maximum
            m = np.float32(r.max() + 1)
            r[rng.choice(n, min(n, 4), replace=False)] = m
        elif kind == 2:  # NaNs and infinities
            r[rng.choice(n, min(n, 8), replace=False)] = NAN
            r[rng.choice(n, min(n, 2), replace=False)] = -INF
        elif kind == 3:  # all non-positive with signed zeros as the maximum
            r = -np.abs(r)
            r[rng.choice(n, min(n, 3), replace=False)] = np.float32(-0.0)
            r[rng.choice(n, min(n, 2), replace=False)] = np.float32(0.0)
        elif kind == 4:  # all -inf / NaN
            r = np.where(rng.random(n) < 0.5, -INF, NAN).astype(np.float32)
        rows.append(r)
    for r in rows:
        assert argmax_fast(r)[0] == argmax_ref(r)[0]
