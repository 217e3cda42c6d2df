"""CPU: the arithmetic of the integer tensor-core GEMV (csrc/fn_qmma.cu), restated in numpy on the dequantiser's own
block fields, against float64 on the exactly dequantised weights.

Per token: s = 29 - e with max |x| in [2^e, 2^(e+1)), X = round(x 2^s) (|X| < 2^30), four balanced base-256 digits
d0..d3 in [-128, 127] with X = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3; per 32-value group the integer sums S_i = sum q d_i
(what one kind::i8 MMA forms), S = S0 + 2^8 S1 + 2^16 S2 + 2^24 S3 (exact in double), and the group's value
dl S - ml SX (Q4_K) or ds0 (S_0 - 32 SX_0) + ds1 (S_1 - 32 SX_1) (Q6_K, per 16-value half); the row is their sum times
2^-s. The bar is the GEMV's: 2e-7 of max |y| against float64.
"""

import numpy as np
import pytest

from oracle import dequant as O
from synth import BY_NAME, random_blocks, random_x


def digits(X):
    """Balanced base-256 digits of int64 X (|X| < 2^30), as the kernel's qm_digits."""
    d = []
    r = X.astype(np.int64)
    for _ in range(3):
        lo = ((r & 255) ^ 128) - 128  # the low byte as a signed value
        d.append(lo)
        r = (r - lo) >> 8
    d.append(r)
    return d


def fixed_point(x):
    m = np.max(np.abs(x))
    e = int(np.floor(np.log2(m))) if m > 0 else 0
    s = 29 - e if m > 0 else 0
    return np.rint(x.astype(np.float64) * 2.0 ** s).astype(np.int64), s


def test_digits_recombine_exactly():
    rng = np.random.default_rng(1)
    X = rng.integers(-(1 << 30) + 1, 1 << 30, 100000)
    d = digits(X)
    assert all(((di >= -128) & (di <= 127)).all() for di in d)
    assert np.array_equal(d[0] + 256 * d[1] + 65536 * d[2] + 16777216 * d[3], X)


def q4k_fields(raw_row, nb):
    """Per group (8 per block): q [32] in 0..15, dl, ml as the kernel computes them (fp32 products, exact)."""
    out = []
    for b in range(nb):
        blk = raw_row[144 * b:144 * (b + 1)]
        d, dmin = np.frombuffer(blk[0:4].tobytes(), np.float16).astype(np.float32)
        sc = blk[4:16]
        qs = blk[16:144]
        for j in range(8):
            if j < 4:
                s_, m_ = sc[j] & 63, sc[j + 4] & 63
            else:
                s_ = (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4)
                m_ = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4)
            chunk = qs[32 * (j // 2):32 * (j // 2) + 32]
            q = (chunk & 15) if j % 2 == 0 else (chunk >> 4)
            out.append((q.astype(np.int64), np.float32(d) * np.float32(s_), np.float32(dmin) * np.float32(m_)))
    return out


def test_q4k_integer_path_matches_float64():
    qtype, rows, cols = BY_NAME["Q4_K"], 24, 2048
    rng = np.random.default_rng(7)
    raw = random_blocks(qtype, rows, cols, rng)
    x = random_x(1, cols, rng)[0]
    W = O.dequant_rows(raw, qtype, rows, cols).astype(np.float64)
    want = W @ x.astype(np.float64)
    X, s = fixed_point(x)
    d = digits(X)
    nb = cols // 256
    got = np.zeros(rows)
    for r in range(rows):
        acc = 0.0
        for g, (q, dl, ml) in enumerate(q4k_fields(raw[r], nb)):
            sl = slice(32 * g, 32 * g + 32)
            S = [int((q * di[sl]).sum()) for di in d]  # the MMA's exact int32 sums, one per digit
            Sv = float(S[0]) + 256.0 * S[1] + 65536.0 * S[2] + 16777216.0 * S[3]
            acc += float(dl) * Sv - float(ml) * float(X[sl].sum())
        got[r] = np.float32(np.ldexp(acc, -s))
    assert np.abs(got - want).max() / np.abs(want).max() <= 2e-7


@pytest.mark.parametrize("scale", [1e-30, 1.0, 1e28])
def test_fixed_point_range(scale):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(2048) * scale).astype(np.float32)
    X, s = fixed_point(x)
    assert np.abs(X).max() < (1 << 30)
    # relative to max |x|, the fixed-point rounding is below 2^-30
    assert np.abs(np.ldexp(X.astype(np.float64), -s) - x.astype(np.float64)).max() <= np.abs(x).max() * 2.0 ** -30
