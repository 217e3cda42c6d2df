"""GPU: the Q4_K / Q6_K GEMV as exact integer products on the tensor cores (csrc/fn_qmma.cu, fn_qmma(1), rows of up
to 2048 columns), against the float64 oracle and against the CUDA-core GEMV (fn_qmma(0)).

The integer path forms sum q X exactly (X = x in 31-bit fixed point per token) and applies the group scales in double,
so its results are within the GEMV bar (2e-7 of max |y| vs float64 on the dequantised weights) with room to spare;
a token's result is the same bits in every batch size (batches of more than the per-launch tokens run as several
launches) and the fused argmax is the index of the largest logit.
"""

import numpy as np
import pytest

from oracle import dequant as O
from synth import BY_NAME, random_blocks, random_x

pytestmark = pytest.mark.gpu
GEMV_TOL = 2e-7
FMTS = [BY_NAME["Q4_K"], BY_NAME["Q6_K"]]


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.fixture
def both(fn):
    fn.qmma(1)
    yield fn
    fn.qmma(0)


@pytest.mark.parametrize("qtype", FMTS)
@pytest.mark.parametrize("rows,cols", [(1, 256), (5, 512), (127, 1024), (129, 2048), (300, 768), (4096, 2048),
                                       (12352, 2048)])
def test_qmma_parity(both, qtype, rows, cols):
    fn = both
    rng = np.random.default_rng(rows * 7 + cols + qtype)
    raw = random_blocks(qtype, rows, cols, rng)
    x = random_x(3, cols, rng)
    W = O.dequant_rows(raw, qtype, rows, cols)
    fn.qmma(1)
    y = fn.gemv(qtype, raw, rows, cols, x)
    assert O.gemv_rel_err(y, O.gemv64(W, x)) <= GEMV_TOL
    fn.qmma(0)
    y0 = fn.gemv(qtype, raw, rows, cols, x)
    assert O.gemv_rel_err(y0, O.gemv64(W, x)) <= GEMV_TOL


@pytest.mark.parametrize("qtype", FMTS)
def test_qmma_batch_invariance(both, qtype):
    fn = both
    rows, cols = 333, 2048
    rng = np.random.default_rng(qtype + 11)
    raw = random_blocks(qtype, rows, cols, rng)
    x = random_x(8, cols, rng)
    y8 = fn.gemv(qtype, raw, rows, cols, x)
    for lo, hi in ((0, 1), (5, 6), (0, 3), (2, 7)):
        y = fn.gemv(qtype, raw, rows, cols, x[lo:hi])
        assert np.array_equal(bits(y), bits(y8[lo:hi])), (lo, hi)


@pytest.mark.parametrize("qtype", FMTS)
@pytest.mark.parametrize("scale", [1e-30, 1e-12, 1e12, 1e28])
def test_qmma_activation_scale_extremes(both, qtype, scale):
    fn = both
    rows, cols = 300, 2048
    rng = np.random.default_rng(int(np.log10(scale)) + 300)
    raw = random_blocks(qtype, rows, cols, rng)
    x = random_x(2, cols, rng)
    x[0] *= np.float32(scale)
    x[1, ::7] = 0.0
    y = fn.gemv(qtype, raw, rows, cols, x)
    W = O.dequant_rows(raw, qtype, rows, cols)
    for t in range(2):
        assert O.gemv_rel_err(y[t:t + 1], O.gemv64(W, x[t:t + 1])) <= GEMV_TOL, t
    z = fn.gemv(qtype, raw, rows, cols, np.zeros((1, cols), np.float32))
    assert not z.any()


def test_qmma_lm_head_argmax(both):
    """The Q6_K lm_head shape with its fused argmax: the index of the largest logit, on both paths."""
    fn = both
    qtype, rows, cols = BY_NAME["Q6_K"], 151936, 2048
    rng = np.random.default_rng(4242)
    raw = random_blocks(qtype, rows, cols, rng)
    x = random_x(2, cols, rng)
    idx, y = fn.gemv_argmax(qtype, raw, rows, cols, x)
    assert [int(i) for i in idx] == [int(np.argmax(y[t])) for t in range(2)]
    sample = np.concatenate([np.arange(128), rng.choice(rows, 2048, replace=False)])
    y64 = O.gemv64(O.dequant_rows(raw[sample], qtype, len(sample), cols), x)
    assert O.gemv_rel_err(y[:, sample], y64) <= GEMV_TOL
