"""GPU parity of the lm_head argmax (k_argmax, engine/faie2fn.cu:1910-1935; lm_head + argmax at :2446-2447) through
the C ABI: the stand-alone kernel over logits and the argmax fused into the lm_head GEMV's last CTA. Bar: the index
is exactly the oracle's (oracle/argmax.py) on the same logits: lowest index of the largest value, NaN never wins, -0
ties +0, index 0 when nothing exceeds -inf."""

import numpy as np
import pytest

from oracle import dequant as O
from oracle.argmax import argmax_fast
from synth import BY_NAME, random_blocks, random_x

pytestmark = pytest.mark.gpu
NAN, INF = np.float32("nan"), np.float32("inf")
VOCAB = 151936


def test_argmax_standalone_edge_rows(fn):
    rng = np.random.default_rng(1)
    n = VOCAB
    rows = []
    r = rng.standard_normal(n).astype(np.float32)
    rows.append(r.copy())
    m = np.float32(r.max() + 1)
    for pos in (n - 1, 77777, 5000, 4097):  # ties spread over threads, warps and the tail
        r[pos] = m
    rows.append(r.copy())
    r = rng.standard_normal(n).astype(np.float32)
    r[rng.choice(n, 1000, replace=False)] = NAN
    rows.append(r)
    rows.append(np.full(n, -INF, np.float32))
    rows.append(np.where(rng.random(n) < 0.5, -INF, NAN).astype(np.float32))
    r = -np.abs(rng.standard_normal(n)).astype(np.float32) - 1
    r[[90001, 123]] = np.float32(-0.0)
    r[[100, 150000]] = np.float32(0.0)
    rows.append(r)
    r = rng.standard_normal(n).astype(np.float32)
    r[[3, 140000]] = INF
    rows.append(r)
    lg = np.stack(rows)
    got = fn.argmax(lg)
    assert np.array_equal(got, argmax_fast(lg)), (got, argmax_fast(lg))


@pytest.mark.parametrize("n", [1, 3, 4, 1023, 4096, 4099])
def test_argmax_standalone_small_and_ragged(fn, n):
    rng = np.random.default_rng(n)
    lg = rng.integers(-3, 3, size=(5, n)).astype(np.float32)  # many ties
    assert np.array_equal(fn.argmax(lg), argmax_fast(lg))


@pytest.mark.parametrize("qtype,rows,cols", [(BY_NAME["Q6_K"], 20000, 2048), (BY_NAME["Q8_0"], 4099, 1024),
                                             (BY_NAME["Q4_K"], 300, 2048), (BY_NAME["BF16"], 777, 512)])
def test_gemv_argmax_fused(fn, qtype, rows, cols):
    """Fused argmax == oracle argmax of the GEMV's own logits; the logits equal the plain GEMV's; the index does not
    depend on whether logits are written; planted duplicate rows (exact ties, equal bits) resolve to the lowest."""
    rng = np.random.default_rng(rows)
    raw = random_blocks(qtype, rows, cols, rng).reshape(rows, -1)
    x = random_x(3, cols, rng)
    y0 = fn.gemv(qtype, raw, rows, cols, x)
    best = int(np.argmax(y0[0]))
    for pos in (rows - 1, rows // 2, 0 if best > 0 else 1):  # duplicate token 0's best row: an exact tie
        raw[pos] = raw[best]
    idx, y = fn.gemv_argmax(qtype, raw, rows, cols, x)
    assert np.array_equal(y, fn.gemv(qtype, raw, rows, cols, x))
    assert np.array_equal(idx, argmax_fast(y))
    assert idx[0] == min(best, rows // 2, 0 if best > 0 else 1, rows - 1)
    idx2, none = fn.gemv_argmax(qtype, raw, rows, cols, x, logits=False)
    assert none is None and np.array_equal(idx2, idx)
    idx1, _ = fn.gemv_argmax(qtype, raw, rows, cols, x[1:2])
    assert idx1[0] == idx[1]


def test_gemv_argmax_nan_rows_never_win(fn):
    qtype, rows, cols = BY_NAME["Q8_0"], 5000, 512
    rng = np.random.default_rng(3)
    raw = random_blocks(qtype, rows, cols, rng).reshape(rows, -1)
    bad = rng.choice(rows, 200, replace=False)
    raw[bad, 0:2] = np.frombuffer(np.float16(np.nan).tobytes(), np.uint8)  # block 0's scale d = NaN
    x = random_x(1, cols, rng)
    idx, y = fn.gemv_argmax(qtype, raw, rows, cols, x)
    assert np.isnan(y[0, bad]).all()
    assert np.array_equal(idx, argmax_fast(y))


def test_gemv_argmax_lm_head_handle(fn):
    """The resident-handle entry with host buffers on the Q6_K lm_head shape, three calls in a row (the ticket is
    reset by each launch), against the oracle argmax of the plain GEMV's logits and the dequantised weights."""
    import torch
    qtype, rows, cols = BY_NAME["Q6_K"], VOCAB, 2048
    rng = np.random.default_rng(5)
    raw = random_blocks(qtype, rows, cols, rng)
    h = fn.w_create(qtype, raw, rows, cols)
    try:
        st = torch.cuda.current_stream().cuda_stream
        for rep in range(3):
            x = random_x(1, cols, rng)
            xh = torch.from_numpy(x).pin_memory()
            yh = torch.empty((1, rows), dtype=torch.float32).pin_memory()
            ih = torch.zeros(1, dtype=torch.int32).pin_memory()
            fn.w_gemv_argmax_host(h, xh.data_ptr(), 1, yh.data_ptr(), ih.data_ptr(), st)
            fn.sync(st)
            y = yh.numpy()
            assert int(ih[0]) == int(argmax_fast(y)[0])
            w = int(ih[0])
            y64 = O.gemv64(O.dequant_rows(raw[w:w + 1], qtype, 1, cols), x)
            assert abs(float(y[0, w]) - float(y64[0, 0])) <= 2e-7 * np.abs(y).max()
    finally:
        fn.w_free(h)


def test_step_host_matches_single_calls(fn):
    """fn_w_step_host (one copy in, the GEMVs as a replayed graph, one copy out) gives the same bits as one-call-per-GEMV
    launches, twice in a row (the second call replays the cached graph), with the lm_head's argmax instead of logits."""
    import torch
    rng = np.random.default_rng(17)
    specs = [("Q4_K", 4096, 2048), ("IQ3_XXS", 512, 2048), ("Q8_0", 2048, 4096), ("Q6_K", 20000, 2048)]
    hs, raws = [], []
    for name, r, c in specs:
        raws.append(random_blocks(BY_NAME[name], r, c, rng))
        hs.append(fn.w_create(BY_NAME[name], raws[-1], r, c))
    try:
        st = torch.cuda.current_stream().cuda_stream
        for rep in range(2):
            xs = [random_x(1, c, rng)[0] for _, _, c in specs]
            xh = torch.from_numpy(np.concatenate(xs)).pin_memory()
            yh = torch.zeros(sum(r for _, r, _ in specs[:-1]), dtype=torch.float32).pin_memory()
            ih = torch.full((1,), -1, dtype=torch.int32).pin_memory()
            fn.w_step_host(hs, xh.data_ptr(), yh.data_ptr(), len(hs) - 1, ih.data_ptr(), st)
            fn.sync(st)
            off = 0
            for i, (name, r, c) in enumerate(specs[:-1]):
                want = fn.gemv(BY_NAME[name], raws[i], r, c, xs[i][None])[0]
                assert np.array_equal(yh.numpy()[off:off + r].view(np.uint32), want.view(np.uint32)), name
                off += r
            name, r, c = specs[-1]
            idx, _ = fn.gemv_argmax(BY_NAME[name], raws[-1], r, c, xs[-1][None], logits=False)
            assert int(ih[0]) == int(idx[0])
    finally:
        for h in hs:
            fn.w_free(h)
