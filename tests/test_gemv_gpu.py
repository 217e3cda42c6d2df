"""GPU parity of the dequantiser and the dequant-GEMV, through the C ABI (flashnext/test_fn_quants.py is the
reference's gate: dequant error exactly 0 vs gguf-py; GEMV rel err vs float64 on the dequantised weights).

Bars: dequant bit-exact (all 19 formats, golden fixtures and seeded blocks); fp32 GEMV max|y - y64| / max|y64|
<= 2e-7 (the reference gate itself was 1e-5, test_fn_quants.py:37); one token's result is
bit-identical in every batch size and with programmatic dependent launch on or off (flashnext/bitcmp_fn.py).
"""

import numpy as np
import pytest

from oracle import dequant as O
from synth import TYPES, BY_NAME, random_blocks, random_x

pytestmark = pytest.mark.gpu
GEMV_TOL = 2e-7
ALL = sorted(TYPES)
SWEEP = [BY_NAME[n] for n in O.SWEEP13]


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("qtype", ALL)
def test_dequant_golden_bit_exact(fn, golden, qtype):
    name = TYPES[qtype][0]
    for key in ("raw", "xraw"):
        if f"{name}/{key}" not in golden:
            continue
        raw = golden[f"{name}/{key}"]
        got = fn.dequant(qtype, raw, raw.shape[0], 512)
        want = golden[f"{name}/{'out' if key == 'raw' else 'xout'}"]
        assert np.array_equal(bits(got), bits(want)), f"{name} {key}"


@pytest.mark.parametrize("qtype", ALL)
@pytest.mark.parametrize("rows,cols", [(64, 2048), (7, 4096), (1, 256)])
def test_dequant_seeded_bit_exact(fn, qtype, rows, cols):
    rng = np.random.default_rng(qtype + rows)
    raw = random_blocks(qtype, rows, cols, rng)
    got = fn.dequant(qtype, raw, rows, cols)
    want = O.dequant_rows(raw, qtype, rows, cols)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("qtype", ALL)
def test_gemv_golden(fn, golden, qtype):
    name = TYPES[qtype][0]
    y = fn.gemv(qtype, golden[f"{name}/raw"], 4, 512, golden[f"{name}/x"])
    assert O.gemv_rel_err(y, golden[f"{name}/y64"]) <= GEMV_TOL


# BASELINE config 1 and the config-2 shapes (out x in), one token, seeded synthetic blocks
@pytest.mark.parametrize("qtype", ALL)
@pytest.mark.parametrize("rows,cols", [(4096, 2048), (2048, 4096), (512, 2048)])
def test_gemv_config_shapes(fn, qtype, rows, cols):
    rng = np.random.default_rng(1000 * qtype + rows)
    raw = random_blocks(qtype, rows, cols, rng)
    x = random_x(1, cols, rng)
    y = fn.gemv(qtype, raw, rows, cols, x)
    y64 = O.gemv64(O.dequant_rows(raw, qtype, rows, cols), x)
    err = O.gemv_rel_err(y, y64)
    assert err <= GEMV_TOL, f"{TYPES[qtype][0]} {rows}x{cols}: rel err {err:.3e}"


# ragged and small shapes: rows not a multiple of a stage or a warp pass, row bytes not a multiple of 16 (padded
# rows), K not a power of two (masked lanes), tiny K with several rows per warp
@pytest.mark.parametrize("qtype", [BY_NAME[n] for n in ("Q4_K", "Q6_K", "IQ3_XXS", "Q2_K", "Q8_0", "BF16", "Q2_0")])
@pytest.mark.parametrize("rows,cols", [(1, 256), (13, 512), (100, 768), (333, 2560), (5, 1280), (37, 6144)])
def test_gemv_ragged_shapes(fn, qtype, rows, cols):
    rng = np.random.default_rng(7 * rows + cols)
    raw = random_blocks(qtype, rows, cols, rng)
    x = random_x(3, cols, rng)
    y = fn.gemv(qtype, raw, rows, cols, x)
    y64 = O.gemv64(O.dequant_rows(raw, qtype, rows, cols), x)
    assert O.gemv_rel_err(y, y64) <= GEMV_TOL


@pytest.mark.parametrize("qtype", SWEEP)
def test_gemv_batch_invariance(fn, qtype):
    """Token t's result is the same bits alone (nt=1, registers) and inside an 8-token batch (shared memory)."""
    rows, cols = 300, 2048
    rng = np.random.default_rng(qtype)
    raw = random_blocks(qtype, rows, cols, rng)
    x = random_x(8, cols, rng)
    y8 = fn.gemv(qtype, raw, rows, cols, x)
    for t in (0, 5):
        y1 = fn.gemv(qtype, raw, rows, cols, x[t:t + 1])
        assert np.array_equal(bits(y1[0]), bits(y8[t]))
    y3 = fn.gemv(qtype, raw, rows, cols, x[:3])
    assert np.array_equal(bits(y3), bits(y8[:3]))


def test_gemv_pdl_off_bit_identical(fn):
    qtype, rows, cols = BY_NAME["Q4_K"], 4096, 2048
    rng = np.random.default_rng(5)
    raw = random_blocks(qtype, rows, cols, rng)
    x = random_x(1, cols, rng)
    y_on = fn.gemv(qtype, raw, rows, cols, x)
    fn.d.fn_pdl(0)
    try:
        y_off = fn.gemv(qtype, raw, rows, cols, x)
    finally:
        fn.d.fn_pdl(1)
    assert np.array_equal(bits(y_on), bits(y_off))


def test_gemv_lm_head_q6k(fn):
    """The Q6_K lm_head shape 151936 x 2048 (255 MB): parity on a row sample and argmax of the full output."""
    qtype, rows, cols = BY_NAME["Q6_K"], 151936, 2048
    rng = np.random.default_rng(151936)
    raw = random_blocks(qtype, rows, cols, rng)
    x = random_x(1, cols, rng)
    y = fn.gemv(qtype, raw, rows, cols, x)
    idx = np.concatenate([np.arange(256), rng.choice(rows, 4096, replace=False), np.arange(rows - 256, rows)])
    y64 = O.gemv64(O.dequant_rows(raw[idx], qtype, len(idx), cols), x)
    assert O.gemv_rel_err(y[:, idx], y64) <= GEMV_TOL
    assert np.isfinite(y).all()


def test_gemv_errors(fn):
    with pytest.raises(RuntimeError):
        fn.gemv(99, np.zeros(144, np.uint8), 1, 256, np.zeros((1, 256), np.float32))
    with pytest.raises(RuntimeError):
        fn.gemv(12, np.zeros(144 * 9, np.uint8), 1, 256, np.zeros((9, 256), np.float32))  # nt > 8
    with pytest.raises(RuntimeError):
        fn.dequant(12, np.zeros(144, np.uint8), 1, 100)


def test_plan_is_batch_independent(fn):
    p = fn.gemv_plan(12, 4096, 2048)
    assert p["ldw"] == 1152 and p["lpr"] == 32 and p["gpl"] == 2
    assert p["ctas"] >= 1 and p["rows_per_stage"] >= 1


@pytest.mark.parametrize("qtype", [BY_NAME[n] for n in ("Q4_K", "Q5_K", "Q6_K", "Q4_1", "Q2_K")])
@pytest.mark.parametrize("scale", [1e-30, 1e-12, 1e12, 1e28])
def test_gemv_activation_scale_extremes(fn, qtype, scale):
    """The fast paths scale x by a per-token power of two (exact) so byte values can enter the FMAs as denormals:
    results must keep full relative accuracy for tiny and huge activations, in a batch whose tokens differ by 40
    orders of magnitude, and every token must match its own single-token result bit for bit."""
    rows, cols = 300, 2048
    rng = np.random.default_rng(int(np.log10(scale)) + 100)
    raw = random_blocks(qtype, rows, cols, rng)
    x = random_x(3, cols, rng)
    x[0] *= np.float32(scale)
    x[2] *= np.float32(1e-10)
    y = fn.gemv(qtype, raw, rows, cols, x)
    W = O.dequant_rows(raw, qtype, rows, cols)
    for t in range(3):
        y64 = O.gemv64(W, x[t:t + 1])
        assert O.gemv_rel_err(y[t:t + 1], y64) <= GEMV_TOL, f"token {t}"
        y1 = fn.gemv(qtype, raw, rows, cols, x[t:t + 1])
        assert np.array_equal(bits(y1), bits(y[t:t + 1]))


# ---- RMSNorm folded into the GEMV (fn_w_norm) ------------------------------------------------------------------
# y = rsqrt(mean x^2 + eps) (W . (x * w)): the float64 reference normalises first. The folded form rounds x * w, the
# row sum and the scale's product separately and takes rsqrtf (2 ulp), so its bar is 4e-7 of max |y| (2e-7 for the
# GEMV plus the scale's error).
NORM_TOL = 4e-7


@pytest.mark.parametrize("name,rows,cols,nt", [("Q4_K", 1024, 2048, 1), ("Q6_K", 512, 2048, 1), ("BF16", 513, 2048, 1),
                                               ("Q5_K", 700, 4096, 1), ("IQ3_XXS", 256, 2048, 3),
                                               ("Q8_0", 300, 1024, 8)])
def test_gemv_folded_rmsnorm(fn, name, rows, cols, nt):
    import torch
    rng = np.random.default_rng(rows + cols)
    qt = BY_NAME[name]
    raw = random_blocks(qt, rows, cols, rng)
    x = (random_x(nt, cols, rng) * rng.uniform(0.1, 30.0, (nt, 1))).astype(np.float32)
    w = (1.0 + 0.2 * rng.standard_normal(cols)).astype(np.float32)
    eps = 1e-6
    h = fn.w_create(qt, raw, rows, cols)
    try:
        dev = torch.device("cuda", 0)
        xd, wd = torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev)
        yd = torch.zeros(nt, rows, device=dev)
        fn.w_norm(h, wd.data_ptr(), eps)
        fn.w_gemv(h, xd.data_ptr(), cols, yd.data_ptr(), rows, nt, 0, 0)
        y = yd.cpu().numpy()
        fn.w_norm(h, 0)  # off again: the plain GEMV
        fn.w_gemv(h, xd.data_ptr(), cols, yd.data_ptr(), rows, nt, 0, 0)
        y_plain = yd.cpu().numpy()
    finally:
        fn.w_free(h)
    W64 = O.dequant_rows(raw, qt, rows, cols).astype(np.float64)
    x64 = x.astype(np.float64)
    xn = x64 / np.sqrt((x64 ** 2).mean(axis=1, keepdims=True) + eps) * w.astype(np.float64)
    y64 = xn @ W64.T
    err = float(np.abs(y - y64).max() / np.abs(y64).max())
    assert err <= NORM_TOL, f"{name} {rows}x{cols} nt={nt}: rel err {err:.3e}"
    assert O.gemv_rel_err(y_plain, O.gemv64(W64.astype(np.float32), x)) <= GEMV_TOL
