"""CPU tests of the synthetic config-5 model's host logic: zero-mean GGUF blocks (synth.model_blocks), the pooled
weight generator, and the decode bench's algorithmic byte count."""

import os
import sys

import numpy as np
import pytest

from oracle import dequant as D
from synth import BY_NAME, TYPES, BlockPool, model_blocks, model_config, model_weights, random_blocks, row_bytes


@pytest.mark.parametrize("name", ["Q4_K", "Q5_K", "Q2_K", "Q4_1", "Q5_1"])
def test_model_blocks_are_zero_mean(name):
    """A random-byte block with a min field has a large common offset; model_blocks writes the min as the mean quant
    times the scale, so the dequantised rows average near zero relative to their spread."""
    qt = BY_NAME[name]
    rng = np.random.default_rng(1)
    rows, cols = 64, 512
    raw = random_blocks(qt, rows, cols, np.random.default_rng(1))
    cen = model_blocks(qt, rows, cols, rng)
    w_raw = D.dequant_rows(raw, qt, rows, cols).astype(np.float64)
    w_cen = D.dequant_rows(cen, qt, rows, cols).astype(np.float64)
    if name != "Q2_K":  # Q2_K's 4-bit scales and mins keep its random-byte offset small already
        assert abs(w_raw.mean()) > 0.3 * w_raw.std()
    assert abs(w_cen.mean()) < 0.05 * w_cen.std()


def test_model_blocks_leave_other_formats_alone():
    qt = BY_NAME["Q6_K"]
    a = model_blocks(qt, 8, 256, np.random.default_rng(5))
    b = random_blocks(qt, 8, 256, np.random.default_rng(5))
    assert np.array_equal(a, b)


def test_block_pool_cuts_distinct_rows():
    qt = BY_NAME["IQ3_XXS"]
    _, qk, tb = TYPES[qt]
    pool = BlockPool(qt, 1000, np.random.default_rng(2))
    t = pool.take(100, 2048)  # 800 blocks, wrapping at most once
    assert t.shape == (100, row_bytes(qt, 2048))
    blocks = t.reshape(-1, tb)
    assert len({bytes(x) for x in blocks}) == len(blocks)


def test_pooled_weights_are_lazy_and_shaped():
    cfg = dict(model_config(small=True), layers=2)
    W = model_weights(cfg, 0, pooled=True)
    assert not isinstance(W["layers"], list)
    L0 = next(W["layers"])
    ne, ffe, d = cfg["ne"], cfg["ffe"], cfg["D"]
    assert L0["moe"][0].shape == (ne * ffe, row_bytes(cfg["gate_up"], d))
    assert L0["moe"][2].shape == (ne * d, row_bytes(cfg["down"], ffe))


def test_decode_step_bytes_config5():
    """The decode bench's algorithmic bytes per step for config 5 (every weight read once, k + 1 experts per layer,
    the DeltaNet states read and written, the caches): about 2.1 GB."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if root not in sys.path:
        sys.path.insert(0, root)
    import bench
    cfg = model_config()
    b = bench.decode_step_bytes(cfg, 160)
    assert 2.0e9 < b < 2.3e9
    # one more layer of the same kind adds its projections, router, 11 experts and (DeltaNet) its state
    cfg2 = dict(cfg, layers=cfg["layers"] + 4)
    assert bench.decode_step_bytes(cfg2, 160) > b
