"""GPU parity of the batched-decode GEMV on the tensor cores (fn_tc_gemv / fn_test_tc_gemv, tcgen05.mma).

The path dequantises each weight exactly (the same values as fn_test_dequant, bit-exact vs gguf-py), splits weights
and x into bf16 hi / lo pairs and accumulates hi*hi + hi*lo + lo*hi in fp32 tensor memory. Stated tolerance: max
|y - y64| <= 1e-4 * max |y64| against float64 on the exactly dequantised weights (the expected error is about 3e-5:
each product keeps about 16 mantissa bits). Also: deterministic, the device-pointer entry equal to the host hook, and
tokens beyond nt never written.
"""

import numpy as np
import pytest

from oracle import dequant as D
from synth import BY_NAME, random_blocks, random_x

pytestmark = pytest.mark.gpu
TC_TOL = 1e-4


def ref(qt, W, rows, cols, x):
    return x.astype(np.float64) @ D.dequant_rows(W, qt, rows, cols).astype(np.float64).T


@pytest.mark.parametrize("name", ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K",
                                  "IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "IQ4_NL", "IQ4_XS", "BF16", "Q2_0"])
@pytest.mark.parametrize("rows,cols,nt", [(4096, 2048, 32), (2048, 4096, 8), (300, 1024, 17)])
def test_tc_gemv_parity(fn, name, rows, cols, nt):
    rng = np.random.default_rng(rows + cols + nt + len(name))
    qt = BY_NAME[name]
    W = random_blocks(qt, rows, cols, rng)
    x = random_x(nt, cols, rng)
    y = fn.test_tc_gemv(qt, W, rows, cols, x)
    y64 = ref(qt, W, rows, cols, x)
    err = float(np.abs(y - y64).max() / np.abs(y64).max())
    assert err <= TC_TOL, f"{name} {rows}x{cols} nt={nt}: rel err {err:.3e}"


@pytest.mark.parametrize("nt", [1, 2, 15, 16, 31, 32])
def test_tc_gemv_token_counts(fn, nt):
    """N = 16 for nt <= 16, else 32; padded token columns are zero and never written."""
    rng = np.random.default_rng(nt)
    qt, rows, cols = BY_NAME["Q4_K"], 512, 2048
    W = random_blocks(qt, rows, cols, rng)
    x = random_x(nt, cols, rng)
    y = fn.test_tc_gemv(qt, W, rows, cols, x)
    y64 = ref(qt, W, rows, cols, x)
    assert np.abs(y - y64).max() <= TC_TOL * np.abs(y64).max()


def test_tc_gemv_device_entry_and_determinism(fn):
    import torch
    rng = np.random.default_rng(5)
    qt, rows, cols, nt = BY_NAME["IQ3_XXS"], 1000, 2048, 24
    W = random_blocks(qt, rows, cols, rng)
    x = random_x(nt, cols, rng)
    h = fn.tc_create(qt, W, rows, cols)
    dev = torch.device("cuda")
    xd = torch.from_numpy(x).to(dev)
    y = torch.full((nt + 1, rows), 7.0, device=dev)  # a guard row past nt
    outs = []
    for _ in range(3):
        fn.tc_gemv(h, xd.data_ptr(), cols, y.data_ptr(), rows, nt)
        fn.sync()
        outs.append(y.cpu().numpy().copy())
    fn.tc_free(h)
    host = fn.test_tc_gemv(qt, W, rows, cols, x)
    assert np.array_equal(outs[0][:nt].view(np.uint32), host.view(np.uint32))
    assert all(np.array_equal(o.view(np.uint32), outs[0].view(np.uint32)) for o in outs)
    assert np.all(outs[0][nt] == 7.0)


def test_tc_gemv_errors(fn):
    rng = np.random.default_rng(0)
    qt = BY_NAME["Q4_K"]
    W = random_blocks(qt, 64, 256, rng)
    with pytest.raises(RuntimeError):
        fn.test_tc_gemv(qt, W, 64, 256, np.zeros((33, 256), np.float32))
    W2 = random_blocks(BY_NAME["Q8_0"], 64, 96, rng)
    with pytest.raises(RuntimeError):
        fn.tc_create(BY_NAME["Q8_0"], W2, 64, 96)
