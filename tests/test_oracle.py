"""CPU: the oracle is pinned before it is trusted.

1. oracle/dequant.py equals the committed gguf-py golden fixtures bit for bit (all 19 formats, extreme scales too);
2. it equals gguf-py 0.19.0 live on fresh seeded blocks at several shapes (18 formats; Q2_0 has no gguf-py decoder);
3. the generated codebook header equals gguf-py's tables, and the ksigns rule equals gguf-py's ksigns bytes;
4. the float64 GEMV reference reproduces the fixture's y64.
"""

import os
import re

import numpy as np
import pytest

from oracle import dequant as O
from synth import TYPES, random_blocks

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
gguf = pytest.importorskip("gguf")


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("qtype", sorted(TYPES))
def test_oracle_matches_golden(golden, qtype):
    name = TYPES[qtype][0]
    raw = golden[f"{name}/raw"]
    got = O.dequant_rows(raw, qtype, raw.shape[0], 512)
    assert np.array_equal(bits(got), bits(golden[f"{name}/out"])), name
    if f"{name}/xraw" in golden:
        xr = golden[f"{name}/xraw"]
        got = O.dequant_rows(xr, qtype, xr.shape[0], 512)
        assert np.array_equal(bits(got), bits(golden[f"{name}/xout"])), name + " (extreme scales)"


@pytest.mark.parametrize("qtype", [t for t in sorted(TYPES) if TYPES[t][0] != "Q2_0"])
@pytest.mark.parametrize("rows,cols", [(3, 256), (17, 2048), (64, 4096)])
def test_oracle_matches_ggufpy_live(qtype, rows, cols):
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as QT
    rng = np.random.default_rng(qtype * 1000 + rows)
    raw = random_blocks(qtype, rows, cols, rng)
    ref = quants.dequantize(raw, QT(qtype)).reshape(rows, cols)
    got = O.dequant_rows(raw, qtype, rows, cols)
    assert np.array_equal(bits(got), bits(ref))


def test_ksigns_rule_matches_ggufpy():
    from gguf import quants
    assert np.array_equal(O.KSIGNS, np.frombuffer(quants.IQ2_XXS.ksigns, np.uint8))


def test_codebook_header_matches_ggufpy():
    from gguf import quants
    txt = open(os.path.join(ROOT, "faie2-flashnext_b200", "csrc", "fn_grids.h")).read()
    for arr, cls in [("kIq2xxsGrid", quants.IQ2_XXS), ("kIq2xsGrid", quants.IQ2_XS), ("kIq2sGrid", quants.IQ2_S),
                     ("kIq3xxsGrid", quants.IQ3_XXS), ("kIq3sGrid", quants.IQ3_S)]:
        body = re.search(arr + r"\[\d+\] = \{(.*?)\};", txt, re.S).group(1)
        words = np.array([int(w, 16) for w in re.findall(r"0x([0-9a-f]{8})u", body)], np.uint32)
        cls.init_grid()
        want = cls.grid.reshape(cls.grid_shape).astype(np.uint8).reshape(-1).view("<u4")
        assert np.array_equal(words, want), arr
    kv = re.search(r"kIq4nlValues\[16\] = \{(.*?)\}", txt).group(1)
    assert tuple(int(v) for v in kv.split(",")) == tuple(quants.IQ4_NL.kvalues)


@pytest.mark.parametrize("qtype", sorted(TYPES))
def test_gemv64_matches_golden(golden, qtype):
    name = TYPES[qtype][0]
    w = O.dequant_rows(golden[f"{name}/raw"], qtype, 4, 512)
    y = O.gemv64(w, golden[f"{name}/x"])
    assert np.allclose(y, golden[f"{name}/y64"], rtol=0, atol=1e-12 * max(1.0, np.abs(y).max()))


def test_rel_err_measure():
    y64 = np.array([[1.0, -2.0, 4.0]])
    assert O.gemv_rel_err(np.array([[1.0, -2.0, 4.0 + 4e-7]], np.float32), y64) == pytest.approx(1e-7, rel=0.2)


def test_row_bytes_and_errors():
    assert O.row_bytes(12, 2048) == 8 * 144
    assert O.row_bytes(42, 128) == 36
    with pytest.raises(ValueError):
        O.row_bytes(12, 100)
