"""CPU oracle for GGUF block dequantisation and the fp32 GEMV.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use this module, and only
as the checker. The product path (the CUDA library) never calls it.

What it restates: the dequantisation the reference relies on, `dequant()` in
flashnext/ref_fn.py:44-53, which calls gguf-py `quants.dequantize` for every ggml format and
restates Q2_0 itself (ref_fn.py:46-52, "ggml-quants.c dequantize_row_q2_0"). gguf-py is a
third-party dependency that is not vendored in the reference (the reference reaches it through an
unshipped `faie2.gguf_reader`, ref_fn.py:26,35); the version pinned here is gguf-py 0.19.0. Each
function below restates the published ggml block layout and the exact float32 rounding sequence
of gguf-py 0.19.0 `gguf/quants.py` (cited per format), in numpy, without importing gguf-py's
decoders. Parity of this restatement is pinned against gguf-py itself by the committed golden
fixtures (tests/golden/, made by tests/golden/make_golden.py) and by a live comparison in the CPU
test-suite.

Layout conventions: `blocks` is a (n, type_size) uint8 array; a decoder returns (n, block_size)
float32. Every arithmetic step is a float32 numpy operation (IEEE round-to-nearest), in the order
gguf-py performs it, so the results are bit-identical.
"""

from __future__ import annotations

import numpy as np

# ggml type ids -> (name, values per block, bytes per block).  Reference table: engine/faie2fn.cu:78-103
# (13 formats); the six extra formats (Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K) use gguf-py GGML_QUANT_SIZES.
TYPES = {
    2: ("Q4_0", 32, 18),
    3: ("Q4_1", 32, 20),
    6: ("Q5_0", 32, 22),
    7: ("Q5_1", 32, 24),
    8: ("Q8_0", 32, 34),
    10: ("Q2_K", 256, 84),
    11: ("Q3_K", 256, 110),
    12: ("Q4_K", 256, 144),
    13: ("Q5_K", 256, 176),
    14: ("Q6_K", 256, 210),
    16: ("IQ2_XXS", 256, 66),
    17: ("IQ2_XS", 256, 74),
    18: ("IQ3_XXS", 256, 98),
    20: ("IQ4_NL", 32, 18),
    21: ("IQ3_S", 256, 110),
    22: ("IQ2_S", 256, 82),
    23: ("IQ4_XS", 256, 136),
    30: ("BF16", 1, 2),
    42: ("Q2_0", 64, 18),
}
BY_NAME = {v[0]: k for k, v in TYPES.items()}
# the 13 formats BASELINE's format sweep grades
SWEEP13 = ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ2_XXS", "IQ3_XXS", "IQ4_XS"]

F32 = np.float32
IQ4NL_VALUES = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.int8)


def row_bytes(qtype: int, cols: int) -> int:
    _, qk, b = TYPES[qtype]
    if cols % qk:
        raise ValueError(f"{TYPES[qtype][0]}: {cols} columns is not a whole number of {qk}-value blocks")
    return cols // qk * b


def _f16(b: np.ndarray, off: int) -> np.ndarray:
    """fp16 field at byte `off` of every block, as float32, shape (n, 1)."""
    return b[:, off:off + 2].copy().view(np.float16).astype(F32)


def _ksigns() -> np.ndarray:
    """ggml ksigns_iq2xs: 7 sign bits plus their parity in bit 7."""
    i = np.arange(128, dtype=np.uint32)
    par = np.zeros(128, np.uint32)
    for k in range(7):
        par ^= (i >> k) & 1
    return (i | (par << 7)).astype(np.uint8)


KSIGNS = _ksigns()


def _sign_bits(sbytes: np.ndarray) -> np.ndarray:
    """(…,) sign bytes -> (…, 8) float32 of +1/-1 (bit k set -> value k negated)."""
    bits = (sbytes[..., None] >> np.arange(8, dtype=np.uint8)) & 1
    return np.where(bits == 0, F32(1), F32(-1))


_GRIDS: dict = {}


def grid(name: str) -> np.ndarray:
    """IQ codebook (entries, values) as float32, from gguf-py's packed tables (ggml-common.h data)."""
    if name not in _GRIDS:
        from gguf import quants
        cls = getattr(quants, name)
        cls.init_grid()
        _GRIDS[name] = cls.grid.reshape(cls.grid_shape).astype(F32)
    return _GRIDS[name]


# ---- 32-value formats (gguf-py quants.py:220-403) -------------------------------------------------------------

def _nibbles16(qs: np.ndarray) -> np.ndarray:
    """16 bytes -> 32 nibbles: values 0..15 are the low nibbles, 16..31 the high nibbles."""
    return np.concatenate([qs & 15, qs >> 4], axis=-1)


def dq_q4_0(b):  # quants.py:241-251  d * (q - 8)
    d = _f16(b, 0)
    q = _nibbles16(b[:, 2:18]).astype(np.int8) - np.int8(8)
    return d * q.astype(F32)


def dq_q4_1(b):  # quants.py:276-288  d * q + m
    d, m = _f16(b, 0), _f16(b, 2)
    q = _nibbles16(b[:, 4:20]).astype(F32)
    return (d * q) + m


def _qh32(b, off):
    qh = b[:, off:off + 4].copy().view("<u4")  # (n, 1)
    return ((qh >> np.arange(32, dtype=np.uint32)) & 1).astype(np.uint8)


def dq_q5_0(b):  # quants.py:314-330  d * (q - 16), q = low nibble | qh bit << 4
    d = _f16(b, 0)
    q = (_nibbles16(b[:, 6:22]) | (_qh32(b, 2) << 4)).astype(np.int8) - np.int8(16)
    return d * q.astype(F32)


def dq_q5_1(b):  # quants.py:357-375  d * q + m
    d, m = _f16(b, 0), _f16(b, 2)
    q = (_nibbles16(b[:, 8:24]) | (_qh32(b, 4) << 4)).astype(F32)
    return (d * q) + m


def dq_q8_0(b):  # quants.py:396-401  q * d
    d = _f16(b, 0)
    return b[:, 2:34].view(np.int8).astype(F32) * d


def dq_iq4_nl(b):  # quants.py IQ4_NL.dequantize_blocks  d * kvalues[q]
    d = _f16(b, 0)
    return d * IQ4NL_VALUES[_nibbles16(b[:, 2:18])].astype(F32)


def dq_q2_0(b):
    """Q2_0 (ggml type 42, 64 values in 18 bytes): value 4i + k = ((qs[i] >> 2k) & 3) - 1, times d.
    Restates flashnext/ref_fn.py:46-52 (there in float64; the product of an fp16 and an integer in
    [-1, 2] is exact, so float32 gives the same value)."""
    d = _f16(b, 0)
    qs = b[:, 2:18]
    q = np.stack([(qs >> s) & 3 for s in (0, 2, 4, 6)], axis=-1).reshape(-1, 64).astype(F32)
    return (q - F32(1)) * d


def dq_bf16(b):  # quants.py:216-217
    return (b.view(np.int16).astype(np.int32) << 16).view(F32)


# ---- K-quants (256 values; quants.py:404-572) ---------------------------------------------------------------

def _scale_min_k4(s: np.ndarray):
    """12 packed bytes -> 8 six-bit scales and 8 six-bit mins (quants.py:479-502)."""
    sc = np.empty((s.shape[0], 8), np.uint8)
    mn = np.empty((s.shape[0], 8), np.uint8)
    sc[:, :4] = s[:, 0:4] & 63
    mn[:, :4] = s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return sc, mn


def _k_low_nibbles(qs: np.ndarray) -> np.ndarray:
    """128 bytes -> 8 sub-blocks of 32 4-bit values: sub-block j = nibble (j & 1) of bytes 32 (j >> 1) .. +31."""
    n = qs.shape[0]
    q = qs.reshape(n, 4, 1, 32) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)
    return (q & 15).reshape(n, 8, 32)


def dq_q4_k(b):  # quants.py:504-522  (d*sc)*q - dmin*m
    n = b.shape[0]
    d, dmin = _f16(b, 0), _f16(b, 2)
    sc, mn = _scale_min_k4(b[:, 4:16])
    dl = (d * sc.astype(F32)).reshape(n, 8, 1)
    ml = (dmin * mn.astype(F32)).reshape(n, 8, 1)
    q = _k_low_nibbles(b[:, 16:144]).astype(F32)
    return (dl * q - ml).reshape(n, 256)


def dq_q5_k(b):  # quants.py:527-549
    n = b.shape[0]
    d, dmin = _f16(b, 0), _f16(b, 2)
    sc, mn = _scale_min_k4(b[:, 4:16])
    dl = (d * sc.astype(F32)).reshape(n, 8, 1)
    ml = (dmin * mn.astype(F32)).reshape(n, 8, 1)
    qh = b[:, 16:48]
    hbit = ((qh.reshape(n, 1, 32) >> np.arange(8, dtype=np.uint8).reshape(1, 8, 1)) & 1)  # sub-block j: bit j
    q = (_k_low_nibbles(b[:, 48:176]) | (hbit << 4)).astype(F32)
    return (dl * q - ml).reshape(n, 256)


def dq_q6_k(b):  # quants.py:554-572  (d*sc)*(q-32), 16-value scale groups
    n = b.shape[0]
    ql, qh = b[:, 0:128], b[:, 128:192]
    sc = b[:, 192:208].view(np.int8).astype(F32)
    d = _f16(b, 208)
    dl = (d * sc).reshape(n, 16, 1)
    lo = ((ql.reshape(n, 2, 1, 64) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)) & 15).reshape(n, 8, 32)
    hi = ((qh.reshape(n, 2, 1, 32) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)) & 3).reshape(n, 8, 32)
    q = ((lo | (hi << 4)).astype(np.int8) - np.int8(32)).reshape(n, 16, 16).astype(F32)
    return (dl * q).reshape(n, 256)


def dq_q2_k(b):  # quants.py:406-428  (d*(sc&15))*q - dmin*(sc>>4), 16-value scale groups
    n = b.shape[0]
    scales, qs = b[:, 0:16], b[:, 16:80]
    d, dmin = _f16(b, 80), _f16(b, 82)
    dl = (d * (scales & 15).astype(F32)).reshape(n, 16, 1)
    ml = (dmin * (scales >> 4).astype(F32)).reshape(n, 16, 1)
    q = ((qs.reshape(n, 2, 1, 32) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)) & 3)
    q = q.reshape(n, 16, 16).astype(F32)
    return (dl * q - ml).reshape(n, 256)


def dq_q3_k(b):  # quants.py:433-472  (d*(sc-32))*q, q = 2 low bits - 4 * (1 - hmask bit)
    n = b.shape[0]
    hmask, qs, s = b[:, 0:32], b[:, 32:96], b[:, 96:108]
    d = _f16(b, 108)
    low = ((s[:, 0:8].reshape(n, 1, 8) >> np.array([0, 4], np.uint8).reshape(1, 2, 1)) & 15).reshape(n, 16)
    high = ((s[:, 8:12].reshape(n, 1, 4) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 4, 1)) & 3).reshape(n, 16)
    sc = ((low | (high << 4)).astype(np.int8) - np.int8(32)).astype(F32)
    dl = (d * sc).reshape(n, 16, 1)
    ql = ((qs.reshape(n, 2, 1, 32) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)) & 3).reshape(n, 16, 16)
    hb = ((hmask.reshape(n, 1, 32) >> np.arange(8, dtype=np.uint8).reshape(1, 8, 1)) & 1).reshape(n, 16, 16)
    q = (ql.astype(np.int8) - ((hb ^ 1) << 2).astype(np.int8)).astype(F32)
    return (dl * q).reshape(n, 256)


# ---- IQ formats (256 values; quants.py:766-1125, 1330-1377) ------------------------------------------------

def _db_half(d, s4, mult):
    """d * (0.5 + s) * mult, rounded after each step as gguf-py does."""
    return (d * (F32(0.5) + s4.astype(F32))) * F32(mult)


def dq_iq2_xxs(b):  # quants.py:802-828
    n = b.shape[0]
    d = _f16(b, 0)
    w = b[:, 2:66].copy().view("<u4").reshape(n, 8, 2)
    db = _db_half(d, w[..., 1] >> 28, 0.25).reshape(n, 8, 1, 1)
    sidx = ((w[..., 1:2] >> np.array([0, 7, 14, 21], np.uint32)) & 127)  # (n, 8, 4)
    signs = _sign_bits(KSIGNS[sidx])  # (n, 8, 4, 8)
    gidx = w[..., 0:1].copy().view(np.uint8).reshape(n, 8, 4)
    g = grid("IQ2_XXS")[gidx]  # (n, 8, 4, 8)
    return (db * g * signs).reshape(n, 256)


def dq_iq2_xs(b):  # quants.py:872-898
    n = b.shape[0]
    d = _f16(b, 0)
    qs = b[:, 2:66].copy().view("<u2").reshape(n, 32)
    sc = b[:, 66:74]
    s4 = np.stack([sc & 15, sc >> 4], axis=-1).reshape(n, 16)
    db = _db_half(d, s4, 0.25).reshape(n, 16, 1, 1)
    signs = _sign_bits(KSIGNS[qs >> 9]).reshape(n, 16, 2, 8)
    g = grid("IQ2_XS")[qs & 511].reshape(n, 16, 2, 8)
    return (db * g * signs).reshape(n, 256)


def dq_iq2_s(b):  # quants.py:974-1002
    n = b.shape[0]
    d = _f16(b, 0)
    qs, sg, qh, sc = b[:, 2:34], b[:, 34:66], b[:, 66:74], b[:, 74:82]
    s4 = np.stack([sc & 15, sc >> 4], axis=-1).reshape(n, 16)
    db = _db_half(d, s4, 0.25).reshape(n, 16, 1, 1)
    signs = _sign_bits(sg).reshape(n, 16, 2, 8)
    hi = ((qh.reshape(n, 8, 1) >> np.array([0, 2, 4, 6], np.uint8)) & 3).reshape(n, 32).astype(np.uint16)
    idx = qs.astype(np.uint16) | (hi << 8)
    g = grid("IQ2_S")[idx].reshape(n, 16, 2, 8)
    return (db * g * signs).reshape(n, 256)


def dq_iq3_xxs(b):  # quants.py:1028-1054
    n = b.shape[0]
    d = _f16(b, 0)
    qs = b[:, 2:66]
    w = b[:, 66:98].copy().view("<u4").reshape(n, 8)
    db = _db_half(d, w >> 28, 0.5).reshape(n, 8, 1, 1)
    sidx = (w[..., None] >> np.array([0, 7, 14, 21], np.uint32)) & 127
    signs = _sign_bits(KSIGNS[sidx])  # (n, 8, 4, 8)
    g = grid("IQ3_XXS")[qs].reshape(n, 8, 4, 8)
    return (db * g * signs).reshape(n, 256)


def dq_iq3_s(b):  # quants.py:1096-1125  d * (1 + 2 s)
    n = b.shape[0]
    d = _f16(b, 0)
    qs, qh, sg, sc = b[:, 2:66], b[:, 66:74], b[:, 74:106], b[:, 106:110]
    s4 = np.stack([sc & 15, sc >> 4], axis=-1).reshape(n, 8)
    db = (d * (1 + 2 * s4).astype(F32)).reshape(n, 8, 1, 1)
    signs = _sign_bits(sg).reshape(n, 8, 4, 8)
    hb = ((qh.reshape(n, 8, 1) >> np.arange(8, dtype=np.uint8)) & 1).reshape(n, 64).astype(np.uint16)
    idx = qs.astype(np.uint16) | (hb << 8)
    g = grid("IQ3_S")[idx].reshape(n, 8, 4, 8)
    return (db * g * signs).reshape(n, 256)


def dq_iq4_xs(b):  # quants.py IQ4_XS.dequantize_blocks
    n = b.shape[0]
    d = _f16(b, 0)
    sh = b[:, 2:4].copy().view("<u2")  # (n, 1)
    sl = b[:, 4:8]
    lo = np.stack([sl & 15, sl >> 4], axis=-1).reshape(n, 8)
    hi = ((sh >> (2 * np.arange(8, dtype=np.uint16))) & 3).astype(np.uint8)
    ls = ((lo | (hi << 4)).astype(np.int8) - np.int8(32)).astype(F32)
    dl = (d * ls).reshape(n, 8, 1)
    qs = b[:, 8:136].reshape(n, 8, 16)
    q = np.concatenate([qs & 15, qs >> 4], axis=-1)  # (n, 8, 32)
    return (dl * IQ4NL_VALUES[q].astype(F32)).reshape(n, 256)


DECODERS = {
    2: dq_q4_0, 3: dq_q4_1, 6: dq_q5_0, 7: dq_q5_1, 8: dq_q8_0, 10: dq_q2_k, 11: dq_q3_k, 12: dq_q4_k,
    13: dq_q5_k, 14: dq_q6_k, 16: dq_iq2_xxs, 17: dq_iq2_xs, 18: dq_iq3_xxs, 20: dq_iq4_nl, 21: dq_iq3_s,
    22: dq_iq2_s, 23: dq_iq4_xs, 30: dq_bf16, 42: dq_q2_0,
}


def dequant_rows(raw: np.ndarray, qtype: int, rows: int, cols: int) -> np.ndarray:
    """GGUF rows (rows x row_bytes uint8) -> (rows, cols) float32, bit-identical to gguf-py."""
    _, qk, tb = TYPES[qtype]
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(rows, row_bytes(qtype, cols))
    blocks = raw.reshape(-1, tb)
    return DECODERS[qtype](blocks).astype(F32, copy=False).reshape(rows, cols)


def gemv64(w32: np.ndarray, x: np.ndarray) -> np.ndarray:
    """float64 y[t][r] = sum_c W[r][c] x[t][c] on the exactly dequantised weights
    (flashnext/test_fn_quants.py:34)."""
    return np.asarray(x, np.float64) @ np.asarray(w32, np.float64).T


def gemv_rel_err(y: np.ndarray, y64: np.ndarray) -> float:
    """max |y - y64| / max |y64|, the reference's GEMV error measure (flashnext/test_fn_quants.py:36)."""
    den = float(np.abs(y64).max())
    return float(np.abs(np.asarray(y, np.float64) - y64).max()) / max(den, 1e-300)
