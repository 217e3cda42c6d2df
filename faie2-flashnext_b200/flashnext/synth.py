"""Seeded synthetic GGUF weights and activations (the benchmark's input distribution).

The reference measured on real model tensors (flashnext/test_fn_quants.py:19-31) that are not
shipped; these synthetic blocks stand in for them. Every block is uniform random bytes, then the
fp16 scale fields are overwritten with float16(|N(0,1)| * 1e-3) so every value is finite. BF16
weights are N(0, 0.05) rounded to bf16 instead (random bf16 bytes would hold NaN and Inf).
"""

from __future__ import annotations

import numpy as np

# ggml type id -> (name, values per block, bytes per block)
TYPES = {
    2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20), 6: ("Q5_0", 32, 22), 7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34),
    10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176),
    14: ("Q6_K", 256, 210), 16: ("IQ2_XXS", 256, 66), 17: ("IQ2_XS", 256, 74), 18: ("IQ3_XXS", 256, 98),
    20: ("IQ4_NL", 32, 18), 21: ("IQ3_S", 256, 110), 22: ("IQ2_S", 256, 82), 23: ("IQ4_XS", 256, 136),
    30: ("BF16", 1, 2), 42: ("Q2_0", 64, 18),
}
BY_NAME = {v[0]: k for k, v in TYPES.items()}

# byte offsets of the fp16 scale fields inside one block
SCALE_OFFSETS = {
    "Q4_0": (0,), "Q5_0": (0,), "Q8_0": (0,), "IQ2_XXS": (0,), "IQ2_XS": (0,), "IQ2_S": (0,), "IQ3_XXS": (0,),
    "IQ3_S": (0,), "IQ4_XS": (0,), "IQ4_NL": (0,), "Q2_0": (0,),
    "Q4_1": (0, 2), "Q5_1": (0, 2), "Q4_K": (0, 2), "Q5_K": (0, 2),
    "Q2_K": (80, 82), "Q3_K": (108,), "Q6_K": (208,),
}


def row_bytes(qtype: int, cols: int) -> int:
    _, qk, b = TYPES[qtype]
    if cols % qk:
        raise ValueError(f"{cols} columns is not a whole number of {qk}-value blocks")
    return cols // qk * b


def random_blocks(qtype: int, rows: int, cols: int, rng: np.random.Generator, scale: float = 1e-3) -> np.ndarray:
    """rows x row_bytes uint8 GGUF rows of format `qtype`."""
    name, qk, tb = TYPES[qtype]
    if name == "BF16":
        v = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.05)).view(np.uint32)
        return (v >> 16).astype(np.uint16).view(np.uint8).reshape(rows, cols * 2)
    nb = rows * (cols // qk)
    raw = rng.integers(0, 256, size=(nb, tb), dtype=np.uint8)
    for off in SCALE_OFFSETS[name]:
        s = (np.abs(rng.standard_normal(nb)) * scale).astype(np.float16)
        raw[:, off:off + 2] = s.view(np.uint8).reshape(nb, 2)
    return raw.reshape(rows, row_bytes(qtype, cols))


def random_x(nt: int, cols: int, rng: np.random.Generator) -> np.ndarray:
    return rng.standard_normal((nt, cols), dtype=np.float32)
