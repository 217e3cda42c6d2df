"""Generate dequant_golden.npz: GGUF blocks and their dequantised values computed by gguf-py 0.19.0.

gguf-py `quants.dequantize` is what the reference's oracle calls for every ggml format (flashnext/ref_fn.py:53);
Q2_0 (not in gguf-py) uses the reference's own restatement (flashnext/ref_fn.py:46-52, float64). Cases per format:
  <name>/raw, <name>/out        4 rows of seeded synthetic blocks (synth.random_blocks, the benchmark's input
                                distribution) and their values (float32; Q2_0 float64 exactly representable)
  <name>/xraw, <name>/xout      extreme scale fields: 0, the smallest fp16 subnormal, the smallest normal, 65504,
                                -1.5 and 1 (one per row), to pin subnormal / overflow-free rounding
  <name>/x, <name>/y64          two fp32 activation rows and float64 y = x . W^T on the `raw` weights
The fixture is small (a few hundred KB). Regenerate with:  python tests/golden/make_golden.py
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "faie2-flashnext_b200", "flashnext"))
from synth import SCALE_OFFSETS, TYPES, random_blocks, row_bytes  # noqa: E402

from gguf import quants  # noqa: E402
from gguf.constants import GGMLQuantizationType as QT  # noqa: E402

EXTREME = np.array([0.0, 2.0 ** -24, 2.0 ** -14, 65504.0, -1.5, 1.0], np.float16)


def ref_dequant(raw: np.ndarray, qtype: int) -> np.ndarray:
    if TYPES[qtype][0] == "Q2_0":  # flashnext/ref_fn.py:46-52
        blk = raw.reshape(-1, 18)
        d = blk[:, :2].copy().view(np.float16).astype(np.float64)
        qs = blk[:, 2:]
        q = np.stack([(qs >> s) & 3 for s in (0, 2, 4, 6)], axis=-1).reshape(-1, 64).astype(np.float64)
        return ((q - 1.0) * d).reshape(raw.shape[0], -1)
    return quants.dequantize(raw, QT(qtype)).astype(np.float64).reshape(raw.shape[0], -1)


def main():
    rng = np.random.default_rng(20260101)
    out = {}
    for t, (name, qk, tb) in sorted(TYPES.items()):
        cols = 512
        raw = random_blocks(t, 4, cols, rng)
        out[f"{name}/raw"] = raw
        val = ref_dequant(raw, t)
        out[f"{name}/out"] = val.astype(np.float32)
        assert np.array_equal(val.astype(np.float32).astype(np.float64), val), name
        x = rng.standard_normal((2, cols), dtype=np.float32)
        out[f"{name}/x"] = x
        out[f"{name}/y64"] = x.astype(np.float64) @ val.T
        if name != "BF16":
            xr = random_blocks(t, len(EXTREME), cols, rng).reshape(len(EXTREME), -1, tb)
            for i, e in enumerate(EXTREME):
                for off in SCALE_OFFSETS[name]:
                    xr[i, :, off:off + 2] = np.frombuffer(e.tobytes(), np.uint8)
            xr = xr.reshape(len(EXTREME), row_bytes(t, cols))
            xv = ref_dequant(xr, t)
            assert np.isfinite(xv).all(), name
            out[f"{name}/xraw"] = xr
            out[f"{name}/xout"] = xv.astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "dequant_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "dequant_golden.npz"), len(out), "arrays")


if __name__ == "__main__":
    main()
