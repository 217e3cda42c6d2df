"""The reference's own CPU path for the dequant-GEMV, restated.  TEST / BASELINE INFRASTRUCTURE ONLY.

Used only by bench.py's CPU-baseline legs (`cpu_baseline`, and `--impl reference`) and by tests.

The reference checks and baselines its GEMV against float64 numpy on weights dequantised by gguf-py:
flashnext/ref_fn.py:44-53 (`dequant`: gguf-py `quants.dequantize` for ggml formats, its own restatement for Q2_0)
and flashnext/test_fn_quants.py:30-34 (`ref = dequant(...)`, `yref = x.astype(np.float64) @ ref.T`). ref_fn.py itself
cannot be imported here (it needs transformers.models.qwen4_exp, an unshipped faie2.gguf_reader and the model's GGUF
shards, ref_fn.py:17-31), so `dequant` below restates it, on gguf-py 0.19.0.
"""

from __future__ import annotations

import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def dequant(data: np.ndarray, qtype: int) -> np.ndarray:
    """flashnext/ref_fn.py:44-53: GGUF rows -> float64 values."""
    data = np.asarray(data)
    if qtype == 42:  # Q2_0: 64 values, fp16 d, 2-bit codes, value = (q - 1) * d
        lead = data.shape[:-1]
        blk = data.reshape(-1, 18)
        d = blk[:, :2].copy().view(np.float16).astype(np.float64)
        qs = blk[:, 2:]
        q = np.stack([(qs >> s) & 3 for s in (0, 2, 4, 6)], axis=-1).reshape(-1, 64).astype(np.float64)
        return ((q - 1.0) * d).reshape(*lead, -1)
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as QT
    return quants.dequantize(data, QT(qtype)).astype(np.float64)


def gemv(raw: np.ndarray, qtype: int, x: np.ndarray) -> np.ndarray:
    """flashnext/test_fn_quants.py:30-34: y = x(float64) . dequant(W)^T."""
    return np.asarray(x, np.float64) @ dequant(raw, qtype).T


# ---- a bounded sample of a GEMV workload, timed on host cores -------------------------------------------------

_SAMPLE = None


def _make_sample(work, row_fraction, seed):
    sys.path.insert(0, os.path.join(HERE, "..", "faie2-flashnext_b200", "flashnext"))
    from synth import random_blocks, random_x
    out = []
    for i, (q, r, c) in enumerate(work):
        rng = np.random.default_rng(seed + i)
        n = max(1, int(np.ceil(r * row_fraction)))
        out.append((q, random_blocks(q, n, c, rng), random_x(1, c, rng)))
    return out


def _init_worker(work, row_fraction, seed):
    global _SAMPLE
    _SAMPLE = _make_sample(work, row_fraction, seed)


def _run_task(i):
    q, raw, x = _SAMPLE[i]
    return float(gemv(raw, q, x).sum())


class CPUSweep:
    """The workload [(qtype, rows, cols)] with each GEMV cut to ceil(rows * row_fraction) rows; step() runs it once
    on `workers` processes (spawned; one BLAS thread each) and returns the wall seconds. bytes = GGUF weight bytes
    of the sample."""

    def __init__(self, work, row_fraction: float, workers: int = 1, seed: int = 0):
        self.work, self.frac, self.workers = list(work), row_fraction, max(1, workers)
        self.pool = None
        if self.workers == 1:
            _init_worker(self.work, row_fraction, seed)
            self.sample = _SAMPLE
        else:
            import multiprocessing as mp
            os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
            os.environ.setdefault("OMP_NUM_THREADS", "1")
            self.pool = mp.get_context("spawn").Pool(self.workers, _init_worker, (self.work, row_fraction, seed))
            self.sample = _make_sample(self.work, row_fraction, seed)
        self.bytes = sum(raw.nbytes for _, raw, _ in self.sample)

    def step(self) -> float:
        t0 = time.perf_counter()
        if self.pool is None:
            from threadpoolctl import threadpool_limits
            with threadpool_limits(1):
                for i in range(len(self.sample)):
                    _run_task(i)
        else:
            self.pool.map(_run_task, range(len(self.sample)), chunksize=1)
        return time.perf_counter() - t0

    def close(self):
        if self.pool is not None:
            self.pool.close()
            self.pool.join()
