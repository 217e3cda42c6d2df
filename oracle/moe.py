"""CPU oracle for the MoE layer (routing, routed SwiGLU experts, gated shared expert).  TEST INFRASTRUCTURE ONLY.

Float64 restatement of the reference's MoE arithmetic for one decode token:
  routing   engine/faie2fn.cu:1742-1800 (k_route): v = expf(l - max l) in float32 over the ne router logits, the k
            experts of largest v (equal v to the lower expert index), weights v / (sum of the k v's)
  experts   engine/faie2fn.cu:1082-1184 (k_tmoe_gu8, k_tmoe_down): act = silu(gate_e . x) * (up_e . x),
            d_e = down_e . act
  shared    engine/faie2fn.cu:2411-2416 and the swiglu of k_route (:1758-1759): sh = down_s . (silu(gate_s . x) * (up_s . x))
  combine   engine/faie2fn.cu:1299-1318 (k_hc_add): y = sum_s w_s d_{sel_s} (slot order) + sigmoid(g) sh, where g is
            the shared-gate logit (row ne of the stacked router + shared-gate GEMV output)
The same semantics are cross-checked in the CPU test-suite against transformers 5.5.0 Qwen3NextSparseMoeBlock
(modeling_qwen3_next.py:722-802) in float64.
Weights are GGUF rows; only the selected experts are dequantised (oracle.dequant, bit-exact fp32 values).
"""

from __future__ import annotations

import numpy as np

from . import dequant as D


def route(logits: np.ndarray, k: int):
    """Top-k of one token's router logits (ne,), following k_route (engine/faie2fn.cu:1747-1800) step by step in
    float32: m = max l; v_i = exp(l_i - m), the difference rounded to float32 and the exponential to the nearest
    float32 (computed in float64, then rounded); the k largest v, equal v to the lower index; s = the k v's summed in
    rank order in float32; w = v / s in float32. Returns sel (int64 [k]) and w (float32 [k]).

    The engine calls CUDA's expf, whose result may differ from the nearest float32 by an ulp; this oracle does not
    model that library. Distinct logits tie exactly where their v's are equal whatever the exponential's rounding:
    equal differences l - m, and results that saturate at 0 (underflow) or 1 (l - m above -2**-25)."""
    l = np.asarray(logits, np.float32)
    m = np.float32(l.max())
    d = (l - m).astype(np.float32)
    v = np.exp(d.astype(np.float64)).astype(np.float32)
    order = np.lexsort((np.arange(l.size), -v.astype(np.float64)))
    sel = order[:k]
    s = np.float32(0.0)
    for i in sel:
        s = np.float32(s + v[i])
    return sel.astype(np.int64), (v[sel] / s).astype(np.float32)


def silu(v):
    return v / (1.0 + np.exp(-v))


def sigmoid(v):
    return 1.0 / (1.0 + np.exp(-v))


class GGUFExperts:
    """Expert-stacked GGUF rows (ne * rows_per_expert rows) with lazy per-expert dequantisation; the most recently
    used `keep` experts stay dequantised (float64)."""

    def __init__(self, raw: np.ndarray, qtype: int, rows_per_expert: int, cols: int, keep: int = 64):
        self.raw, self.qtype, self.rpe, self.cols, self.keep = raw, qtype, rows_per_expert, cols, keep
        self.cache = {}

    def __getitem__(self, e: int) -> np.ndarray:
        if e in self.cache:
            self.cache[e] = self.cache.pop(e)  # most recent last
        else:
            rows = self.raw[e * self.rpe:(e + 1) * self.rpe]
            self.cache[e] = D.dequant_rows(rows, self.qtype, self.rpe, self.cols).astype(np.float64)
            while len(self.cache) > self.keep:
                self.cache.pop(next(iter(self.cache)))
        return self.cache[e]


def moe_layer(x, logits, k, gate, up, down, sh_gate, sh_up, sh_down):
    """x [nt][d] (fp32), logits [nt][ne + 1]; gate/up/down: GGUFExperts (or arrays indexable by expert id);
    sh_*: float64 matrices. Returns y [nt][d] float64, sel [nt][k], w [nt][k]."""
    x = np.asarray(x, np.float64)
    nt, ne = x.shape[0], logits.shape[1] - 1
    y = np.zeros_like(x)
    sels, ws = [], []
    for t in range(nt):
        sel, w = route(logits[t, :ne], k)
        acc = np.zeros(x.shape[1])
        for s, e in enumerate(sel):
            act = silu(gate[e] @ x[t]) * (up[e] @ x[t])
            acc += w[s] * (down[e] @ act)
        sh = sh_down @ (silu(sh_gate @ x[t]) * (sh_up @ x[t]))
        y[t] = acc + sigmoid(float(logits[t, ne])) * sh
        sels.append(sel)
        ws.append(w)
    return y, np.array(sels), np.array(ws)
