"""CPU oracle for the gated-DeltaNet decode core.  TEST INFRASTRUCTURE ONLY.

Float64 restatement of k_gdn (engine/faie2fn.cu:1349-1431) for one layer, token by token:
  conv     causal depthwise conv, kernel 4, over [3 previous inputs, current input] of every q / k / v channel, then
           silu (faie2fn.cu:1395-1400); the conv state keeps the last 3 inputs per channel
  l2norm   q, k of every key head: x / sqrt(sum x^2 + 1e-6) (:1401-1404)
  gates    beta = sigmoid(b_h), g = ssm_a_h * softplus(a_h + dt_bias_h) with softplus(u) = u for u > 20,
           ssm_a = -exp(A_log) (:1409-1412); decay = exp(g)
  delta    kv = S^T k; delta = (v - decay kv) * beta; S = decay S + k delta^T; o = S^T q / sqrt(128) (:1413-1421)
  norm     out = o / sqrt(mean(o^2) + 1e-6) * w * sigmoid(z) (:1422-1425)
Value head h reads key head h % NKH (the GGUF tiled head order, faie2fn.cu:10-11, 1374). The same recurrence is
cross-checked in the CPU test-suite against transformers 5.5.0 torch_recurrent_gated_delta_rule and
torch_causal_conv1d_update (modeling_qwen3_next.py:350-366, 454-495), which differ only in conventions (head
grouping h // (nv / nk) and a silu(z) gate in the norm), mapped there explicitly.

Shapes: qkv [CONVCH] = [q (NKH*DS) | k (NKH*DS) | v (NVH*DS)], z [NVH*DS], ab [2*NVH] = [alpha | beta];
conv_w [CONVCH][4] (taps for the oldest .. current input); S [NVH][DS][DS] with S[h][i][j] (i: key dim, j: value dim);
conv_state [3][CONVCH] (oldest first).
"""

from __future__ import annotations

import numpy as np


def silu(v):
    return v / (1.0 + np.exp(-v))


def sigmoid(v):
    return 1.0 / (1.0 + np.exp(-v))


def softplus20(u):
    return np.where(u > 20.0, u, np.log1p(np.exp(np.minimum(u, 20.0))))


def gdn_step(qkv, z, ab, conv_w, dt_bias, ssm_a, norm_w, S, conv_state, nkh, nvh, ds=128, eps=1e-6):
    """One token. Updates S and conv_state in place (float64 arrays); returns out [NVH*DS] float64."""
    qkv = np.asarray(qkv, np.float64)
    win = np.concatenate([conv_state, qkv[None]], axis=0)  # [4][CONVCH], oldest first
    x = silu((win.T * conv_w).sum(axis=1))
    conv_state[:] = win[1:]
    q = x[:nkh * ds].reshape(nkh, ds)
    k = x[nkh * ds:2 * nkh * ds].reshape(nkh, ds)
    v = x[2 * nkh * ds:].reshape(nvh, ds)
    q = q / np.sqrt((q * q).sum(axis=1, keepdims=True) + 1e-6)
    k = k / np.sqrt((k * k).sum(axis=1, keepdims=True) + 1e-6)
    ab = np.asarray(ab, np.float64)
    beta = sigmoid(ab[nvh:2 * nvh])
    decay = np.exp(np.asarray(ssm_a, np.float64) * softplus20(ab[:nvh] + np.asarray(dt_bias, np.float64)))
    out = np.empty((nvh, ds))
    zz = np.asarray(z, np.float64).reshape(nvh, ds)
    for h in range(nvh):
        kh = h % nkh
        Sh = S[h]
        kv = Sh.T @ k[kh]
        delta = (v[h] - decay[h] * kv) * beta[h]
        Sh *= decay[h]
        Sh += np.outer(k[kh], delta)
        o = (Sh.T @ q[kh]) / np.sqrt(ds)
        out[h] = o / np.sqrt((o * o).mean() + eps) * np.asarray(norm_w, np.float64) * sigmoid(zz[h])
    return out.reshape(-1)


def gdn_run(qkv, z, ab, conv_w, dt_bias, ssm_a, norm_w, S0, conv0, nkh, nvh, ds=128):
    """nt tokens: returns out [nt][NVH*DS], final S, final conv state (float64)."""
    S = np.array(S0, np.float64, copy=True)
    cs = np.array(conv0, np.float64, copy=True)
    outs = [gdn_step(qkv[t], z[t], ab[t], conv_w, dt_bias, ssm_a, norm_w, S, cs, nkh, nvh, ds) for t in range(len(qkv))]
    return np.array(outs), S, cs
