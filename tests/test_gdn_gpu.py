"""GPU parity of the gated-DeltaNet core and of the BASELINE config-4 decode step, through the C ABI.

The reference checks its DeltaNet against a float64 oracle of the whole model (flashnext/gate_fn_ref.py: residual rel
err per layer, |dlogprob| < 0.05); here the core and the layer step are checked against oracle/gdn.py (float64,
itself pinned to transformers' recurrence on the CPU). Bars: per-token outputs max|out - out64| / max|out64| <= 1e-4
and the final state max|S - S64| / max|S64| <= 1e-4 after the run (fp32 recurrence vs float64); results do not depend
on how many tokens one launch covers.
"""

import numpy as np
import pytest

from oracle import dequant as D
from oracle import gdn as G
from synth import BY_NAME, random_blocks, random_x

pytestmark = pytest.mark.gpu
NKH, NVH, DS = 16, 32, 128
CONVCH = 2 * NKH * DS + NVH * DS
TOL = 1e-4


def params(rng):
    conv_w = (rng.standard_normal((CONVCH, 4)) * 0.5).astype(np.float32)
    dt_bias = (rng.standard_normal(NVH) * 0.5).astype(np.float32)
    ssm_a = (-np.exp(rng.standard_normal(NVH) * 0.5)).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(DS)).astype(np.float32)
    S0 = (rng.standard_normal((NVH, DS, DS)) * 0.02).astype(np.float32)  # N(0, 0.02)
    c0 = rng.standard_normal((3, CONVCH)).astype(np.float32)
    return conv_w, dt_bias, ssm_a, norm_w, S0, c0


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


@pytest.mark.parametrize("tpl", [1, 8])
def test_gdn_core_vs_oracle(fn, tpl):
    rng = np.random.default_rng(4)
    conv_w, dt_bias, ssm_a, norm_w, S0, c0 = params(rng)
    nt = 48
    qkv = rng.standard_normal((nt, CONVCH)).astype(np.float32)
    z = rng.standard_normal((nt, NVH * DS)).astype(np.float32)
    ab = rng.standard_normal((nt, 2 * NVH)).astype(np.float32)
    out, S, cs = fn.gdn(NKH, NVH, qkv, z, ab, conv_w, dt_bias, ssm_a, norm_w, S0, c0, tokens_per_launch=tpl)
    out64, S64, cs64 = G.gdn_run(qkv, z, ab, conv_w, dt_bias, ssm_a, norm_w, S0, c0, NKH, NVH, DS)
    assert rel(out, out64) <= TOL
    assert rel(S, S64) <= TOL
    assert np.array_equal(cs, cs64.astype(np.float32))  # the conv history is the inputs themselves


def test_gdn_launch_size_invariance(fn):
    rng = np.random.default_rng(9)
    conv_w, dt_bias, ssm_a, norm_w, S0, c0 = params(rng)
    nt = 16
    qkv = rng.standard_normal((nt, CONVCH)).astype(np.float32)
    z = rng.standard_normal((nt, NVH * DS)).astype(np.float32)
    ab = rng.standard_normal((nt, 2 * NVH)).astype(np.float32)
    a = fn.gdn(NKH, NVH, qkv, z, ab, conv_w, dt_bias, ssm_a, norm_w, S0, c0, tokens_per_launch=1)
    b = fn.gdn(NKH, NVH, qkv, z, ab, conv_w, dt_bias, ssm_a, norm_w, S0, c0, tokens_per_launch=16)
    for u, v in zip(a, b):
        assert np.array_equal(u.view(np.uint32), v.view(np.uint32))


def test_gdn_softplus_threshold_and_saturated_gates(fn):
    """alpha + dt_bias far above 20 (softplus(u) = u branch), far below (decay -> 1), beta saturated."""
    rng = np.random.default_rng(2)
    conv_w, dt_bias, ssm_a, norm_w, S0, c0 = params(rng)
    nt = 6
    qkv = rng.standard_normal((nt, CONVCH)).astype(np.float32)
    z = rng.standard_normal((nt, NVH * DS)).astype(np.float32)
    ab = np.zeros((nt, 2 * NVH), np.float32)
    ab[:, :NVH] = np.array([30.0, -30.0, 19.99, 20.01] * (NVH // 4), np.float32)
    ab[:, NVH:] = np.array([40.0, -40.0] * (NVH // 2), np.float32)
    out, S, _ = fn.gdn(NKH, NVH, qkv, z, ab, conv_w, dt_bias * 0, ssm_a, norm_w, S0, c0)
    out64, S64, _ = G.gdn_run(qkv, z, ab, conv_w, dt_bias * 0, ssm_a, norm_w, S0, c0, NKH, NVH, DS)
    assert rel(out, out64) <= TOL and rel(S, S64) <= TOL


def test_gdn_config4_decode_1024_steps(fn):
    """Q5_K in-projection 2048 -> 8192 (qkv) + 4096 (z), Q8_0 alpha/beta 2048 -> 64, the core, Q5_K
    out-projection 4096 -> 2048; 1024 sequential one-token steps from seed, all on the device."""
    import torch
    rng = np.random.default_rng(44)
    d = 2048
    q5, q8 = BY_NAME["Q5_K"], BY_NAME["Q8_0"]
    w_in = random_blocks(q5, CONVCH + NVH * DS, d, rng)
    w_ab = random_blocks(q8, 2 * NVH, d, rng)
    w_out = random_blocks(q5, d, NVH * DS, rng)
    conv_w, dt_bias, ssm_a, norm_w, S0, c0 = params(rng)
    steps = 1024
    xs = random_x(steps, d, rng)
    dev = torch.device("cuda", 0)
    h_in, h_ab, h_out = fn.w_create(q5, w_in, CONVCH + NVH * DS, d), fn.w_create(q8, w_ab, 2 * NVH, d), \
        fn.w_create(q5, w_out, d, NVH * DS)
    hg = fn.gdn_create(NKH, NVH, conv_w, dt_bias, ssm_a, norm_w, S0, c0)
    x_d = torch.from_numpy(xs).to(dev)
    qkvz = torch.empty(CONVCH + NVH * DS, device=dev)
    ab = torch.empty(2 * NVH, device=dev)
    core = torch.empty(NVH * DS, device=dev)
    y = torch.empty(steps, d, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    try:
        for t in range(steps):
            xp = x_d[t].data_ptr()
            fn.w_gemv(h_in, xp, d, qkvz.data_ptr(), CONVCH + NVH * DS, 1, 0, st)
            fn.w_gemv(h_ab, xp, d, ab.data_ptr(), 2 * NVH, 1, 0, st)
            # the previous step's core launch is 4 kernels back, so its state may be read before the wait
            fn.gdn_run(hg, qkvz.data_ptr(), CONVCH, qkvz.data_ptr() + 4 * CONVCH, NVH * DS, ab.data_ptr(), 2 * NVH,
                       core.data_ptr(), NVH * DS, 1, 1, st)
            fn.w_gemv(h_out, core.data_ptr(), NVH * DS, y[t].data_ptr(), d, 1, 0, st)
        fn.sync(st)
        y_gpu = y.cpu().numpy()
        S_gpu, _ = fn.gdn_state(hg, NKH, NVH)
    finally:
        for h in (h_in, h_ab, h_out):
            fn.w_free(h)
        fn.gdn_free(hg)
    W_in = D.dequant_rows(w_in, q5, CONVCH + NVH * DS, d).astype(np.float64)
    W_ab = D.dequant_rows(w_ab, q8, 2 * NVH, d).astype(np.float64)
    W_out = D.dequant_rows(w_out, q5, d, NVH * DS).astype(np.float64)
    S = S0.astype(np.float64)
    cs = c0.astype(np.float64)
    y64 = np.empty((steps, d))
    for t in range(steps):
        v = W_in @ xs[t].astype(np.float64)
        o = G.gdn_step(v[:CONVCH], v[CONVCH:], W_ab @ xs[t].astype(np.float64), conv_w, dt_bias, ssm_a, norm_w, S, cs,
                       NKH, NVH, DS)
        y64[t] = W_out @ o
    assert rel(y_gpu, y64) <= TOL, f"layer output rel err {rel(y_gpu, y64):.3e}"
    assert rel(S_gpu, S) <= TOL, f"state rel err {rel(S_gpu, S):.3e}"
