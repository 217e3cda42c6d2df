"""GPU parity of routing and the MoE layer through the C ABI.

Routing: the reference's KAT (flashnext/route_fn.py:29-47: 200 random router outputs with forced ties, ks split-K
partials summed in split order): the engine's routing (variant 1) is bit-identical to the reference's order counted
out expert by expert (variant 0, k_route_ref's role), its selection equals the CPU oracle's and its weights are
within 1e-6 relative (the CPU rounds exp from float64, the GPU calls expf); and router outputs where distinct logits
share one float32 probability select the hand-derived experts (equal v to the lower index, not the larger logit). MoE layer (and small shapes):
max |y - y64| / max |y64| <= 1e-5 against the float64 oracle on the exactly dequantised weights (the reference's own
GEMV gate bar, flashnext/test_fn_quants.py:37), routing identical; one token's output is bit-identical alone and
inside a batch.
"""

import numpy as np
import pytest

from oracle import moe as M
from oracle import dequant as D
from synth import BY_NAME, random_blocks, random_x

pytestmark = pytest.mark.gpu
MOE_TOL = 1e-5


def make_moe(rng, gu, dn, ne, ffe, d, scale_gu=1e-3, scale_dn=1e-3):
    Wg = random_blocks(gu, ne * ffe, d, rng, scale_gu)
    Wu = random_blocks(gu, ne * ffe, d, rng, scale_gu)
    Wd = random_blocks(dn, ne * d, ffe, rng, scale_dn)
    Wsg = random_blocks(gu, ffe, d, rng, scale_gu)
    Wsu = random_blocks(gu, ffe, d, rng, scale_gu)
    Wsd = random_blocks(dn, d, ffe, rng, scale_dn)
    return Wg, Wu, Wd, Wsg, Wsu, Wsd


def oracle(gu, dn, ne, k, ffe, d, W, logits, x):
    Wg, Wu, Wd, Wsg, Wsu, Wsd = W
    return M.moe_layer(x, logits, k, M.GGUFExperts(Wg, gu, ffe, d), M.GGUFExperts(Wu, gu, ffe, d),
                       M.GGUFExperts(Wd, dn, d, ffe),
                       D.dequant_rows(Wsg, gu, ffe, d).astype(np.float64), D.dequant_rows(Wsu, gu, ffe, d).astype(np.float64),
                       D.dequant_rows(Wsd, dn, d, ffe).astype(np.float64))


def check(fn, gu, dn, ne, k, ffe, d, nt, seed, logit_scale=2.0):
    rng = np.random.default_rng(seed)
    W = make_moe(rng, gu, dn, ne, ffe, d)
    x = random_x(nt, d, rng)
    logits = (rng.standard_normal((nt, ne + 1)) * logit_scale).astype(np.float32)
    y, sel, w = fn.moe(gu, dn, ne, k, ffe, d, *W, logits, x)
    y64, sel64, w64 = oracle(gu, dn, ne, k, ffe, d, W, logits, x)
    assert np.array_equal(sel, sel64)
    assert np.allclose(w, w64, rtol=1e-6, atol=0)
    err = float(np.abs(y - y64).max() / np.abs(y64).max())
    assert err <= MOE_TOL, f"moe rel err {err:.3e}"
    return y, W, logits, x


def test_moe_config3(fn):
    """512 experts, top-10, width 512, hidden 2048, IQ3_XXS gate/up, Q4_K down, logits N(0, 2)."""
    check(fn, BY_NAME["IQ3_XXS"], BY_NAME["Q4_K"], 512, 10, 512, 2048, 1, seed=3)


@pytest.mark.parametrize("gu,dn", [("Q4_K", "Q6_K"), ("IQ2_XXS", "Q8_0"), ("Q8_0", "IQ4_XS"), ("BF16", "Q5_K")])
@pytest.mark.parametrize("nt", [1, 3])
def test_moe_small(fn, gu, dn, nt):
    check(fn, BY_NAME[gu], BY_NAME[dn], 24, 4, 256, 512, nt, seed=nt * 7 + len(gu))


@pytest.mark.parametrize("nt", [9, 17, 32])
def test_moe_batched_tokens(fn, nt):
    """More than 8 tokens per call (batched decode, up to 32): the gate/up warps move through several tokens' units."""
    check(fn, BY_NAME["IQ3_XXS"], BY_NAME["Q4_K"], 64, 10, 512, 2048, nt, seed=nt)


@pytest.mark.parametrize("ne,k,nt", [(700, 8, 1), (1024, 16, 2), (513, 10, 1)])
def test_moe_many_experts(fn, ne, k, nt):
    """More than 512 experts (two logits per routing lane), the largest k, and an expert count that is not a multiple
    of the routing warps' share."""
    check(fn, BY_NAME["Q4_K"], BY_NAME["Q4_K"], ne, k, 256, 512, nt, seed=ne + k)


def test_moe_batch_invariance(fn):
    gu, dn, ne, k, ffe, d = BY_NAME["IQ3_XXS"], BY_NAME["Q4_K"], 32, 6, 256, 2048
    y4, W, logits, x = check(fn, gu, dn, ne, k, ffe, d, 4, seed=11)
    for t in (0, 3):
        y1, _, _ = fn.moe(gu, dn, ne, k, ffe, d, *W, logits[t:t + 1], x[t:t + 1])
        assert np.array_equal(y1[0].view(np.uint32), y4[t].view(np.uint32))


def test_moe_shared_gate_extremes(fn):
    """sigmoid of a very negative / positive shared-gate logit switches the shared expert off / fully on."""
    gu, dn, ne, k, ffe, d = BY_NAME["Q4_K"], BY_NAME["Q4_K"], 16, 2, 256, 256
    rng = np.random.default_rng(5)
    W = make_moe(rng, gu, dn, ne, ffe, d)
    x = random_x(2, d, rng)
    logits = rng.standard_normal((2, ne + 1)).astype(np.float32)
    logits[0, ne], logits[1, ne] = -80.0, 80.0
    y, _, _ = fn.moe(gu, dn, ne, k, ffe, d, *W, logits, x)
    y64, _, _ = oracle(gu, dn, ne, k, ffe, d, W, logits, x)
    assert np.abs(y - y64).max() <= MOE_TOL * np.abs(y64).max()


def test_moe_errors(fn):
    z = np.zeros(1, np.uint8)
    with pytest.raises(RuntimeError):  # k > 16
        fn.moe(12, 12, 32, 20, 256, 256, z, z, z, z, z, z, np.zeros((1, 33), np.float32), np.zeros((1, 256), np.float32))


# ---- routing KAT (flashnext/route_fn.py) -------------------------------------------------------------------------

RSG, MAXT, NEU = 528, 8, 10


def test_route_kat_200_cases(fn):
    rng = np.random.default_rng(1)
    for trial in range(200):
        ks = int(rng.integers(1, 6))
        nt = int(rng.integers(1, 9))
        part = (rng.standard_normal((ks, MAXT, RSG)) * rng.choice([0.1, 1, 4])).astype(np.float32)
        if trial % 3 == 0:  # ties: copy some logits onto others (one split, so the sums tie exactly)
            part[1:] = 0
            for t in range(nt):
                src = rng.integers(0, 512, 20)
                dst = rng.integers(0, 512, 20)
                part[0, t, dst] = part[0, t, src]
        if trial % 7 == 0:  # many exact ties
            part[:, :, :512] = np.round(part[:, :, :512])
        sel0, w0, _ = fn.bench_route(0, part, nt, ks)
        sel, w, _ = fn.bench_route(1, part, nt, ks)
        assert np.array_equal(sel0, sel) and np.array_equal(w0.view(np.uint32), w.view(np.uint32)), f"trial {trial}"
        sel, w = sel.reshape(nt, NEU), w.reshape(nt, NEU)
        for t in range(nt):
            lg = part[0, t, :512].copy()
            for j in range(1, ks):  # split order, float32, as the engine adds them
                lg = (lg + part[j, t, :512]).astype(np.float32)
            s64, w64 = M.route(lg, NEU)
            assert np.array_equal(sel[t], s64), f"trial {trial} token {t}"
            assert np.allclose(w[t], w64, rtol=1e-6, atol=0), f"trial {trial} token {t}"


def test_route_probability_collisions(fn):
    from route_cases import collision_cases
    cases = collision_cases()
    part = np.zeros((1, MAXT, RSG), np.float32)
    for t, (l, _) in enumerate(cases):
        part[0, t, :512] = l
    nt = len(cases)
    for variant in (0, 1):
        sel, w, _ = fn.bench_route(variant, part, nt, 1)
        sel, w = sel.reshape(nt, NEU), w.reshape(nt, NEU)
        for t, (l, want) in enumerate(cases):
            assert sel[t].tolist() == want, f"variant {variant} case {t}"
            _, w64 = M.route(l, NEU)
            assert np.allclose(w[t], w64, rtol=1e-6, atol=0), f"variant {variant} case {t}"


def test_route_small_logit_collisions_variants_agree(fn):
    # logits within 1e-3 of the max: many v's land on neighbouring floats just below 1, where expf's own rounding
    # decides ties; both variants call the same expf, so they must agree bit for bit
    rng = np.random.default_rng(3)
    part = (-rng.uniform(0, 1e-3, (1, MAXT, RSG))).astype(np.float32)
    s0, w0, _ = fn.bench_route(0, part, MAXT, 1)
    s1, w1, _ = fn.bench_route(1, part, MAXT, 1)
    assert np.array_equal(s0, s1) and np.array_equal(w0.view(np.uint32), w1.view(np.uint32))


# ---- the fused single-kernel layer (fn_moe_var(2): gate/up and down with per-slot counters) ----------------------
@pytest.mark.parametrize("gu,dn,ne,k,ffe,d", [("IQ3_XXS", "Q4_K", 512, 10, 512, 2048), ("IQ3_XXS", "Q4_K", 16, 4, 256, 512),
                                              ("Q4_K", "Q4_K", 64, 8, 512, 1024), ("IQ2_XXS", "Q4_K", 32, 6, 256, 2048),
                                              ("Q4_K", "Q6_K", 32, 4, 512, 2048)])
def test_moe_fused_bit_identical(fn, gu, dn, ne, k, ffe, d):
    """One token: the fused kernel's output equals the two-kernel layer's bit for bit (the same arithmetic in the same
    order), over several calls in a row (the counters are zeroed by each call's last CTA), and stays within the
    float64 bar."""
    rng = np.random.default_rng(ne + ffe + d)
    gq, dq = BY_NAME[gu], BY_NAME[dn]
    W = make_moe(rng, gq, dq, ne, ffe, d)
    outs = {}
    try:
        for var in (0, 2):
            fn.moe_var(var)
            rng2 = np.random.default_rng(5)
            outs[var] = []
            for _ in range(3):
                lg = (rng2.standard_normal((1, ne + 1)) * 2).astype(np.float32)
                x = random_x(1, d, rng2)
                y, sel, w = fn.moe(gq, dq, ne, k, ffe, d, *W, lg, x)
                outs[var].append((y, sel, w, lg, x))
    finally:
        fn.moe_var(0)
    for (y0, s0, w0, lg, x), (y2, s2, w2, _, _) in zip(outs[0], outs[2]):
        assert np.array_equal(s0, s2) and np.array_equal(w0.view(np.uint32), w2.view(np.uint32))
        assert np.array_equal(y0.view(np.uint32), y2.view(np.uint32))
        y64, _, _ = oracle(gq, dq, ne, k, ffe, d, W, lg, x)
        assert np.abs(y2 - y64).max() <= MOE_TOL * np.abs(y64).max()


def test_moe_fused_repeated_calls_on_one_handle(fn):
    """Config 3 through one resident handle, five calls in a row with different tokens: the fused layer (whose last CTA
    zeroes the per-slot counters for the next call) matches the two-kernel layer bit for bit on every call."""
    import torch
    gq, dq, ne, k, ffe, d = BY_NAME["IQ3_XXS"], BY_NAME["Q4_K"], 512, 10, 512, 2048
    rng = np.random.default_rng(41)
    W = make_moe(rng, gq, dq, ne, ffe, d)
    h = fn.moe_create(gq, dq, ne, k, ffe, d, *W)
    dev = torch.device("cuda", 0)
    lg = torch.from_numpy((rng.standard_normal((5, ne + 1)) * 2).astype(np.float32)).to(dev)
    x = torch.from_numpy(random_x(5, d, rng)).to(dev)
    ys = {}
    try:
        for var in (0, 2):
            fn.moe_var(var)
            y = torch.zeros(5, d, device=dev)
            for i in range(5):
                fn.moe_run(h, lg[i].data_ptr(), ne + 1, x[i].data_ptr(), y[i].data_ptr(), 1, 0, 0)
            fn.sync()
            ys[var] = y.cpu().numpy()
    finally:
        fn.moe_var(0)
        fn.moe_free(h)
    assert np.array_equal(ys[0].view(np.uint32), ys[2].view(np.uint32))
