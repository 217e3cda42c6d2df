"""One-GPU runs of the multi-GPU data paths (a peer group of one rank): the row-split lm_head's key publish + combine
and the expert-parallel MoE's slot-output publish + combine go through the same kernels and counters as on n GPUs
(stores into the group buffer, release counts, bounded waits), so the single-GPU suite covers them. Bars: the
index equals the oracle argmax of the one-GPU logits; the expert-parallel layer is bit-identical to the one-GPU
layer. The n-GPU versions run in tests/test_mgpu.py."""

import numpy as np
import pytest

from oracle.argmax import argmax_fast
from parallel import LmHeadSplit, PeerGroup
from synth import BY_NAME, random_blocks, random_x

pytestmark = pytest.mark.gpu


@pytest.fixture
def group(fn):
    g = PeerGroup(fn, 0, 1, lambda obj: [obj], lambda: None)
    yield g
    g.close()


def test_lm_head_group_of_one(fn, group):
    import torch
    q, V, cols = BY_NAME["Q6_K"], 30011, 2048
    rng = np.random.default_rng(8)
    raw = random_blocks(q, V, cols, rng)
    xs = random_x(8, cols, rng)
    y_full = np.concatenate([fn.gemv(q, raw, V, cols, xs[i:i + 4]) for i in (0, 4)])
    want = argmax_fast(y_full)
    head = LmHeadSplit(fn, group, q, raw, V, cols)
    try:
        st = torch.cuda.current_stream().cuda_stream
        x_d = torch.from_numpy(xs).cuda()
        idx = torch.full((8,), -2, dtype=torch.int32, device="cuda")
        y = torch.empty((8, V), device="cuda")
        for i in range(5):
            head.run(x_d[i].data_ptr(), cols, idx.data_ptr(), 1, y.data_ptr(), 0, st)
            fn.sync(st)
            assert int(idx[0]) == int(want[i])
            assert np.array_equal(y[0].cpu().numpy().view(np.uint32), y_full[i].view(np.uint32))
        head.run(x_d[5].data_ptr(), cols, idx.data_ptr(), 3, 0, 0, st)
        fn.sync(st)
        assert np.array_equal(idx[:3].cpu().numpy(), want[5:8])
    finally:
        head.close()


def test_moe_expert_parallel_group_of_one(fn, group):
    import torch
    gu, dn, ne, k, ffe, d = BY_NAME["IQ3_XXS"], BY_NAME["Q4_K"], 64, 10, 512, 2048
    rng = np.random.default_rng(9)
    Wg, Wu = random_blocks(gu, ne * ffe, d, rng), random_blocks(gu, ne * ffe, d, rng)
    Wd = random_blocks(dn, ne * d, ffe, rng)
    Wsg, Wsu, Wsd = random_blocks(gu, ffe, d, rng), random_blocks(gu, ffe, d, rng), random_blocks(dn, d, ffe, rng)
    h_ep = fn.moe_ep_create(gu, dn, ne, k, ffe, d, group.id, Wg, Wu, Wd, Wsg, Wsu, Wsd)
    h_one = fn.moe_create(gu, dn, ne, k, ffe, d, Wg, Wu, Wd, Wsg, Wsu, Wsd)
    try:
        with pytest.raises(RuntimeError):  # an expert-parallel handle is not a one-GPU handle
            fn.moe_run(h_ep, 0, ne + 1, 0, 0, 1, 0, 0)
        st = torch.cuda.current_stream().cuda_stream
        xs = torch.from_numpy(random_x(8, d, rng)).cuda()
        lg = torch.from_numpy((rng.standard_normal((8, ne + 1)) * 2).astype(np.float32)).cuda()
        a, b = torch.zeros((8, d), device="cuda"), torch.zeros((8, d), device="cuda")
        for i in range(4):
            fn.moe_ep_run(h_ep, lg[i].data_ptr(), ne + 1, xs[i].data_ptr(), a.data_ptr(), 1, 0, st)
            fn.moe_run(h_one, lg[i].data_ptr(), ne + 1, xs[i].data_ptr(), b.data_ptr(), 1, 0, st)
            fn.sync(st)
            assert np.array_equal(a[0].cpu().numpy().view(np.uint32), b[0].cpu().numpy().view(np.uint32))
        fn.moe_ep_run(h_ep, lg[4].data_ptr(), ne + 1, xs[4].data_ptr(), a.data_ptr(), 3, 0, st)
        fn.moe_run(h_one, lg[4].data_ptr(), ne + 1, xs[4].data_ptr(), b.data_ptr(), 3, 0, st)
        fn.sync(st)
        assert np.array_equal(a[:3].cpu().numpy().view(np.uint32), b[:3].cpu().numpy().view(np.uint32))
    finally:
        fn.moe_free(h_ep)
        fn.moe_free(h_one)
