"""CPU: the MoE oracle's semantics are pinned against transformers' Qwen3NextSparseMoeBlock (float64), and its
routing against the reference's KAT cases (ties forced by copying and rounding logits, flashnext/route_fn.py:29-40)
and against hand-derived selections where distinct logits share one float32 probability (k_route's order,
engine/faie2fn.cu:1757-1785: equal v to the lower index)."""

import numpy as np
import pytest

from oracle import moe as M
from route_cases import collision_cases

torch = pytest.importorskip("torch")


def test_route_ties_lower_index():
    l = np.array([1.0, 3.0, 3.0, 2.0, 3.0, -1.0], np.float32)
    sel, w = M.route(l, 4)
    assert sel.tolist() == [1, 2, 4, 3]
    assert np.isclose(w.sum(), 1.0)
    assert w[0] == w[1] == w[2] > w[3]


def test_route_matches_softmax_topk_renorm():
    rng = np.random.default_rng(0)
    for _ in range(50):
        l = (rng.standard_normal(512) * 2).astype(np.float32)
        sel, w = M.route(l, 10)
        p = np.exp(l.astype(np.float64) - l.max())
        p /= p.sum()
        top = np.argsort(-p, kind="stable")[:10]
        assert sel.tolist() == top.tolist()
        assert w.dtype == np.float32
        assert np.allclose(w, p[top] / p[top].sum(), rtol=1e-6)


def test_route_probability_ties_go_to_lower_index():
    for l, want in collision_cases():
        sel, w = M.route(l, 10)
        assert sel.tolist() == want
        by_logit = np.lexsort((np.arange(l.size), -l.astype(np.float64)))[:10].tolist()
        assert by_logit != want  # each case separates the two orders


def test_route_weights_follow_the_reference_arithmetic():
    # v = expf(l - m) in float32, s summed in rank order from 0 in float32, w = v / s
    l = np.array([0.0, -1.0, -0.5, -3.0], np.float32)
    sel, w = M.route(l, 3)
    assert sel.tolist() == [0, 2, 1]
    v = [np.float32(np.exp(np.float64(np.float32(l[i] - np.float32(0.0))))) for i in sel]
    s = np.float32(0.0)
    for x in v:
        s = np.float32(s + x)
    assert np.array_equal(w, np.array([x / s for x in v], np.float32))


def test_moe_layer_matches_transformers_qwen3next():
    from transformers import Qwen3NextConfig
    from transformers.models.qwen3_next.modeling_qwen3_next import Qwen3NextSparseMoeBlock
    cfg = Qwen3NextConfig(hidden_size=64, num_experts=16, num_experts_per_tok=4, moe_intermediate_size=32,
                          shared_expert_intermediate_size=32, norm_topk_prob=True, hidden_act="silu")
    blk = Qwen3NextSparseMoeBlock(cfg).double()
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        for p in blk.parameters():
            p.copy_(torch.randn(p.shape, generator=g, dtype=torch.float64) * 0.2)
    x = torch.randn(3, 1, 64, generator=g, dtype=torch.float64)
    with torch.no_grad():
        want = blk(x).reshape(3, 64).numpy()
        logits = torch.nn.functional.linear(x.reshape(3, 64), blk.gate.weight).numpy()
        sg = blk.shared_expert_gate(x.reshape(3, 64)).numpy()
    gu = blk.experts.gate_up_proj.detach().numpy()
    gate, up = gu[:, :32], gu[:, 32:]
    down = blk.experts.down_proj.detach().numpy()
    lg = np.concatenate([logits, sg], axis=1)
    y, sel, w = M.moe_layer(x.reshape(3, 64).numpy(), lg, 4, gate, up, down,
                            blk.shared_expert.gate_proj.weight.detach().numpy(),
                            blk.shared_expert.up_proj.weight.detach().numpy(),
                            blk.shared_expert.down_proj.weight.detach().numpy())
    # transformers computes the router softmax in float32 (softmax(..., dtype=torch.float)), so its weights carry
    # ~1e-7 relative rounding; the selection must agree exactly
    _, _, ri = blk.gate(x.reshape(3, 64))
    assert np.array_equal(sel, ri.numpy())
    assert np.abs(y - want).max() <= 1e-6 * np.abs(want).max()
