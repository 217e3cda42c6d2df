"""GPU parity of the whole-model decode path (the reference's fn_forward, engine/faie2fn.cu:2733, with layer_forward
:2380-2447) on a small model of the config-5 structure (flashnext/synth.py model_config(small=True): 4 layers, 3 gated
DeltaNet + 1 gated attention, MoE on every layer, Q4_K / IQ3_XXS / Q6_K / BF16 weights), and of the kernels only that
path uses: embedding, RMSNorm, gated attention with RoPE and the KV cache.

Bars: the embedding row bit-exact vs the gguf-py dequantisation; RMSNorm and the rotated q / k within 2e-6 of float64
and the attention output within 1e-6 sqrt(positions) of the largest cached value (fp32 sums over the positions); the
model's log-probabilities within 1e-4 of the float64 oracle (oracle/model.py) at every step, and its greedy token ids
equal to the oracle's wherever the oracle's top two logits are more than 1e-3 apart."""

import numpy as np
import pytest

from oracle import dequant as O
from oracle.model import OracleModel, gated_attention, rmsnorm
from synth import BY_NAME, model_blocks, model_config, model_weights, rope_inv_freq

pytestmark = pytest.mark.gpu
LOGPROB_TOL = 1e-4
TIE = 1e-3


def logprobs(lg):
    lg = np.asarray(lg, np.float64)
    m = lg.max()
    return lg - m - np.log(np.exp(lg - m).sum())


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch


@pytest.fixture(scope="module")
def small(fn, torch_cuda):
    from model import DecodeModel
    cfg = model_config(small=True)
    W = model_weights(cfg, 1)
    m = DecodeModel(fn, cfg, W, max_ctx=96, logits=True)
    yield cfg, W, m
    m.free()


@pytest.mark.parametrize("name", ["Q4_K", "Q6_K", "IQ3_XXS", "BF16", "Q8_0"])
def test_embed_bit_exact(fn, torch_cuda, name):
    torch = torch_cuda
    rng = np.random.default_rng(3)
    qt, vocab, d = BY_NAME[name], 300, 1024
    E = model_blocks(qt, vocab, d, rng, scale=1e-2)
    ref = O.dequant_rows(E, qt, vocab, d)
    dev = torch.device("cuda")
    Ed = torch.from_numpy(E.reshape(-1)).to(dev)
    toks = torch.tensor([0, 299, 17, 150], dtype=torch.int32, device=dev)
    h = torch.empty(d, device=dev)
    for i in range(4):
        pos = torch.tensor([i], dtype=torch.int32, device=dev)
        fn.embed(qt, Ed.data_ptr(), d, toks.data_ptr(), pos.data_ptr(), h.data_ptr())
        fn.sync()
        assert np.array_equal(h.cpu().numpy().view(np.uint32), ref[int(toks[i])].view(np.uint32))


@pytest.mark.parametrize("d", [4, 512, 2048, 4100])
def test_rmsnorm(fn, torch_cuda, d):
    torch = torch_cuda
    rng = np.random.default_rng(d)
    x = (rng.standard_normal(d) * 7).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    dev = torch.device("cuda")
    xd, wd, out = torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev), torch.empty(d, device=dev)
    fn.rmsnorm(xd.data_ptr(), wd.data_ptr(), out.data_ptr(), d, 1e-6)
    fn.sync()
    ref = rmsnorm(x, w, 1e-6)
    assert np.abs(out.cpu().numpy() - ref).max() <= 2e-6 * np.abs(ref).max()


@pytest.mark.parametrize("nh,nkv,steps,start", [(4, 1, 40, 0), (16, 2, 12, 3000), (8, 8, 6, 0)])
def test_attention_positions(fn, torch_cuda, nh, nkv, steps, start):
    """Several consecutive positions: each call appends k, v at *pos and attends over 0..*pos. start > 0 pre-fills the
    cache (positions 0..start-1) with random rotated keys, so long-context angles and score rows are covered."""
    torch = torch_cuda
    rng = np.random.default_rng(nh * 100 + steps)
    HD, eps, max_ctx = 256, 1e-6, start + steps + 5
    inv = rope_inv_freq(1e7)
    wq = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
    wk = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
    Kc, Vc = torch.zeros(max_ctx, nkv, HD, device=dev), torch.zeros(max_ctx, nkv, HD, device=dev)
    cache = ([], [])
    if start:
        K0 = rng.standard_normal((start, nkv, HD)).astype(np.float32)
        V0 = rng.standard_normal((start, nkv, HD)).astype(np.float32)
        Kc[:start] = t(K0)
        Vc[:start] = t(V0)
        cache[0].extend(K0.astype(np.float64))
        cache[1].extend(V0.astype(np.float64))
    wqd, wkd, invd = t(wq), t(wk), t(inv)
    Q, out = torch.empty(nh * HD, device=dev), torch.empty(nh * HD, device=dev)
    for p in range(start, start + steps):
        qg = (rng.standard_normal(nh * 2 * HD) * 2).astype(np.float32)
        k = (rng.standard_normal(nkv * HD) * 2).astype(np.float32)
        v = rng.standard_normal(nkv * HD).astype(np.float32)
        pos = torch.tensor([p], dtype=torch.int32, device=dev)
        qgd, kd, vd = t(qg), t(k), t(v)
        fn.attn_decode(qgd.data_ptr(), kd.data_ptr(), vd.data_ptr(), wqd.data_ptr(), wkd.data_ptr(), invd.data_ptr(),
                       Q.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), out.data_ptr(), pos.data_ptr(), nh, nkv, max_ctx,
                       eps)
        fn.sync()
        ref, qr = gated_attention(qg, k, v, wq, wk, inv, p, cache, nh, nkv, eps)
        assert np.abs(Q.cpu().numpy() - qr.reshape(-1)).max() <= 2e-6 * np.abs(qr).max(), p
        got = out.cpu().numpy()
        # fp32 sums over n = p + 1 positions: a random-walk bound, 1e-6 sqrt(n) of the largest cached value
        n = p + 1
        assert np.abs(got - ref).max() <= 1e-6 * np.sqrt(n) * np.abs(np.stack(cache[1])).max(), p
        assert np.abs(Kc[p].cpu().numpy() - cache[0][-1]).max() <= 2e-6 * np.abs(cache[0][-1]).max()


def test_model_steps_match_oracle(fn, small, torch_cuda):
    """Step by step (eager launches): the model's logits against the float64 oracle fed the same tokens, the prompt
    then the model's own greedy continuation."""
    torch = torch_cuda
    cfg, W, m = small
    o = OracleModel(cfg, W, rope_inv_freq(cfg["rope_base"]))
    rng = np.random.default_rng(7)
    prompt = rng.integers(0, cfg["vocab"], 6)
    s = torch.cuda.Stream()
    m.start(prompt, s)
    worst = 0.0
    for i in range(20):
        m.launch_step(s.cuda_stream)
        fn.sync(s.cuda_stream)
        tok = int(m.tokens[i].item())
        if i < len(prompt):
            assert tok == prompt[i]
        ref = o.step(tok)
        lg = m.logits.cpu().numpy()
        diff = np.abs(logprobs(lg) - logprobs(ref)).max()
        worst = max(worst, diff)
        assert diff <= LOGPROB_TOL, (i, diff)
        top = np.sort(ref)[::-1]
        if top[0] - top[1] > TIE:
            assert int(m.next.item()) == int(np.argmax(ref)), i
        assert int(m.pos.item()) == i + 1
        if i + 1 >= len(prompt):
            assert int(m.tokens[i + 1].item()) == int(m.next.item())
    print(f"max log-prob diff {worst:.3g}")


def test_model_graph_greedy(fn, small, torch_cuda):
    """The captured step replayed once per token: greedy ids equal the oracle's own greedy chain; a second prompt in
    between does not change a replayed generation (the reset clears every state), bit for bit."""
    torch = torch_cuda
    cfg, W, m = small
    s = torch.cuda.Stream()
    m.capture(s)
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, cfg["vocab"], 8)
    n_new = 24
    ids = m.generate(prompt, n_new, s)
    last = m.logits.cpu().numpy().copy()
    o = OracleModel(cfg, W, rope_inv_freq(cfg["rope_base"]))
    ref_ids = list(prompt)
    for i in range(len(prompt) + n_new - 1):
        lg = o.step(ref_ids[i])
        if i + 1 >= len(prompt):
            top = np.sort(lg)[::-1]
            if top[0] - top[1] <= TIE:  # a near tie: the chains may part here
                break
            ref_ids.append(int(np.argmax(lg)))
    n = len(ref_ids)
    assert list(ids[:n]) == ref_ids
    assert n >= len(prompt) + 4, "near tie early in the oracle chain"
    m.generate(rng.integers(0, cfg["vocab"], 3), 5, s)
    ids2 = m.generate(prompt, n_new, s)
    assert np.array_equal(ids, ids2)
    assert np.array_equal(last.view(np.uint32), m.logits.cpu().numpy().view(np.uint32))
