"""GPU parity of the model API (FN.load / reset / forward / debug_layers; the reference's fn_load / fn_forward,
engine/faie2fn.cu:2466-2490, 2524, 2703-2743): a small model of the config-5 structure saved as a GGUF file, loaded
and stepped from host token ids.

Bars: the log-probabilities of every forwarded token within 1e-4 of the float64 oracle (oracle/model.py) fed the same
tokens, and the returned greedy ids equal to the oracle's wherever its top two logits are more than 1e-3 apart; a
reset replays bit for bit; eager steps (use_graphs(0)) and debug runs equal the graph's bit for bit; the debug
buffer's last layer, put through the final RMSNorm and the dequantised lm_head in float64, gives the logits within
1e-4 of max |logit|; the reference's errors (nt out of range, context full, not loaded)."""

import numpy as np
import pytest

from oracle import dequant as O
from oracle.model import OracleModel, rmsnorm
from synth import model_config, model_weights, rope_inv_freq

pytestmark = pytest.mark.gpu
LOGPROB_TOL = 1e-4
TIE = 1e-3
MAX_CTX = 40


def logprobs(lg):
    lg = np.asarray(lg, np.float64)
    m = lg.max()
    return lg - m - np.log(np.exp(lg - m).sum())


@pytest.fixture(scope="module")
def loaded(fn, tmp_path_factory):
    from runner import save_model
    cfg = model_config(small=True)
    W = model_weights(cfg, 5)
    p = tmp_path_factory.mktemp("model") / "small.gguf"
    save_model(str(p), cfg, W)
    fn.load(max_ctx=MAX_CTX, shard1=str(p))
    yield cfg, W
    fn.free()


def test_forward_matches_oracle(fn, loaded):
    cfg, W = loaded
    fn.reset()
    o = OracleModel(cfg, W, rope_inv_freq(cfg["rope_base"]))
    rng = np.random.default_rng(13)
    prompt = rng.integers(0, cfg["vocab"], 7)
    worst = 0.0

    def check(tokens, am, lg):
        nonlocal worst
        for i, tok in enumerate(tokens):
            ref = o.step(int(tok))
            diff = np.abs(logprobs(lg[i]) - logprobs(ref)).max()
            worst = max(worst, diff)
            assert diff <= LOGPROB_TOL, (int(tok), diff)
            top = np.sort(ref)[::-1]
            if top[0] - top[1] > TIE:
                assert int(am[i]) == int(np.argmax(ref))

    am, lg = fn.forward(prompt, logits=True)
    assert am.shape == (7,) and lg.shape == (7, cfg["vocab"])
    check(prompt, am, lg)
    assert fn.n_past() == 7
    tok = int(am[-1])
    for _ in range(6):  # greedy continuation, one token per call
        a1, l1 = fn.forward([tok], logits=True)
        check([tok], a1, l1)
        tok = int(a1[0])
    chunk = rng.integers(0, cfg["vocab"], 8)  # a full 8-token call mid-sequence
    a8, l8 = fn.forward(chunk, logits=True)
    check(chunk, a8, l8)
    assert fn.n_past() == 21 and fn.last_ms() > 0
    assert fn.split() == cfg["layers"] and fn.dev_gb(0) > 0
    print(f"max log-prob diff {worst:.3g}")


def test_reset_graph_eager_debug_identical(fn, loaded):
    cfg, W = loaded
    rng = np.random.default_rng(17)
    toks = rng.integers(0, cfg["vocab"], 5)
    fn.reset()
    a1, l1 = fn.forward(toks, logits=True)
    am_only = fn.forward(rng.integers(0, cfg["vocab"], 2))  # argmax only
    assert am_only.shape == (2,)
    fn.reset()
    a2, l2 = fn.forward(toks, logits=True)
    fn.reset()
    fn.use_graphs(0)
    try:
        a3, l3 = fn.forward(toks, logits=True)
    finally:
        fn.use_graphs(1)
    buf = np.zeros((cfg["layers"], len(toks), cfg["D"]), np.float32)
    fn.reset()
    fn.debug_layers(buf)
    try:
        a4, l4 = fn.forward(toks, logits=True)
    finally:
        fn.debug_layers(None)
    for a, lg in ((a2, l2), (a3, l3), (a4, l4)):
        assert np.array_equal(a, a1)
        assert np.array_equal(lg.view(np.uint32), l1.view(np.uint32))
    assert np.isfinite(buf).all() and (np.abs(buf).max(axis=2) > 0).all()
    head = O.dequant_rows(W["head"], cfg["head"], cfg["vocab"], cfg["D"]).astype(np.float64)
    for i in range(len(toks)):
        ref = head @ rmsnorm(buf[-1, i], W["final_norm"], cfg["eps"]).astype(np.float64)
        assert np.abs(l1[i] - ref).max() <= 1e-4 * np.abs(ref).max(), i


def test_errors(fn, loaded):
    cfg, _ = loaded
    fn.reset()
    with pytest.raises(RuntimeError, match="nt out of range"):
        fn.forward(np.zeros(9, np.int32))
    with pytest.raises(RuntimeError, match="nt out of range"):
        fn.forward(np.zeros(0, np.int32))
    with pytest.raises(RuntimeError, match="token id out of range"):
        fn.forward([cfg["vocab"]])
    for _ in range(MAX_CTX // 8):
        fn.forward(np.arange(8, dtype=np.int32))
    assert fn.n_past() == MAX_CTX
    with pytest.raises(RuntimeError, match="context full"):
        fn.forward([1])
    with pytest.raises(RuntimeError):
        fn.debug_layers(np.zeros((1, 1, 1), np.float32))
    fn.reset()
    assert fn.n_past() == 0


def test_mixed_formats_file(fn, loaded, tmp_path):
    """A file whose weights do not share one format: a Q6_K DeltaNet output projection, Q8_0 attention values (so the
    attention's q / k / v run as three GEMVs) and a Q5_K lm_head; forward against the oracle on the same weights."""
    from runner import load_model, save_model
    from synth import BY_NAME, model_blocks
    cfg, W = loaded
    rng = np.random.default_rng(23)
    layers = [dict(L) for L in W["layers"]]
    g = next(i for i, L in enumerate(layers) if L["kind"] == "G")
    a = next(i for i, L in enumerate(layers) if L["kind"] == "A")
    layers[g]["w_out"] = model_blocks(BY_NAME["Q6_K"], cfg["D"], cfg["nvh"] * 128, rng)
    layers[g]["qt"] = {"w_out": BY_NAME["Q6_K"]}
    layers[a]["w_v"] = model_blocks(BY_NAME["Q8_0"], cfg["nkv"] * 256, cfg["D"], rng)
    layers[a]["qt"] = {"w_v": BY_NAME["Q8_0"]}
    cfg2 = dict(cfg, head=BY_NAME["Q5_K"])
    W2 = dict(W, layers=layers, head=model_blocks(BY_NAME["Q5_K"], cfg["vocab"], cfg["D"], rng, scale=1e-4))
    p = str(tmp_path / "mixed.gguf")
    save_model(p, cfg2, W2)
    cfg3, W3, _ = load_model(p)
    fn.load(max_ctx=16, shard1=p)
    o = OracleModel(cfg3, W3, rope_inv_freq(cfg3["rope_base"]))
    toks = rng.integers(0, cfg["vocab"], 6)
    am, lg = fn.forward(toks, logits=True)
    for i, t in enumerate(toks):
        ref = o.step(int(t))
        assert np.abs(logprobs(lg[i]) - logprobs(ref)).max() <= LOGPROB_TOL, i
        top = np.sort(ref)[::-1]
        if top[0] - top[1] > TIE:
            assert int(am[i]) == int(np.argmax(ref))
    with pytest.raises(RuntimeError, match="one format"):  # the batched path stacks q / k / v into one weight
        fn.load(max_ctx=16, shard1=p, batch=2)


BATCH_LOGPROB_TOL = 1e-3  # the tensor-core path's stated model-level tolerance (tests/test_batch_gpu.py)
BATCH_TIE = 1e-2


def test_forward_batch(fn, loaded, tmp_path):
    """forward_batch: three sequences against three float64 oracles (tensor-core tolerance); forward's own sequence
    alongside, untouched by the batch; reset and eager steps replay the batch bit for bit; the batched errors."""
    from runner import save_model
    cfg, W = loaded
    p = str(tmp_path / "small.gguf")
    save_model(p, cfg, W)
    fn.load(max_ctx=24, shard1=p, batch=3)
    rng = np.random.default_rng(29)
    prompts = rng.integers(0, cfg["vocab"], (3, 5))
    oracles = [OracleModel(cfg, W, rope_inv_freq(cfg["rope_base"])) for _ in range(3)]
    worst = 0.0

    def check(tokens, am, lg):
        nonlocal worst
        for b in range(3):
            for i, tok in enumerate(tokens[b]):
                ref = oracles[b].step(int(tok))
                diff = np.abs(logprobs(lg[b, i]) - logprobs(ref)).max()
                worst = max(worst, diff)
                assert diff <= BATCH_LOGPROB_TOL, (b, i, diff)
                top = np.sort(ref)[::-1]
                if top[0] - top[1] > BATCH_TIE:
                    assert int(am[b, i]) == int(np.argmax(ref)), (b, i)

    am0, lg0 = fn.forward_batch(prompts, logits=True)
    assert am0.shape == (3, 5) and lg0.shape == (3, 5, cfg["vocab"])
    check(prompts, am0, lg0)
    toks = am0[:, -1:]
    for _ in range(4):
        a, lg = fn.forward_batch(toks, logits=True)
        check(toks, a, lg)
        toks = a
    assert fn.n_past_batch() == 9
    one = OracleModel(cfg, W, rope_inv_freq(cfg["rope_base"]))  # forward's sequence: its own states
    a1, l1 = fn.forward(prompts[1], logits=True)
    for i, tok in enumerate(prompts[1]):
        assert np.abs(logprobs(l1[i]) - logprobs(one.step(int(tok)))).max() <= LOGPROB_TOL
    assert fn.n_past() == 5 and fn.n_past_batch() == 9
    with pytest.raises(RuntimeError, match=r"tokens must be \[3\]\[nt\]"):
        fn.forward_batch(np.zeros((2, 1), np.int32))
    with pytest.raises(RuntimeError, match="nt out of range"):
        fn.forward_batch(np.zeros((3, 9), np.int32))
    fn.reset()
    assert fn.n_past_batch() == 0 and fn.n_past() == 0
    am2, lg2 = fn.forward_batch(prompts, logits=True)
    fn.reset()
    fn.use_graphs(0)
    try:
        am3, lg3 = fn.forward_batch(prompts, logits=True)
    finally:
        fn.use_graphs(1)
    for a, lg in ((am2, lg2), (am3, lg3)):
        assert np.array_equal(a, am0) and np.array_equal(lg.view(np.uint32), lg0.view(np.uint32))
    for _ in range(24 // 8 - 1):
        fn.forward_batch(np.zeros((3, 8), np.int32))
    fn.forward_batch(np.zeros((3, 3), np.int32))
    with pytest.raises(RuntimeError, match="context full"):
        fn.forward_batch(np.zeros((3, 1), np.int32))
    print(f"batch max log-prob diff {worst:.3g}")


def test_not_loaded(fn, loaded, tmp_path):
    fn.free()
    assert fn.n_past() == -1 and fn.last_ms() == -1.0 and fn.dev_gb(0) == -1.0
    with pytest.raises(RuntimeError, match="not loaded"):
        fn.forward([1])
    with pytest.raises(RuntimeError, match="not loaded"):
        fn.reset()
    with pytest.raises(RuntimeError, match="not loaded"):
        fn.forward_batch(np.zeros((1, 1), np.int32))
    with pytest.raises(RuntimeError):
        fn.load(shard1=str(tmp_path / "missing.gguf"))
    with pytest.raises(RuntimeError, match="not loaded"):
        fn.forward([1])
