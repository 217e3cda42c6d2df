"""Host side of the model API (flashnext/gguf_file.py, flashnext/runner.py): GGUF v3 files written and read back byte for
byte, a synthetic config-5-structure model saved under the qwen3next tensor names the reference's loader reads
(engine/faie2fn.cu:2617-2657) and loaded back into the runner's layout, one file or two shards, and the loader's
refusals (not GGUF, truncated, a missing or unexpected tensor, tensors the runner has no kernels for, mixed formats
inside a stacked weight). No GPU."""

import os

import numpy as np
import pytest

import gguf_file as gguf
from runner import load_model, save_model
from synth import BY_NAME, model_blocks, model_config, model_weights


def test_gguf_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    q4 = model_blocks(BY_NAME["Q4_K"], 6, 512, rng)
    ex = model_blocks(BY_NAME["IQ3_XXS"], 3 * 4, 256, rng)
    v = rng.standard_normal(96).astype(np.float32)
    h = rng.standard_normal((3, 64)).astype(np.float16)
    meta = {"general.architecture": "test", "a.u32": 7, "a.neg": -5, "a.big": 2**40, "a.f": 0.5, "a.b": True,
            "a.s": "hello", "a.ints": [1, 2, 3], "a.strs": ["x", "yz"], "a.empty": []}
    p = str(tmp_path / "t.gguf")
    gguf.write(p, meta, [("v", gguf.GGML_F32, [96], v), ("w", BY_NAME["Q4_K"], [512, 6], q4),
                         ("e", BY_NAME["IQ3_XXS"], [256, 4, 3], ex), ("h", gguf.GGML_F16, [64, 3], h)])
    m, t = gguf.read(p)
    assert m == meta
    assert np.array_equal(t["v"].f32(), v)
    assert np.array_equal(t["w"].rows_u8(), q4) and t["w"].dims == (512, 6) and t["w"].rows == 6
    assert np.array_equal(t["e"].rows_u8(), ex) and t["e"].rows == 12 and t["e"].cols == 256
    assert np.array_equal(t["h"].f32(), h.astype(np.float32))
    for x in t.values():  # every tensor starts on the alignment
        assert (x.data.ctypes.data - t["v"].data.ctypes.data) % gguf.ALIGN == 0


def test_gguf_refusals(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUX" + b"\0" * 64)
    with pytest.raises(gguf.GGUFError, match="not a GGUF"):
        gguf.read(str(p))
    good = str(tmp_path / "g.gguf")
    gguf.write(good, {"k": 1}, [("v", gguf.GGML_F32, [32], np.zeros(32, np.float32))])
    raw = open(good, "rb").read()
    (tmp_path / "cut.gguf").write_bytes(raw[:-8])
    with pytest.raises(gguf.GGUFError, match="out of range"):
        gguf.read(str(tmp_path / "cut.gguf"))
    (tmp_path / "cut2.gguf").write_bytes(raw[:30])
    with pytest.raises(gguf.GGUFError, match="truncated"):
        gguf.read(str(tmp_path / "cut2.gguf"))
    (tmp_path / "empty.gguf").write_bytes(b"")
    with pytest.raises(gguf.GGUFError, match="truncated"):
        gguf.read(str(tmp_path / "empty.gguf"))
    key = b"\xff\xfe"  # a metadata key that is not UTF-8
    (tmp_path / "utf.gguf").write_bytes(b"GGUF" + (3).to_bytes(4, "little") + (0).to_bytes(8, "little")
                                        + (1).to_bytes(8, "little") + (2).to_bytes(8, "little") + key + b"\0" * 16)
    with pytest.raises(gguf.GGUFError, match="not UTF-8"):
        gguf.read(str(tmp_path / "utf.gguf"))
    with pytest.raises(gguf.GGUFError):  # bytes that do not match the dims
        gguf.write(str(tmp_path / "x.gguf"), {}, [("v", gguf.GGML_F32, [32], np.zeros(31, np.float32))])


@pytest.fixture(scope="module")
def small():
    cfg = model_config(small=True)
    return cfg, model_weights(cfg, 3)


def _same_model(cfg, W, cfg2, W2):
    for k in ("D", "layers", "vocab", "nkh", "nvh", "nh", "nkv", "ne", "k", "ffe", "proj", "gate_up", "down", "embed",
              "head", "router"):
        assert cfg2[k] == cfg[k], k
    assert cfg2["pattern"] == cfg["pattern"] * (cfg["layers"] // len(cfg["pattern"]))
    assert np.float32(cfg2["eps"]) == np.float32(cfg["eps"]) and cfg2["rope_base"] == cfg["rope_base"]
    for k in ("embed", "head", "final_norm"):
        assert np.array_equal(W2[k], W[k]), k
    for L, L2 in zip(W["layers"], W2["layers"]):
        assert L2["kind"] == L["kind"]
        for k, v in L.items():
            if k == "moe":
                assert all(np.array_equal(a, b) for a, b in zip(v, L2["moe"]))
            elif k not in ("kind", "qt"):
                assert np.array_equal(np.asarray(L2[k]).reshape(np.shape(v)), v), k


def test_save_load_model(small, tmp_path):
    cfg, W = small
    p = str(tmp_path / "m.gguf")
    save_model(p, cfg, W)
    cfg2, W2, nbytes = load_model(p)
    _same_model(cfg, W, cfg2, W2)
    assert nbytes > W["embed"].nbytes + W["head"].nbytes
    assert all(L["qt"]["w_in" if L["kind"] == "G" else "w_q"] == cfg["proj"] for L in W2["layers"])


def test_two_shards(small, tmp_path):
    """The tensors split over two files (the reference's shard1 / shard2) load as one model."""
    cfg, W = small
    one = str(tmp_path / "m.gguf")
    save_model(one, cfg, W)
    meta, t = gguf.read(one)
    names = list(t)
    half = len(names) // 2
    rows = lambda n: (n, t[n].qtype, list(t[n].dims), t[n].data)  # noqa: E731
    gguf.write(str(tmp_path / "s1.gguf"), meta, [rows(n) for n in names[:half]])
    gguf.write(str(tmp_path / "s2.gguf"), {}, [rows(n) for n in names[half:]])
    cfg2, W2, _ = load_model(str(tmp_path / "s1.gguf"), str(tmp_path / "s2.gguf"))
    _same_model(cfg, W, cfg2, W2)
    with pytest.raises(gguf.GGUFError, match="more than one shard"):
        load_model(one, str(tmp_path / "s2.gguf"))
    with pytest.raises(gguf.GGUFError, match="missing tensor"):
        load_model(str(tmp_path / "s1.gguf"))


def test_mixed_formats_per_weight(small, tmp_path):
    """Per-weight formats survive the file: a Q6_K output projection and Q8_0 attention values in one layer each."""
    cfg, W = small
    rng = np.random.default_rng(1)
    layers = [dict(L) for L in W["layers"]]
    g = next(i for i, L in enumerate(layers) if L["kind"] == "G")
    a = next(i for i, L in enumerate(layers) if L["kind"] == "A")
    layers[g]["w_out"] = model_blocks(BY_NAME["Q6_K"], cfg["D"], cfg["nvh"] * 128, rng)
    layers[g]["qt"] = {"w_out": BY_NAME["Q6_K"]}
    layers[a]["w_v"] = model_blocks(BY_NAME["Q8_0"], cfg["nkv"] * 256, cfg["D"], rng)
    layers[a]["qt"] = {"w_v": BY_NAME["Q8_0"]}
    W2 = dict(W, layers=layers)
    p = str(tmp_path / "m.gguf")
    save_model(p, cfg, W2)
    _, W3, _ = load_model(p)
    assert W3["layers"][g]["qt"]["w_out"] == BY_NAME["Q6_K"]
    assert W3["layers"][a]["qt"]["w_v"] == BY_NAME["Q8_0"] and W3["layers"][a]["qt"]["w_q"] == cfg["proj"]
    assert np.array_equal(W3["layers"][g]["w_out"], layers[g]["w_out"])


def test_loader_refusals(small, tmp_path):
    cfg, W = small
    p = str(tmp_path / "m.gguf")
    save_model(p, cfg, W)
    meta, t = gguf.read(p)
    rows = lambda n: (n, t[n].qtype, list(t[n].dims), t[n].data)  # noqa: E731

    def variant(name, tensors, meta_=meta):
        q = str(tmp_path / name)
        gguf.write(q, meta_, tensors)
        return q

    with pytest.raises(gguf.GGUFError, match="missing tensor blk.1.ssm_a"):
        load_model(variant("a.gguf", [rows(n) for n in t if n != "blk.1.ssm_a"]))
    extra = [rows(n) for n in t] + [("blk.0.hc_attn_norm.weight", gguf.GGML_F32, [32], np.zeros(32, np.float32))]
    with pytest.raises(gguf.GGUFError, match="no kernels for"):
        load_model(variant("b.gguf", extra))
    extra = [rows(n) for n in t] + [("blk.0.something.weight", gguf.GGML_F32, [32], np.zeros(32, np.float32))]
    with pytest.raises(gguf.GGUFError, match="does not use"):
        load_model(variant("c.gguf", extra))
    with pytest.raises(gguf.GGUFError, match="expert_used_count"):
        load_model(variant("d.gguf", [rows(n) for n in t], {k: v for k, v in meta.items() if "expert_used" not in k}))
    rng = np.random.default_rng(2)
    mixed = [rows(n) for n in t if n != "blk.0.attn_gate.weight"]
    mixed.append(("blk.0.attn_gate.weight", BY_NAME["Q8_0"], [cfg["D"], cfg["nvh"] * 128],
                  model_blocks(BY_NAME["Q8_0"], cfg["nvh"] * 128, cfg["D"], rng)))
    with pytest.raises(gguf.GGUFError, match="different formats"):
        load_model(variant("e.gguf", mixed))
    short = [rows(n) for n in t if n != "blk.3.attn_v.weight"]
    short.append(("blk.3.attn_v.weight", t["blk.3.attn_v.weight"].qtype, [cfg["D"], 128],
                  t["blk.3.attn_v.weight"].data[:t["blk.3.attn_v.weight"].data.nbytes // 2]))
    with pytest.raises(gguf.GGUFError, match="blk.3.attn_v.weight: shape"):
        load_model(variant("f.gguf", short))
    attn_only = [rows(n) for n in t if not n.startswith(("blk.0.", "blk.1.", "blk.2."))]  # blk.3 is the attention layer
    attn_only = [(n.replace("blk.3.", "blk.0."), q, d, x) for n, q, d, x in attn_only]
    with pytest.raises(gguf.GGUFError, match="both gated-DeltaNet and attention"):
        load_model(variant("g.gguf", attn_only, dict(meta, **{"qwen3next.block_count": 1})))
    assert not os.path.exists(str(tmp_path / "never.gguf"))
    with pytest.raises(OSError):
        load_model(str(tmp_path / "never.gguf"))


def test_fn_model_api_without_a_model(libpath, tmp_path):
    """FN's model methods before a model is loaded, and loads that fail in the file reader (before any device work):
    the reference's return values (-1) and RuntimeError messages."""
    from fn import FN
    f = FN(libpath)
    assert f.n_past() == -1 and f.n_past_batch() == -1 and f.last_ms() == -1.0 and f.dev_gb(0) == -1.0
    assert f.split() == -1
    for call in (lambda: f.forward([1]), f.reset, lambda: f.forward_batch([[1]]), lambda: f.debug_layers(None),
                 lambda: f.use_graphs(1)):
        with pytest.raises(RuntimeError, match="not loaded"):
            call()
    f.free()  # nothing loaded: no-op
    with pytest.raises(RuntimeError):
        f.load(shard1=str(tmp_path / "missing.gguf"))
    (tmp_path / "bad.gguf").write_bytes(b"GGML" + b"\0" * 60)
    with pytest.raises(RuntimeError, match="not a GGUF"):
        f.load(shard1=str(tmp_path / "bad.gguf"))
    with pytest.raises(RuntimeError, match="batch out of range"):
        f.load(shard1=str(tmp_path / "bad.gguf"), batch=33)
    with pytest.raises(RuntimeError, match="not loaded"):
        f.forward([1])
    import fn as fnmod  # the reference's call form: paths from SH1 / SH2 (env FN_SHARD1 / FN_SHARD2)
    old = fnmod.SH1, fnmod.SH2
    try:
        fnmod.SH1, fnmod.SH2 = None, None
        with pytest.raises(RuntimeError, match="no model file"):
            f.load(max_ctx=4096)
        fnmod.SH1 = str(tmp_path / "bad.gguf")
        with pytest.raises(RuntimeError, match="not a GGUF"):
            f.load(max_ctx=8192, split=0)
    finally:
        fnmod.SH1, fnmod.SH2 = old


def test_save_streams_generator_layers(tmp_path):
    """Pooled weights (layers from a generator, consumed once) write the same file, byte for byte, as the same seed's
    layers held in a list; the writer refuses data that does not match its tensor list."""
    cfg = model_config(small=True)
    a, b = str(tmp_path / "gen.gguf"), str(tmp_path / "list.gguf")
    Wg = model_weights(cfg, 4, pooled=True)
    assert not isinstance(Wg["layers"], list)
    save_model(a, cfg, Wg)
    Wl = model_weights(cfg, 4, pooled=True)
    Wl["layers"] = list(Wl["layers"])
    save_model(b, cfg, Wl)
    assert open(a, "rb").read() == open(b, "rb").read()
    cfg2, W2, _ = load_model(a)
    _same_model(cfg, Wl, cfg2, W2)
    v = np.zeros(32, np.float32)
    with pytest.raises(gguf.GGUFError, match="no data"):
        gguf.write(str(tmp_path / "x.gguf"), {}, [("a", gguf.GGML_F32, [32]), ("b", gguf.GGML_F32, [32])], [v])
    with pytest.raises(gguf.GGUFError, match="more data"):
        gguf.write(str(tmp_path / "y.gguf"), {}, [("a", gguf.GGML_F32, [32])], [v, v])


def test_library_loader_refusals(libpath, small, tmp_path):
    """The library's fn_load (csrc/fn_runner.cu) reads the same files with its own C++ reader and refuses the same
    ones with the same messages; every check here fires before any device work, so it runs without a GPU."""
    from fn import FN
    f = FN(libpath)
    cfg, W = small
    p = str(tmp_path / "m.gguf")
    save_model(p, cfg, W)
    meta, t = gguf.read(p)
    rows = lambda n: (n, t[n].qtype, list(t[n].dims), t[n].data)  # noqa: E731

    def variant(name, tensors, meta_=meta):
        q = str(tmp_path / name)
        gguf.write(q, meta_, tensors)
        return q

    def refuses(match, s1, s2=None):
        with pytest.raises(RuntimeError, match=match):
            f.load(max_ctx=64, shard1=s1, shard2=s2)
        assert f.n_past() == -1  # nothing loaded

    (tmp_path / "x.gguf").write_bytes(b"GGUX" + b"\0" * 64)
    refuses("not a GGUF", str(tmp_path / "x.gguf"))
    raw = open(p, "rb").read()
    (tmp_path / "cut.gguf").write_bytes(raw[:-8])
    refuses("out of range", str(tmp_path / "cut.gguf"))
    (tmp_path / "cut2.gguf").write_bytes(raw[:30])
    refuses("truncated", str(tmp_path / "cut2.gguf"))
    (tmp_path / "empty.gguf").write_bytes(b"")
    refuses("truncated", str(tmp_path / "empty.gguf"))
    (tmp_path / "utf.gguf").write_bytes(b"GGUF" + (3).to_bytes(4, "little") + (0).to_bytes(8, "little")
                                        + (1).to_bytes(8, "little") + (2).to_bytes(8, "little") + b"\xff\xfe" + b"\0" * 16)
    refuses("not UTF-8", str(tmp_path / "utf.gguf"))
    refuses("No such file", str(tmp_path / "never.gguf"))
    refuses("missing tensor blk.1.ssm_a", variant("a.gguf", [rows(n) for n in t if n != "blk.1.ssm_a"]))
    extra = [rows(n) for n in t] + [("blk.0.hc_attn_norm.weight", gguf.GGML_F32, [32], np.zeros(32, np.float32))]
    refuses("no kernels for", variant("b.gguf", extra))
    extra = [rows(n) for n in t] + [("blk.0.something.weight", gguf.GGML_F32, [32], np.zeros(32, np.float32))]
    refuses("does not use", variant("c.gguf", extra))
    refuses("expert_used_count", variant("d.gguf", [rows(n) for n in t], {k: v for k, v in meta.items()
                                                                          if "expert_used" not in k}))
    rng = np.random.default_rng(2)
    mixed = [rows(n) for n in t if n != "blk.0.attn_gate.weight"]
    mixed.append(("blk.0.attn_gate.weight", BY_NAME["Q8_0"], [cfg["D"], cfg["nvh"] * 128],
                  model_blocks(BY_NAME["Q8_0"], cfg["nvh"] * 128, cfg["D"], rng)))
    refuses("different formats", variant("e.gguf", mixed))
    short = [rows(n) for n in t if n != "blk.3.attn_v.weight"]
    short.append(("blk.3.attn_v.weight", t["blk.3.attn_v.weight"].qtype, [cfg["D"], 128],
                  t["blk.3.attn_v.weight"].data[:t["blk.3.attn_v.weight"].data.nbytes // 2]))
    refuses("blk.3.attn_v.weight: shape", variant("f.gguf", short))
    attn_only = [rows(n) for n in t if not n.startswith(("blk.0.", "blk.1.", "blk.2."))]
    attn_only = [(n.replace("blk.3.", "blk.0."), q, d, x) for n, q, d, x in attn_only]
    refuses("both gated-DeltaNet and attention", variant("g.gguf", attn_only, dict(meta, **{"qwen3next.block_count": 1})))
    names = list(t)
    half = len(names) // 2
    s1 = variant("s1.gguf", [rows(n) for n in names[:half]])
    s2 = variant("s2.gguf", [rows(n) for n in names[half:]], {})
    refuses("more than one shard", p, s2)
    refuses("missing tensor", s1)


def test_reference_binding_lines(libpath):
    """The reference's own FN.__init__ binding lines (flashnext/fn.py:27-33), run verbatim against this library: every
    symbol they name exists and takes the argtypes / restypes they set."""
    import ctypes as C
    P = np.ctypeslib.ndpointer
    F32 = P(np.float32, flags="C_CONTIGUOUS")
    I32 = P(np.int32, flags="C_CONTIGUOUS")
    U8 = P(np.uint8, flags="C_CONTIGUOUS")
    d = C.CDLL(libpath)
    d.fn_error.restype = C.c_char_p
    d.fn_load.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_int]
    d.fn_forward.argtypes = [I32, C.c_int, C.c_void_p, C.c_void_p]
    d.fn_debug_layers.argtypes = [C.c_void_p]
    d.fn_test_dequant.argtypes = [C.c_uint32, U8, C.c_int, C.c_int, F32]
    d.fn_test_gemv.argtypes = [C.c_uint32, U8, C.c_int, C.c_int, F32, C.c_int, F32]
    d.fn_dev_gb.restype = C.c_double
    d.fn_dev_gb.argtypes = [C.c_int]
    d.fn_last_ms.restype = C.c_double
    # the reference's FN methods' calls with nothing loaded: its return values and messages
    assert d.fn_dev_gb(0) == -1.0 and d.fn_last_ms() == -1.0 and d.fn_n_past() == -1 and d.fn_split() == -1
    assert d.fn_forward(np.zeros(1, np.int32), 1, None, np.zeros(1, np.int32).ctypes.data) == -1
    assert d.fn_error() == b"not loaded"
    assert d.fn_reset() == -1 and d.fn_debug_layers(None) == -1
    assert d.fn_load(b"/nonexistent.gguf", None, 4096, 0) == -1 and b"No such file" in d.fn_error()
