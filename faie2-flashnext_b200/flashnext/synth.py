"""Seeded synthetic GGUF weights and activations (the benchmark's input distribution).

The reference measured on real model tensors (flashnext/test_fn_quants.py:19-31) that are not
shipped; these synthetic blocks stand in for them. Every block is uniform random bytes, then the
fp16 scale fields are overwritten with float16(|N(0,1)| * 1e-3) so every value is finite. BF16
weights are N(0, 0.05) rounded to bf16 instead (random bf16 bytes would hold NaN and Inf).
"""

from __future__ import annotations

import numpy as np

# ggml type id -> (name, values per block, bytes per block)
TYPES = {
    2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20), 6: ("Q5_0", 32, 22), 7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34),
    10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176),
    14: ("Q6_K", 256, 210), 16: ("IQ2_XXS", 256, 66), 17: ("IQ2_XS", 256, 74), 18: ("IQ3_XXS", 256, 98),
    20: ("IQ4_NL", 32, 18), 21: ("IQ3_S", 256, 110), 22: ("IQ2_S", 256, 82), 23: ("IQ4_XS", 256, 136),
    30: ("BF16", 1, 2), 42: ("Q2_0", 64, 18),
}
BY_NAME = {v[0]: k for k, v in TYPES.items()}

# byte offsets of the fp16 scale fields inside one block
SCALE_OFFSETS = {
    "Q4_0": (0,), "Q5_0": (0,), "Q8_0": (0,), "IQ2_XXS": (0,), "IQ2_XS": (0,), "IQ2_S": (0,), "IQ3_XXS": (0,),
    "IQ3_S": (0,), "IQ4_XS": (0,), "IQ4_NL": (0,), "Q2_0": (0,),
    "Q4_1": (0, 2), "Q5_1": (0, 2), "Q4_K": (0, 2), "Q5_K": (0, 2),
    "Q2_K": (80, 82), "Q3_K": (108,), "Q6_K": (208,),
}


def row_bytes(qtype: int, cols: int) -> int:
    _, qk, b = TYPES[qtype]
    if cols % qk:
        raise ValueError(f"{cols} columns is not a whole number of {qk}-value blocks")
    return cols // qk * b


def random_blocks(qtype: int, rows: int, cols: int, rng: np.random.Generator, scale: float = 1e-3) -> np.ndarray:
    """rows x row_bytes uint8 GGUF rows of format `qtype`."""
    name, qk, tb = TYPES[qtype]
    if name == "BF16":
        v = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.05)).view(np.uint32)
        return (v >> 16).astype(np.uint16).view(np.uint8).reshape(rows, cols * 2)
    nb = rows * (cols // qk)
    raw = rng.integers(0, 256, size=(nb, tb), dtype=np.uint8)
    for off in SCALE_OFFSETS[name]:
        s = (np.abs(rng.standard_normal(nb)) * scale).astype(np.float16)
        raw[:, off:off + 2] = s.view(np.uint8).reshape(nb, 2)
    return raw.reshape(rows, row_bytes(qtype, cols))


# formats whose blocks carry a min beside the scale: (scale offset, min offset, mean quant); the min written as
# mean quant x scale makes a block's expected value zero
CENTER = {"Q4_K": (0, 2, 7.5), "Q5_K": (0, 2, 15.5), "Q2_K": (80, 82, 1.5), "Q4_1": (0, 2, -7.5), "Q5_1": (0, 2, -15.5)}


def model_blocks(qtype: int, rows: int, cols: int, rng: np.random.Generator, scale: float = 1e-3) -> np.ndarray:
    """random_blocks with zero-mean blocks: a random-byte Q4_K row otherwise has a large common offset (its mins), which
    drives every layer's output along one direction, so a model built from such rows predicts the same token and routes
    to the same experts whatever the input."""
    raw = random_blocks(qtype, rows, cols, rng, scale)
    name, _, tb = TYPES[qtype]
    if name in CENTER:
        so, mo, k = CENTER[name]
        r = raw.reshape(-1, tb)
        d = r[:, so:so + 2].copy().view(np.float16).astype(np.float32)
        r[:, mo:mo + 2] = (d * np.float32(k)).astype(np.float16).view(np.uint8)
    return raw


def random_x(nt: int, cols: int, rng: np.random.Generator) -> np.ndarray:
    return rng.standard_normal((nt, cols), dtype=np.float32)


# ---- the synthetic hybrid MoE decoder ---------------------------------------------------------------

def model_config(small: bool = False) -> dict:
    """Config 5 (48 layers, 3 gated-DeltaNet layers then 1 gated-attention layer, MoE on every layer, vocab 151936),
    or a small model of the same structure for parity tests. Formats: a mixed Q4_K / Q6_K / IQ3_XXS recipe (expert
    gate/up IQ3_XXS, everything else Q4_K, the lm_head Q6_K, the router BF16)."""
    if small:
        return dict(D=512, layers=4, pattern="GGGA", vocab=2048, eps=1e-6, nkh=2, nvh=4, nh=4, nkv=1, rope_base=1e7,
                    ne=16, k=4, ffe=256, proj=BY_NAME["Q4_K"], gate_up=BY_NAME["IQ3_XXS"], down=BY_NAME["Q4_K"],
                    embed=BY_NAME["Q4_K"], head=BY_NAME["Q6_K"], router=BY_NAME["BF16"])
    return dict(D=2048, layers=48, pattern="GGGA", vocab=151936, eps=1e-6, nkh=16, nvh=32, nh=16, nkv=2, rope_base=1e7,
                ne=512, k=10, ffe=512, proj=BY_NAME["Q4_K"], gate_up=BY_NAME["IQ3_XXS"], down=BY_NAME["Q4_K"],
                embed=BY_NAME["Q4_K"], head=BY_NAME["Q6_K"], router=BY_NAME["BF16"])


def layer_kind(cfg: dict, l: int) -> str:
    return cfg["pattern"][l % len(cfg["pattern"])]


class BlockPool:
    """Zero-mean random blocks of one format (model_blocks), cut into tensors at random offsets (wrapping): the full
    config-5 expert set (34 GB) then costs the host one pool per format and one copy per tensor, and every tensor no
    larger than the pool still holds distinct blocks."""

    def __init__(self, qtype: int, nblocks: int, rng: np.random.Generator, scale: float = 1e-3):
        _, self.qk, self.tb = TYPES[qtype]
        self.qtype, self.rng = qtype, rng
        self.blocks = model_blocks(qtype, nblocks, self.qk, rng, scale).reshape(nblocks, self.tb)

    def take(self, rows: int, cols: int) -> np.ndarray:
        nb, n = rows * (cols // self.qk), len(self.blocks)
        o = int(self.rng.integers(0, n))
        parts = []
        while nb > 0:
            c = min(nb, n - o)
            parts.append(self.blocks[o:o + c])
            nb, o = nb - c, 0
        return np.concatenate(parts).reshape(rows, row_bytes(self.qtype, cols))


def model_weights(cfg: dict, seed: int = 0, pooled: bool = False, wscale: float = 1e-3) -> dict:
    """Seeded synthetic weights of the config-5 model as GGUF rows (uint8, zero-mean blocks: model_blocks) and fp32
    vectors. DeltaNet projections are stacked as in the reference's load_qw_cat: in = [q | k | v | z] (CONVCH + NVH*128
    rows), ab = [alpha | beta]. The lm_head's scales are 1e-4 (logits of a few units, as a trained head gives).

    pooled: the routed experts' tensors are cut from one BlockPool per format and W["layers"] is a generator (each
    layer made when it is consumed), so the full model never sits in host memory at once.
    wscale: the block scale of every layer's quantised projections and experts (the scale field's mean magnitude);
    1e-3 gives Q4_K elements of rms about 0.13, 2.5e-4 about 0.03, the size of a trained model's weights."""
    rng = np.random.default_rng(seed)
    D = cfg["D"]
    f32 = lambda a: np.asarray(a, np.float32)  # noqa: E731
    W = dict(embed=model_blocks(cfg["embed"], cfg["vocab"], D, rng, scale=1e-2),
             head=model_blocks(cfg["head"], cfg["vocab"], D, rng, scale=1e-4), final_norm=f32(1 + 0.1 * rng.standard_normal(D)))
    pools = None
    if pooled:
        n = cfg["ne"] * cfg["ffe"] * max(D // TYPES[cfg["gate_up"]][1], 1)
        pools = (BlockPool(cfg["gate_up"], n + n // 16, rng, wscale),
                 BlockPool(cfg["down"], cfg["ne"] * D * max(cfg["ffe"] // TYPES[cfg["down"]][1], 1) * 17 // 16, rng,
                           wscale))
    gen = (_model_layer(cfg, l, rng, pools, wscale) for l in range(cfg["layers"]))
    W["layers"] = gen if pooled else list(gen)
    return W


def _model_layer(cfg: dict, l: int, rng: np.random.Generator, pools, wscale: float = 1e-3) -> dict:
    D, DS, HD = cfg["D"], 128, 256
    nkh, nvh, nh, nkv = cfg["nkh"], cfg["nvh"], cfg["nh"], cfg["nkv"]
    convch = 2 * nkh * DS + nvh * DS
    ne, ffe = cfg["ne"], cfg["ffe"]
    P, ws = cfg["proj"], wscale
    f32 = lambda a: np.asarray(a, np.float32)  # noqa: E731
    L = dict(kind=layer_kind(cfg, l), norm1=f32(1 + 0.1 * rng.standard_normal(D)),
             norm2=f32(1 + 0.1 * rng.standard_normal(D)))
    if L["kind"] == "G":
        L.update(w_in=model_blocks(P, convch + nvh * DS, D, rng, ws), w_ab=model_blocks(P, 2 * nvh, D, rng, ws),
                 w_out=model_blocks(P, D, nvh * DS, rng, ws), conv_w=f32(rng.standard_normal((convch, 4)) * 0.5),
                 dt_bias=f32(rng.standard_normal(nvh) * 0.5), ssm_a=f32(-np.exp(rng.standard_normal(nvh) * 0.5)),
                 gnorm=f32(1 + 0.1 * rng.standard_normal(DS)))
    else:
        L.update(w_q=model_blocks(P, nh * 2 * HD, D, rng, ws), w_k=model_blocks(P, nkv * HD, D, rng, ws),
                 w_v=model_blocks(P, nkv * HD, D, rng, ws), w_o=model_blocks(P, D, nh * HD, rng, ws),
                 q_norm=f32(1 + 0.1 * rng.standard_normal(HD)), k_norm=f32(1 + 0.1 * rng.standard_normal(HD)))
    gu, dn = cfg["gate_up"], cfg["down"]
    L["router"] = model_blocks(cfg["router"], ne + 1, D, rng)
    if pools is None:
        routed = [model_blocks(gu, ne * ffe, D, rng, ws), model_blocks(gu, ne * ffe, D, rng, ws),
                  model_blocks(dn, ne * D, ffe, rng, ws)]
    else:
        routed = [pools[0].take(ne * ffe, D), pools[0].take(ne * ffe, D), pools[1].take(ne * D, ffe)]
    L["moe"] = routed + [model_blocks(gu, ffe, D, rng, ws), model_blocks(gu, ffe, D, rng, ws),
                         model_blocks(dn, D, ffe, rng, ws)]
    return L


def rope_inv_freq(base: float, nrot: int = 64) -> np.ndarray:
    """float32 inverse frequencies of the partial RoPE, as the reference computes them (engine/faie2fn.cu:2575)."""
    return np.array([1.0 / base ** (2 * i / nrot) for i in range(nrot // 2)], np.float32)
