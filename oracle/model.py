"""CPU oracle for a whole decode step of the synthetic hybrid MoE.  TEST INFRASTRUCTURE ONLY.

Float64 restatement of the reference's decode forward for this model (engine/faie2fn.cu layer_forward, :2380-2447;
the reference's own oracle is ref_fn.py's float64 transformers forward over dequantised GGUF weights, :123-215), one
token at a time:
  embed      h = dequant(E[token])                                               (k_embed, :1334-1347)
  per layer  x = rmsnorm(h) * norm1                                              (k_groupnorm, :1222-1235)
             DeltaNet layer: [qkv | z] = W_in x, [alpha | beta] = W_ab x, o = gdn_step(...) (oracle/gdn.py),
                             h += W_out o                                        (:2386-2390)
             attention layer: [q_h | gate_h] = W_q x, k = W_k x, v = W_v x; q, k per head rmsnorm * w, RoPE on the
                             first 64 dims (pairs i, i + 32, angle pos * inv_freq[i]); k, v appended to the cache;
                             o_h = softmax(q_h . K / 16) V (kv head h / (NH / NKV)) * sigmoid(gate_h); h += W_o o
                             (k_qk_norm_rope, k_attn_split, k_attn_combine, :1452-1478, 1598-1690; no QSA indexer)
             x2 = rmsnorm(h) * norm2; logits_r = W_r x2 (row ne: the shared-expert gate); h += moe(x2) (oracle/moe.py)
  head       logits = W_head (rmsnorm(h) * final_norm)                           (:2446)
All weights are the exactly dequantised GGUF values (oracle/dequant.py); everything else is float64. The RoPE
frequencies are the float32 values the reference uploads (:2575), used exactly.
"""

from __future__ import annotations

import numpy as np

from . import dequant as D
from . import gdn as G
from . import moe as M

DS, HD, NROT = 128, 256, 64


def rmsnorm(x, w, eps):
    x = np.asarray(x, np.float64)
    return x / np.sqrt((x * x).mean() + eps) * np.asarray(w, np.float64)


def sigmoid(v):
    return 1.0 / (1.0 + np.exp(-v))


def rope(x, pos, inv_freq):
    """Partial RoPE on the last axis: dims (i, i + 32) for i < 32 rotated by pos * inv_freq[i] (k_qk_norm_rope,
    engine/faie2fn.cu:1452-1478); dims 64.. unchanged."""
    y = np.array(x, np.float64, copy=True)
    ang = pos * np.asarray(inv_freq, np.float64)
    c, s = np.cos(ang), np.sin(ang)
    x0, x1 = y[..., :NROT // 2].copy(), y[..., NROT // 2:NROT].copy()
    y[..., :NROT // 2] = x0 * c - x1 * s
    y[..., NROT // 2:NROT] = x1 * c + x0 * s
    return y


def gated_attention(qg, k, v, q_norm, k_norm, inv_freq, pos, cache, nh, nkv, eps):
    """One token of the gated-attention layer at position pos: qg [nh][2 HD] (q, then the gate), k, v [nkv][HD]. q and
    k are RMS-normed per head and rotated; k and v are appended to cache = (K list, V list); returns o [nh * HD] =
    softmax(q . K / 16) V * sigmoid(gate), q head h reading kv head h / (nh / nkv) (k_attn_split / k_attn_combine,
    engine/faie2fn.cu:1598-1690)."""
    qg = np.asarray(qg, np.float64).reshape(nh, 2 * HD)
    q, gate = qg[:, :HD], qg[:, HD:]
    k = np.asarray(k, np.float64).reshape(nkv, HD)
    v = np.asarray(v, np.float64).reshape(nkv, HD)
    qn = np.stack([rmsnorm(q[i], q_norm, eps) for i in range(nh)])
    kn = np.stack([rmsnorm(k[i], k_norm, eps) for i in range(nkv)])
    cache[0].append(rope(kn, pos, inv_freq))
    cache[1].append(v)
    K, V = np.stack(cache[0]), np.stack(cache[1])  # [n][nkv][HD]
    qr = rope(qn, pos, inv_freq)
    o = np.empty((nh, HD))
    for i in range(nh):
        kv = i // (nh // nkv)
        sc = K[:, kv] @ qr[i] / 16.0
        p = np.exp(sc - sc.max())
        o[i] = (p / p.sum()) @ V[:, kv] * sigmoid(gate[i])
    return o.reshape(-1), qr


class _LazyRows:
    """GGUF rows dequantised (to float64) one at a time when indexed, for an embedding table of any vocabulary."""

    def __init__(self, raw, qtype, cols):
        self.raw, self.qtype, self.cols = raw, qtype, cols

    def __getitem__(self, i):
        return D.dequant_rows(self.raw[int(i):int(i) + 1], self.qtype, 1, self.cols)[0].astype(np.float64)


class OracleModel:
    """The float64 model of a config dict and its weights (flashnext/synth.py model_config / model_weights)."""

    @classmethod
    def from_dense(cls, cfg: dict, dense: dict, inv_freq: np.ndarray):
        """The same model over float weights given directly (no GGUF rows): dense has E [vocab][D], Hd [vocab][D],
        final_norm, and layers, each a dict of the keys step() reads (norm1, norm2; w_in, w_ab, w_out, conv_w,
        dt_bias, ssm_a, gnorm or w_q, w_k, w_v, w_o, q_norm, k_norm; router [ne + 1][D]; experts = (gate, up, down
        [ne][..], shared gate, up, down))."""
        o = cls.__new__(cls)
        o.cfg, o.W = cfg, dict(final_norm=dense["final_norm"], layers=dense["layers"])
        o.inv_freq = np.asarray(inv_freq, np.float64)
        o.E, o.Hd = np.asarray(dense["E"], np.float64), np.asarray(dense["Hd"], np.float64)
        o.L = [dict(L) for L in dense["layers"]]
        o.reset()
        return o

    def __init__(self, cfg: dict, W: dict, inv_freq: np.ndarray):
        self.cfg, self.W = cfg, W
        d = cfg["D"]
        self.inv_freq = np.asarray(inv_freq, np.float32).astype(np.float64)
        deq = lambda raw, t, r, c: D.dequant_rows(raw, t, r, c).astype(np.float64)  # noqa: E731
        self.E = _LazyRows(W["embed"], cfg["embed"], d)  # only the rows of the tokens stepped are dequantised
        self.Hd = deq(W["head"], cfg["head"], cfg["vocab"], d)
        nkh, nvh, nh, nkv = cfg["nkh"], cfg["nvh"], cfg["nh"], cfg["nkv"]
        convch = 2 * nkh * DS + nvh * DS
        P, ne, ffe = cfg["proj"], cfg["ne"], cfg["ffe"]
        self.L = []
        for L in W["layers"]:
            o = dict(kind=L["kind"], norm1=L["norm1"], norm2=L["norm2"])
            T = L.get("qt", {})  # per-weight formats (a GGUF file's tensor types); default: the config's
            ty = lambda n, T=T: T.get(n, P)  # noqa: E731
            if L["kind"] == "G":
                o.update(w_in=deq(L["w_in"], ty("w_in"), convch + nvh * DS, d), w_ab=deq(L["w_ab"], ty("w_ab"), 2 * nvh, d),
                         w_out=deq(L["w_out"], ty("w_out"), d, nvh * DS), conv_w=L["conv_w"], dt_bias=L["dt_bias"],
                         ssm_a=L["ssm_a"], gnorm=L["gnorm"])
            else:
                o.update(w_q=deq(L["w_q"], ty("w_q"), nh * 2 * HD, d), w_k=deq(L["w_k"], ty("w_k"), nkv * HD, d),
                         w_v=deq(L["w_v"], ty("w_v"), nkv * HD, d), w_o=deq(L["w_o"], ty("w_o"), d, nh * HD),
                         q_norm=L["q_norm"], k_norm=L["k_norm"])
            gu, dn = T.get("gate_up", cfg["gate_up"]), T.get("down", cfg["down"])
            Wg, Wu, Wd, Wsg, Wsu, Wsd = L["moe"]
            o.update(router=deq(L["router"], T.get("router", cfg["router"]), ne + 1, d),
                     experts=(M.GGUFExperts(Wg, gu, ffe, d), M.GGUFExperts(Wu, gu, ffe, d), M.GGUFExperts(Wd, dn, d, ffe),
                              deq(Wsg, gu, ffe, d), deq(Wsu, gu, ffe, d), deq(Wsd, dn, d, ffe)))
            self.L.append(o)
        self.reset()

    def reset(self):
        cfg = self.cfg
        nkh, nvh = cfg["nkh"], cfg["nvh"]
        convch = 2 * nkh * DS + nvh * DS
        self.pos = 0
        self.state = []
        for L in self.L:
            if L["kind"] == "G":
                self.state.append(dict(S=np.zeros((nvh, DS, DS)), cs=np.zeros((3, convch))))
            else:
                self.state.append(dict(K=[], V=[]))

    def step(self, token: int) -> np.ndarray:
        """One decode step at the current position; returns the float64 logits (the residual stream before the final
        norm is left in self.h) and advances the position."""
        cfg, eps = self.cfg, self.cfg["eps"]
        nkh, nvh, nh, nkv = cfg["nkh"], cfg["nvh"], cfg["nh"], cfg["nkv"]
        convch = 2 * nkh * DS + nvh * DS
        h = self.E[token].copy()
        for L, st in zip(self.L, self.state):
            x = rmsnorm(h, L["norm1"], eps)
            if L["kind"] == "G":
                v = L["w_in"] @ x
                o = G.gdn_step(v[:convch], v[convch:], L["w_ab"] @ x, L["conv_w"], L["dt_bias"], L["ssm_a"], L["gnorm"],
                               st["S"], st["cs"], nkh, nvh, DS)
                h = h + L["w_out"] @ o
            else:
                o, _ = gated_attention(L["w_q"] @ x, L["w_k"] @ x, L["w_v"] @ x, L["q_norm"], L["k_norm"], self.inv_freq,
                                       self.pos, (st["K"], st["V"]), nh, nkv, eps)
                h = h + L["w_o"] @ o
            x2 = rmsnorm(h, L["norm2"], eps)
            logits_r = L["router"] @ x2
            y, _, _ = M.moe_layer(x2[None], logits_r[None], cfg["k"], *L["experts"])
            h = h + y[0]
            if getattr(self, "trace", None) is not None:  # the residual after every layer, when asked
                self.trace.append(h.copy())
        self.pos += 1
        self.h = h
        return self.Hd @ rmsnorm(h, self.W["final_norm"], eps)
