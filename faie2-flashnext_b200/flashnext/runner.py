"""GGUF model files for the model-level API: save_model writes a model of the config-5 structure (synth.model_weights)
as a GGUF v3 file; load_model reads one back into that layout (the CPU-side twin of the library's fn_load,
csrc/fn_runner.cu, with the same checks and messages); BatchEngine is forward_batch's runner (the batched entry for
independent sequences on the tensor-core path). The batch-1 model API itself (fn_load / fn_reset / fn_forward /
fn_n_past / fn_last_ms / fn_dev_gb / fn_split / fn_use_graphs / fn_debug_layers / fn_free, engine/faie2fn.cu:2466-2492
and :2680-2740) is the library's.

Files: GGUF v3 (gguf_file.py) with the qwen3next tensor names the reference's loader reads (engine/faie2fn.cu:2617-2657):
token_embd / output / output_norm; per layer blk.N.attn_norm and post_attention_norm; the gated DeltaNet's attn_qkv,
attn_gate, ssm_alpha, ssm_beta, ssm_out, ssm_conv1d, ssm_dt.bias, ssm_a, ssm_norm; the gated attention's attn_q (query
and gate rows interleaved per head), attn_k, attn_v, attn_output, attn_q_norm, attn_k_norm; the MoE's ffn_gate_inp
with ffn_gate_inp_shexp (the shared-expert gate row, stacked under the router as the reference's load_qw_cat does,
:2651), ffn_gate_exps / ffn_up_exps / ffn_down_exps and the shared expert's ffn_gate_shexp / ffn_up_shexp /
ffn_down_shexp. The layer kind comes from which tensors a layer has; the sizes from the tensor shapes; the routed
experts per token from the metadata key <arch>.expert_used_count; eps and the RoPE base from
<arch>.attention.layer_norm_rms_epsilon and <arch>.rope.freq_base. The reference's own model adds tensors this runner
has no kernels for (hyper-connections, the PLE n-gram table, the attention indexer); such files are refused by name.

forward_batch follows forward's contract (:2466-2490) per sequence: 1..8 tokens per call (MAXT, :67), appended at
n_past_batch (an error once it would pass max_ctx), each token's greedy next id returned (and its logits when asked).
"""

from __future__ import annotations

import re
import time

import numpy as np

import gguf_file as gguf
from model import DS, HD, BatchDecodeModel
from synth import TYPES, layer_kind

ARCH = "qwen3next"
MAXT = 8  # tokens per forward call (engine/faie2fn.cu:67)
_UNSUPPORTED = ("hc_", "ple_", "indexer.", "per_layer_token_embd", "output_hc_")


def _layer_specs(cfg: dict, kind: str, T: dict, p: str):
    """(name, ggml type, dims, the tensor's data from the layer dict) of one layer, in file order."""
    D, nkh, nvh, nh, nkv, ne, ffe = cfg["D"], cfg["nkh"], cfg["nvh"], cfg["nh"], cfg["nkv"], cfg["ne"], cfg["ffe"]
    convch = 2 * nkh * DS + nvh * DS
    P, F = cfg["proj"], gguf.GGML_F32
    ty = lambda n: T.get(n, P)  # noqa: E731
    f32 = lambda k: lambda L: np.asarray(L[k], np.float32)  # noqa: E731
    sp = [("attn_norm.weight", F, [D], f32("norm1")), ("post_attention_norm.weight", F, [D], f32("norm2"))]
    if kind == "G":
        sp += [("attn_qkv.weight", ty("w_in"), [D, convch], lambda L: L["w_in"][:convch]),
               ("attn_gate.weight", ty("w_in"), [D, nvh * DS], lambda L: L["w_in"][convch:]),
               ("ssm_alpha.weight", ty("w_ab"), [D, nvh], lambda L: L["w_ab"][:nvh]),
               ("ssm_beta.weight", ty("w_ab"), [D, nvh], lambda L: L["w_ab"][nvh:]),
               ("ssm_out.weight", ty("w_out"), [nvh * DS, D], lambda L: L["w_out"]),
               ("ssm_conv1d.weight", F, [4, convch], f32("conv_w")), ("ssm_dt.bias", F, [nvh], f32("dt_bias")),
               ("ssm_a", F, [nvh], f32("ssm_a")), ("ssm_norm.weight", F, [DS], f32("gnorm"))]
    else:
        sp += [("attn_q.weight", ty("w_q"), [D, nh * 2 * HD], lambda L: L["w_q"]),
               ("attn_k.weight", ty("w_k"), [D, nkv * HD], lambda L: L["w_k"]),
               ("attn_v.weight", ty("w_v"), [D, nkv * HD], lambda L: L["w_v"]),
               ("attn_output.weight", ty("w_o"), [nh * HD, D], lambda L: L["w_o"]),
               ("attn_q_norm.weight", F, [HD], f32("q_norm")), ("attn_k_norm.weight", F, [HD], f32("k_norm"))]
    rt, gu, dn = T.get("router", cfg["router"]), T.get("gate_up", cfg["gate_up"]), T.get("down", cfg["down"])
    sp += [("ffn_gate_inp.weight", rt, [D, ne], lambda L: L["router"][:ne]),
           ("ffn_gate_inp_shexp.weight", rt, [D], lambda L: L["router"][ne:]),
           ("ffn_gate_exps.weight", gu, [D, ffe, ne], lambda L: L["moe"][0]),
           ("ffn_up_exps.weight", gu, [D, ffe, ne], lambda L: L["moe"][1]),
           ("ffn_down_exps.weight", dn, [ffe, D, ne], lambda L: L["moe"][2]),
           ("ffn_gate_shexp.weight", gu, [D, ffe], lambda L: L["moe"][3]),
           ("ffn_up_shexp.weight", gu, [D, ffe], lambda L: L["moe"][4]),
           ("ffn_down_shexp.weight", dn, [ffe, D], lambda L: L["moe"][5])]
    return [(p + n, q, d, g) for n, q, d, g in sp]


def save_model(path: str, cfg: dict, W: dict) -> None:
    """Write a model of the config-5 structure (synth.model_weights layout) as one GGUF v3 file. W["layers"] may be a
    generator (synth.model_weights(pooled=True)): the layers are then written as they are made, in the config's
    formats, so the whole model never sits in host memory."""
    D, V, nh, nkv, nkh, nvh = cfg["D"], cfg["vocab"], cfg["nh"], cfg["nkv"], cfg["nkh"], cfg["nvh"]
    ne, ffe = cfg["ne"], cfg["ffe"]
    layers = W["layers"]
    listed = isinstance(layers, list)
    kinds = [L["kind"] for L in layers] if listed else [layer_kind(cfg, l) for l in range(cfg["layers"])]
    Ts = [L.get("qt", {}) for L in layers] if listed else [{} for _ in kinds]
    meta = {"general.architecture": ARCH, "general.alignment": gguf.ALIGN, f"{ARCH}.block_count": len(kinds),
            f"{ARCH}.embedding_length": D, f"{ARCH}.attention.head_count": nh, f"{ARCH}.attention.head_count_kv": nkv,
            f"{ARCH}.attention.key_length": HD, f"{ARCH}.attention.value_length": HD,
            f"{ARCH}.attention.layer_norm_rms_epsilon": float(cfg["eps"]), f"{ARCH}.rope.freq_base": float(cfg["rope_base"]),
            f"{ARCH}.rope.dimension_count": 64, f"{ARCH}.expert_count": ne, f"{ARCH}.expert_used_count": cfg["k"],
            f"{ARCH}.expert_feed_forward_length": ffe, f"{ARCH}.expert_shared_feed_forward_length": ffe,
            f"{ARCH}.ssm.conv_kernel": 4, f"{ARCH}.ssm.state_size": DS, f"{ARCH}.ssm.group_count": nkh,
            f"{ARCH}.ssm.time_step_rank": nvh, f"{ARCH}.ssm.inner_size": nvh * DS,
            f"{ARCH}.full_attention_interval": len(cfg["pattern"])}
    top = [("token_embd.weight", cfg["embed"], [D, V], lambda: W["embed"]),
           ("output.weight", cfg["head"], [D, V], lambda: W["head"]),
           ("output_norm.weight", gguf.GGML_F32, [D], lambda: np.asarray(W["final_norm"], np.float32))]
    per = [_layer_specs(cfg, k, T, f"blk.{l}.") for l, (k, T) in enumerate(zip(kinds, Ts))]

    def data():
        for *_, get in top:
            yield get()
        for l, L in enumerate(layers):  # a generator is consumed here, once
            if l >= len(per) or L["kind"] != kinds[l] or L.get("qt", {}) != Ts[l]:
                raise gguf.GGUFError(f"layer {l} does not match the config (kind or formats)")
            for *_, get in per[l]:
                yield get(L)

    infos = [(n, q, d) for n, q, d, _ in top] + [(n, q, d) for sp in per for n, q, d, _ in sp]
    gguf.write(path, meta, infos, data())


class _Tensors:
    """The tensors of one or two GGUF shards by name, with shape checks that name the tensor."""

    def __init__(self, paths):
        self.meta, self.t = {}, {}
        for path in paths:
            meta, t = gguf.read(path)
            for k, v in meta.items():
                self.meta.setdefault(k, v)
            for k, v in t.items():
                if k in self.t:
                    raise gguf.GGUFError(f"tensor {k} in more than one shard")
                self.t[k] = v
        self.used = set()

    def has(self, name):
        return name in self.t

    def get(self, name, cols=None, rows=None, quant=True):
        if name not in self.t:
            raise gguf.GGUFError(f"missing tensor {name}")
        t = self.t[name]
        self.used.add(name)
        if cols is not None and t.cols != cols or rows is not None and t.rows != rows:
            raise gguf.GGUFError(f"{name}: shape {list(t.dims)}, expected {cols} columns x {rows} rows")
        if quant and t.qtype not in TYPES:
            raise gguf.GGUFError(f"{name}: ggml type {t.qtype} has no GEMV kernel")
        return t

    def vec(self, name, n, rows=None):
        t = self.get(name, cols=n, rows=rows, quant=False)
        return np.array(t.f32(), np.float32)  # a writable copy (device tensors are made from it)


def load_model(shard1: str, shard2: str | None = None):
    """-> (cfg, W, weight bytes): a GGUF model (one file, or two shards) in the layout model.DecodeModel builds from
    (synth.model_weights' dictionary, plus per-weight formats in W["layers"][l]["qt"])."""
    T = _Tensors([shard1] + ([shard2] if shard2 else []))
    bad = sorted(n for n in T.t if any(n.startswith(u) or ("." + u) in n for u in _UNSUPPORTED))
    if bad:
        raise gguf.GGUFError(f"tensors this runner has no kernels for: {', '.join(bad[:4])}{' ...' if len(bad) > 4 else ''}")
    arch = T.meta.get("general.architecture", ARCH)
    emb = T.get("token_embd.weight")
    D, V = emb.cols, emb.rows
    head = T.get("output.weight", cols=D, rows=V)
    idx = sorted({int(m.group(1)) for n in T.t for m in [re.match(r"blk\.(\d+)\.", n)] if m})
    if not idx or idx != list(range(len(idx))):
        raise gguf.GGUFError("layers blk.0 .. blk.N-1 expected")
    if f"{arch}.expert_used_count" not in T.meta:
        raise gguf.GGUFError(f"missing metadata {arch}.expert_used_count")
    k = int(T.meta[f"{arch}.expert_used_count"])
    W = dict(embed=np.array(emb.rows_u8()), head=head.rows_u8(), final_norm=T.vec("output_norm.weight", D))
    kinds, cfg_t = [], {}
    nkh = nvh = nh = nkv = None
    layers = []
    for l in idx:
        p = f"blk.{l}."
        L = dict(norm1=T.vec(p + "attn_norm.weight", D), norm2=T.vec(p + "post_attention_norm.weight", D), qt={})
        if T.has(p + "attn_q.weight"):
            L["kind"] = "A"
            q = T.get(p + "attn_q.weight", cols=D)
            kv = T.get(p + "attn_k.weight", cols=D)
            if q.rows % (2 * HD) or kv.rows % HD:
                raise gguf.GGUFError(f"{p}attn_q / attn_k: head size {HD} expected")
            nh, nkv = q.rows // (2 * HD), kv.rows // HD
            v = T.get(p + "attn_v.weight", cols=D, rows=nkv * HD)
            o = T.get(p + "attn_output.weight", cols=nh * HD, rows=D)
            L.update(w_q=q.rows_u8(), w_k=kv.rows_u8(), w_v=v.rows_u8(), w_o=o.rows_u8(),
                     q_norm=T.vec(p + "attn_q_norm.weight", HD), k_norm=T.vec(p + "attn_k_norm.weight", HD))
            L["qt"].update(w_q=q.qtype, w_k=kv.qtype, w_v=v.qtype, w_o=o.qtype)
        else:
            L["kind"] = "G"
            a = T.get(p + "ssm_a", quant=False)
            nvh = a.cols
            qkv = T.get(p + "attn_qkv.weight", cols=D)
            if (qkv.rows - nvh * DS) % (2 * DS) or qkv.rows <= nvh * DS:
                raise gguf.GGUFError(f"{p}attn_qkv: {qkv.rows} rows do not fit {nvh} value heads of {DS}")
            nkh = (qkv.rows - nvh * DS) // (2 * DS)
            convch = qkv.rows
            z = T.get(p + "attn_gate.weight", cols=D, rows=nvh * DS)
            al = T.get(p + "ssm_alpha.weight", cols=D, rows=nvh)
            be = T.get(p + "ssm_beta.weight", cols=D, rows=nvh)
            out = T.get(p + "ssm_out.weight", cols=nvh * DS, rows=D)
            if qkv.qtype != z.qtype or al.qtype != be.qtype:
                raise gguf.GGUFError(f"{p}attn_qkv / attn_gate (or ssm_alpha / ssm_beta) in different formats")
            L.update(w_in=np.concatenate([qkv.rows_u8(), z.rows_u8()]), w_ab=np.concatenate([al.rows_u8(), be.rows_u8()]),
                     w_out=out.rows_u8(), conv_w=T.vec(p + "ssm_conv1d.weight", 4, rows=convch),
                     dt_bias=T.vec(p + "ssm_dt.bias", nvh), ssm_a=np.array(a.f32(), np.float32).reshape(nvh),
                     gnorm=T.vec(p + "ssm_norm.weight", DS))
            L["qt"].update(w_in=qkv.qtype, w_ab=al.qtype, w_out=out.qtype)
        r = T.get(p + "ffn_gate_inp.weight", cols=D)
        ne = r.rows
        rs = T.get(p + "ffn_gate_inp_shexp.weight", cols=D, rows=1)
        ge = T.get(p + "ffn_gate_exps.weight", cols=D)
        if ge.rows % ne:
            raise gguf.GGUFError(f"{p}ffn_gate_exps: {ge.rows} rows for {ne} experts")
        ffe = ge.rows // ne
        ue = T.get(p + "ffn_up_exps.weight", cols=D, rows=ne * ffe)
        de = T.get(p + "ffn_down_exps.weight", cols=ffe, rows=ne * D)
        gs = T.get(p + "ffn_gate_shexp.weight", cols=D, rows=ffe)
        us = T.get(p + "ffn_up_shexp.weight", cols=D, rows=ffe)
        ds = T.get(p + "ffn_down_shexp.weight", cols=ffe, rows=D)
        if r.qtype != rs.qtype:
            raise gguf.GGUFError(f"{p}ffn_gate_inp / ffn_gate_inp_shexp in different formats")
        if len({ge.qtype, ue.qtype, gs.qtype, us.qtype}) > 1 or de.qtype != ds.qtype:
            raise gguf.GGUFError(f"{p}expert gate / up (or down) tensors in different formats")
        L["router"] = np.concatenate([r.rows_u8(), rs.rows_u8()])
        L["moe"] = [ge.rows_u8(), ue.rows_u8(), de.rows_u8(), gs.rows_u8(), us.rows_u8(), ds.rows_u8()]
        L["qt"].update(router=r.qtype, gate_up=ge.qtype, down=de.qtype)
        if cfg_t.setdefault("moe", (ne, ffe)) != (ne, ffe):
            raise gguf.GGUFError(f"{p}: expert count or size differs between layers")
        kinds.append(L["kind"])
        layers.append(L)
    if nkh is None or nh is None:
        raise gguf.GGUFError("a model with both gated-DeltaNet and attention layers expected")
    unused = sorted(set(T.t) - T.used)
    if unused:
        raise gguf.GGUFError(f"tensors this runner does not use: {', '.join(unused[:4])}")
    ne, ffe = cfg_t["moe"]
    if not 1 <= k <= min(ne, 16):
        raise gguf.GGUFError(f"{arch}.expert_used_count {k} out of range")
    first = layers[0]["qt"]
    cfg = dict(D=D, layers=len(layers), pattern="".join(kinds), vocab=V,
               eps=float(T.meta.get(f"{arch}.attention.layer_norm_rms_epsilon", 1e-6)), nkh=nkh, nvh=nvh, nh=nh,
               nkv=nkv, rope_base=float(T.meta.get(f"{arch}.rope.freq_base", 1e7)), ne=ne, k=k, ffe=ffe,
               proj=first.get("w_in", first.get("w_q")), gate_up=first["gate_up"], down=first["down"],
               embed=emb.qtype, head=head.qtype, router=first["router"])
    W["layers"] = layers
    nbytes = sum(t.data.nbytes for t in T.t.values())
    return cfg, W, nbytes


class BatchEngine:
    """forward_batch's runner (the batched entry for independent sequences, which the reference lacks): the GGUF model
    loaded again into the tensor-core BatchDecodeModel on the current GPU, `batch` sequences stepping together from
    position n_past_batch. The batch-1 model API is the library's (fn_load .. fn_free, csrc/fn_runner.cu)."""

    def __init__(self, fn, shard1: str, shard2: str | None = None, max_ctx: int = 32768, batch: int = 8):
        import torch
        if max_ctx < 1:
            raise RuntimeError("max_ctx out of range")
        if not 1 <= batch <= 32:
            raise RuntimeError("batch out of range (1..32)")
        try:
            cfg, W, _ = load_model(shard1, shard2)
        except (OSError, gguf.GGUFError) as e:
            raise RuntimeError(str(e)) from e
        self.cfg, self.fn, self.max_ctx = cfg, fn, max_ctx
        self.n_past_batch, self.last_ms, self.use_graphs, self.blg = 0, -1.0, True, None
        self.stream = torch.cuda.Stream()
        try:
            self.bmodel = BatchDecodeModel(fn, cfg, W, batch, max_ctx=max_ctx)
        except ValueError as e:
            raise RuntimeError(str(e)) from e
        self.bmodel.capture(self.stream)
        self.bam = torch.zeros(MAXT, batch, dtype=torch.int32).pin_memory()
        self.reset()

    def reset(self):
        """fn_reset for the batched sequences: their DeltaNet states and conv histories zeroed, position 0."""
        import torch
        b = self.bmodel
        with torch.cuda.stream(self.stream):
            b.tokens.zero_()
            b.pos.zero_()
            b.plen.zero_()
        for g in b.gdns:
            self.fn.gdn_reset(g, self.stream.cuda_stream)
        self.fn.sync(self.stream.cuda_stream)
        self.n_past_batch = 0

    def forward_batch(self, tokens, logits=None, argmax=None):
        """tokens int32 [batch][nt] (nt 1..8), one row per sequence, all sequences at position n_past_batch (their own
        states and caches); argmax[b][i] = sequence b's greedy next id after its token i, logits[b][i] its logits
        (tensor-core GEMVs: within 1e-4 of max |y| per projection of the CUDA-core path). forward's errors, plus a
        shape check."""
        import torch
        b = self.bmodel
        t = np.ascontiguousarray(tokens, np.int32)
        if t.ndim != 2 or t.shape[0] != b.B:
            raise RuntimeError(f"tokens must be [{b.B}][nt]")
        nt = t.shape[1]
        if nt < 1 or nt > MAXT:
            raise RuntimeError("nt out of range")
        if self.n_past_batch + nt > self.max_ctx:
            raise RuntimeError("context full")
        if t.min() < 0 or t.max() >= self.cfg["vocab"]:
            raise RuntimeError("token id out of range")
        if logits is not None and self.blg is None:
            self.blg = torch.zeros(MAXT, b.B, self.cfg["vocab"], dtype=torch.float32).pin_memory()
        t0 = time.perf_counter()
        s, n = self.stream, self.n_past_batch
        with torch.cuda.stream(s):
            b.tokens[:, n:n + nt].copy_(torch.from_numpy(t))
            b.plen.fill_(n + nt)
            for i in range(nt):
                if self.use_graphs:
                    b.graph.replay()
                else:
                    b.launch_step(s.cuda_stream)
                self.bam[i].copy_(b.next, non_blocking=True)
                if logits is not None:
                    self.blg[i].copy_(b.logits, non_blocking=True)
        self.fn.sync(s.cuda_stream)
        if argmax is not None:
            argmax[:, :nt] = self.bam[:nt].numpy().T
        if logits is not None:
            logits[:, :nt] = self.blg[:nt].numpy().transpose(1, 0, 2)
        self.n_past_batch += nt
        self.last_ms = (time.perf_counter() - t0) * 1e3
        return 0

    def free(self):
        self.bmodel.free()
