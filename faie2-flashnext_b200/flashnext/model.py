"""The synthetic hybrid MoE decoder of BASELINE config 5 on the engine: one decode step as one CUDA graph.

The model (flashnext/synth.py model_config / model_weights): token embedding, then per layer an RMSNorm, a gated
DeltaNet layer (three of every four layers) or a gated-attention layer, a residual add, an RMSNorm and the MoE layer
(routed experts + gated shared expert) with its residual add; a final RMSNorm and the lm_head with its argmax. Every
piece is an engine kernel behind the C ABI (fn.py); the residual adds are the accumulate flag of the projection GEMVs
and of the MoE layer. The step's position and the token ids live in device memory (fn_step_advance feeds the argmax
back as the next input once the prompt is consumed), so a whole generation is the step's graph replayed once per
token with no host work in between (the reference's fn_forward, engine/faie2fn.cu:2733, runs the same loop with the
host feeding tokens).
"""

from __future__ import annotations

import numpy as np

from synth import rope_inv_freq

DS, HD = 128, 256


class DecodeModel:
    def __init__(self, fn, cfg: dict, W: dict, max_ctx: int = 512, logits: bool = False, warps: int = 16,
                 stack: bool = True, prefetch: bool = True, fuse_norm: bool = True):
        """warps: GEMV warps per CTA of the model's weights; stack: the projections that read the same input as one
        GEMV each ([q k v z | alpha beta], [q gate | k | v]) rather than one GEMV per weight; prefetch: each
        projection brings the step's next dense weight into L2 while it runs (input -> output projection -> router,
        the MoE layer -> the next layer's input projection); fuse_norm: every RMSNorm folded into the GEMVs and MoE
        layer that read its output (fn_w_norm / fn_moe_norm: no norm launches) rather than run as its own kernel."""
        import torch
        self.fn, self.cfg, self.max_ctx = fn, cfg, max_ctx
        self.stack, self.fuse_norm = stack, fuse_norm
        dev = torch.device("cuda", torch.cuda.current_device())
        f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
        nkh, nvh, nh, nkv = cfg["nkh"], cfg["nvh"], cfg["nh"], cfg["nkv"]
        self.convch = 2 * nkh * DS + nvh * DS
        self.n_in = self.convch + nvh * DS + 2 * nvh  # q k v | z | alpha beta
        self.n_qkv = nh * 2 * HD + 2 * nkv * HD  # q gate | k | v
        self.handles, self.moes, self.gdns = [], [], []
        # a decode step is a chain of dependent GEMVs at batch 1: each is latency-bound, so its CTAs run 16 warps
        # (more loads and decodes in flight per SM) rather than the few that let independent GEMVs share an SM
        fn.gemv_tune(warps=warps)
        try:
            self._build(fn, cfg, W, max_ctx, logits, dev, f32)
        except BaseException:
            self.free()  # a weight the engine refused: release what was uploaded before it
            raise
        finally:
            fn.gemv_tune(warps=0)
        try:
            self._create_decoder(prefetch, fuse_norm)
        except BaseException:
            self.free()
            raise

    def _create_decoder(self, prefetch, fuse_norm):
        """The step itself is the library's (fn_decoder_create / fn_decoder_step, csrc/fn_decoder.cu): the handles and
        buffers built here, described as fn_model_t / fn_layer_t."""
        import ctypes as C
        from fn import FnLayer, FnModel
        fn, cfg = self.fn, self.cfg
        p = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
        Ls = (FnLayer * len(self.layers))()
        for o, L in zip(Ls, self.layers):
            w_in = L["w_in"] if L["kind"] == "G" else L["w_qkv"]
            ins = w_in if isinstance(w_in, list) else [(w_in, self.n_in if L["kind"] == "G" else self.n_qkv)]
            o.kind = 0 if L["kind"] == "G" else 1
            for i, (h, rows) in enumerate(ins):
                o.w_in[i], o.w_in_rows[i] = h, rows
            o.w_out = L["w_out"] if L["kind"] == "G" else L["w_o"]
            o.gdn = L.get("gdn", 0)
            o.router, o.moe = L["router"], L["moe"]
            o.norm1, o.norm2 = p(L["norm1"]), p(L["norm2"])
            if L["kind"] == "A":
                o.q_norm, o.k_norm, o.Kc, o.Vc = p(L["q_norm"]), p(L["k_norm"]), p(L["Kc"]), p(L["Vc"])
        m = FnModel(D=cfg["D"], nkh=cfg["nkh"], nvh=cfg["nvh"], nh=cfg["nh"], nkv=cfg["nkv"], ne=cfg["ne"],
                    vocab=cfg["vocab"], max_ctx=self.max_ctx, eps=cfg["eps"], embed_type=cfg["embed"], embed=p(self.E),
                    head=self.head, final_norm=p(self.final_norm), inv_freq=p(self.inv_freq),
                    fuse_norm=int(fuse_norm), prefetch=int(prefetch), hidden=p(self.h), xnorm=p(self.x),
                    proj=p(self.proj), core=p(self.core), Q=p(self.Q), att=p(self.att), router_out=p(self.lr),
                    logits=p(self.logits), tokens=p(self.tokens), pos=p(self.pos), next=p(self.next),
                    prompt_len=p(self.plen))
        h = fn.d.fn_decoder_create(C.byref(m), Ls, len(self.layers))
        if h < 0:
            raise RuntimeError(fn.d.fn_error().decode())
        self.dec = h

    def _build(self, fn, cfg, W, max_ctx, logits, dev, f32):
        import torch
        d, nkh, nvh, nh, nkv = cfg["D"], cfg["nkh"], cfg["nvh"], cfg["nh"], cfg["nkv"]
        ne, ffe, P = cfg["ne"], cfg["ffe"], cfg["proj"]
        self.E = torch.from_numpy(np.ascontiguousarray(W["embed"]).reshape(-1)).to(dev)
        self.head = self._w(cfg["head"], W["head"], cfg["vocab"], d)
        self.final_norm = f32(W["final_norm"])
        self.inv_freq = f32(rope_inv_freq(cfg["rope_base"]))
        self.layers = []
        for L in W["layers"]:
            # per-weight formats (a GGUF file's own tensor types, flashnext/runner.py); default: the config's
            T = L.get("qt", {})
            ty = lambda n, T=T: T.get(n, P)  # noqa: E731
            o = dict(kind=L["kind"], norm1=f32(L["norm1"]), norm2=f32(L["norm2"]),
                     router=self._w(T.get("router", cfg["router"]), L["router"], ne + 1, d))
            if L["kind"] == "G":  # [q k v z | alpha beta]: one GEMV over the stacked rows (when one format)
                if self.stack and ty("w_in") == ty("w_ab"):
                    o["w_in"] = self._w(ty("w_in"), np.concatenate([L["w_in"], L["w_ab"]]), self.n_in, d)
                else:
                    o["w_in"] = [(self._w(ty("w_in"), L["w_in"], self.convch + nvh * DS, d), self.convch + nvh * DS),
                                 (self._w(ty("w_ab"), L["w_ab"], 2 * nvh, d), 2 * nvh)]
                o["w_out"] = self._w(ty("w_out"), L["w_out"], d, nvh * DS)
                g = fn.gdn_create(nkh, nvh, L["conv_w"], L["dt_bias"], L["ssm_a"], L["gnorm"],
                                  np.zeros((nvh, DS, DS), np.float32), np.zeros((3, self.convch), np.float32))
                self.gdns.append(g)
                o["gdn"] = g
            else:
                one = ty("w_q") == ty("w_k") == ty("w_v")
                o.update(w_qkv=self._w(ty("w_q"), np.concatenate([L["w_q"], L["w_k"], L["w_v"]]), self.n_qkv, d)
                         if self.stack and one
                         else [(self._w(ty(n), L[n], r, d), r) for n, r in (("w_q", nh * 2 * HD), ("w_k", nkv * HD),
                                                                               ("w_v", nkv * HD))],
                         w_o=self._w(ty("w_o"), L["w_o"], d, nh * HD),
                         q_norm=f32(L["q_norm"]), k_norm=f32(L["k_norm"]),
                         Kc=torch.zeros(max_ctx, nkv, HD, device=dev), Vc=torch.zeros(max_ctx, nkv, HD, device=dev))
            m = fn.moe_create(T.get("gate_up", cfg["gate_up"]), T.get("down", cfg["down"]), ne, cfg["k"], ffe, d, *L["moe"])
            self.moes.append(m)
            o["moe"] = m
            self.layers.append(o)
        z = lambda n: torch.zeros(n, device=dev)  # noqa: E731
        self.h, self.x, self.proj = z(d), z(d), z(max(self.n_in, self.n_qkv))
        self.core = z(nvh * DS)
        self.Q, self.att, self.lr = z(nh * HD), z(nh * HD), z(ne + 1)
        self.logits = z(cfg["vocab"]) if logits else None
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.next = torch.zeros(1, dtype=torch.int32, device=dev)
        self.tokens = torch.zeros(max_ctx, dtype=torch.int32, device=dev)
        self.plen = torch.zeros(1, dtype=torch.int32, device=dev)
        self.graph = None

    def _w(self, qtype, raw, rows, cols):
        h = self.fn.w_create(qtype, raw, rows, cols)
        self.handles.append(h)
        return h

    def launch_step(self, s: int, dbg=None):
        """Launch one decode step on stream s (device pointers only; capturable). dbg (host float32 [layers][D],
        eager steps only): the residual after every layer."""
        import ctypes as C
        self.fn.check(self.fn.d.fn_decoder_step(self.dec, C.c_void_p(s), dbg.ctypes.data if dbg is not None else None,
                                                self.cfg["D"]))

    def launches_per_step(self) -> int:
        """Kernel launches of one step: the embedding; per layer the input GEMV(s), the DeltaNet core or the two
        attention kernels, the output GEMV, the router GEMV and the MoE layer's two kernels (three with a routing
        kernel, fn_moe_var(0)), plus two norms unless they are folded; the lm_head with its argmax and the step
        counter (and the final norm unless folded)."""
        n = self.fn.d.fn_decoder_launches(self.dec)
        if n < 0:
            raise RuntimeError(self.fn.d.fn_error().decode())
        return n

    def start(self, prompt, stream=None):
        """A new sequence: the prompt loaded, the position at 0, the DeltaNet states and conv histories zeroed (the
        attention caches need no reset: a step reads positions 0..pos only)."""
        import torch
        prompt = np.asarray(prompt, np.int32)
        if not 1 <= len(prompt) <= self.max_ctx:
            raise ValueError("prompt length out of range")
        s = stream or torch.cuda.current_stream()
        with torch.cuda.stream(s):
            self.tokens.zero_()
            self.tokens[:len(prompt)] = torch.from_numpy(prompt).to(self.tokens.device)
            self.pos.zero_()
            self.plen.fill_(len(prompt))
        for g in self.gdns:
            self.fn.gdn_reset(g, s.cuda_stream)

    def capture(self, stream):
        """Capture one step as a CUDA graph on `stream` (one step runs first, outside the capture, to set the kernels'
        attributes: call start() afterwards)."""
        import torch
        self.start([0], stream)
        self.launch_step(stream.cuda_stream)
        self.fn.sync(stream.cuda_stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
            self.launch_step(torch.cuda.current_stream().cuda_stream)
        self.graph = g

    def generate_host(self, prompt, n_new, out, stream, marks=None):
        """Greedy decode on host buffers, everything on `stream` (nothing synchronises): prompt (int32 host tensor,
        pinned for an asynchronous copy) is copied in, the states reset, the step's graph replayed once per position,
        and the ids of the n_new generated tokens copied out into out (int32 host tensor, pinned). marks: optional
        CUDA events recorded after the reset, after the last prompt-only step and after the last step."""
        import torch
        if self.graph is None:
            raise RuntimeError("capture() the step first")
        n = len(prompt)
        if not 1 <= n or n + n_new > self.max_ctx or n_new < 1:
            raise ValueError("prompt + new tokens exceed the context")
        with torch.cuda.stream(stream):  # copies, resets and replays all go to `stream`
            self.tokens.zero_()
            self.tokens[:n].copy_(prompt, non_blocking=True)
            self.pos.zero_()
            self.plen.fill_(n)
            for g in self.gdns:
                self.fn.gdn_reset(g, stream.cuda_stream)
            if marks:
                marks[0].record(stream)
            for i in range(n + n_new - 1):
                if marks and i == n - 1:
                    marks[1].record(stream)
                self.graph.replay()
            if marks:
                marks[2].record(stream)
            out[:n_new].copy_(self.tokens[n:n + n_new], non_blocking=True)

    def generate(self, prompt, n_new, stream):
        """Greedy decode: the prompt, then n_new tokens; returns the token ids of all positions (device replays only)."""
        import torch
        prompt = torch.from_numpy(np.asarray(prompt, np.int32)).pin_memory()
        out = torch.zeros(n_new, dtype=torch.int32).pin_memory()
        self.generate_host(prompt, n_new, out, stream)
        self.fn.sync(stream.cuda_stream)
        return np.concatenate([prompt.numpy(), out.numpy()])

    def free(self):
        self.graph = None
        if getattr(self, "dec", 0):
            self.fn.d.fn_decoder_free(self.dec)
            self.dec = 0
        for h in self.handles:
            self.fn.w_free(h)
        for m in self.moes:
            self.fn.moe_free(m)
        for g in self.gdns:
            self.fn.gdn_free(g)
        self.handles, self.moes, self.gdns = [], [], []


class BatchDecodeModel:
    """Batched decode of the same model: `batch` (1..32) independent sequences step together at one position, every
    projection, router and lm_head on the tensor cores (fn_tc_gemv: each weight tile dequantised once for all the
    batch's tokens), the MoE layer for all the batch's tokens in one call, one DeltaNet state and one attention cache per
    sequence. The argmax of each sequence's logits feeds its next input, so a generation is again one CUDA graph
    replayed per position. Results are those of DecodeModel within the tensor-core GEMV's tolerance (1e-4 of max |y|
    per projection)."""

    def __init__(self, fn, cfg: dict, W: dict, batch: int, max_ctx: int = 512):
        import torch
        if not 1 <= batch <= 32:
            raise ValueError("batch out of range (1..32)")
        self.fn, self.cfg, self.B, self.max_ctx = fn, cfg, batch, max_ctx
        dev = torch.device("cuda", torch.cuda.current_device())
        f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
        d, nkh, nvh, nh, nkv = cfg["D"], cfg["nkh"], cfg["nvh"], cfg["nh"], cfg["nkv"]
        ne, ffe, P = cfg["ne"], cfg["ffe"], cfg["proj"]
        self.convch = 2 * nkh * DS + nvh * DS
        self.n_in = self.convch + nvh * DS + 2 * nvh
        self.n_qkv = nh * 2 * HD + 2 * nkv * HD
        self.tcs, self.moes, self.gdns = [], [], []
        tc = lambda q, raw, r, c: self._tc(q, raw, r, c)  # noqa: E731
        self.E = torch.from_numpy(np.ascontiguousarray(W["embed"]).reshape(-1)).to(dev)
        self.head = tc(cfg["head"], W["head"], cfg["vocab"], d)
        self.final_norm = f32(W["final_norm"])
        self.inv_freq = f32(rope_inv_freq(cfg["rope_base"]))
        self.layers = []
        B = batch
        for L in W["layers"]:
            T = L.get("qt", {})  # per-weight formats, as DecodeModel; a weight stacked into one projection needs one
            ty = lambda n, T=T: T.get(n, P)  # noqa: E731
            if len({ty(n) for n in (("w_in", "w_ab") if L["kind"] == "G" else ("w_q", "w_k", "w_v"))}) > 1:
                self.free()  # (W["layers"] may be a generator: checked layer by layer, what was built is released)
                raise ValueError("batched decode: the weights stacked into one projection need one format")
            o = dict(kind=L["kind"], norm1=f32(L["norm1"]), norm2=f32(L["norm2"]),
                     router=tc(T.get("router", cfg["router"]), L["router"], ne + 1, d))
            if L["kind"] == "G":
                o["w_in"] = tc(ty("w_in"), np.concatenate([L["w_in"], L["w_ab"]]), self.n_in, d)
                o["w_out"] = tc(ty("w_out"), L["w_out"], d, nvh * DS)
                g = fn.gdn_create_batch(nkh, nvh, L["conv_w"], L["dt_bias"], L["ssm_a"], L["gnorm"], B)
                self.gdns.append(g)
                o["gdn"] = g
            else:
                o.update(w_qkv=tc(ty("w_q"), np.concatenate([L["w_q"], L["w_k"], L["w_v"]]), self.n_qkv, d),
                         w_o=tc(ty("w_o"), L["w_o"], d, nh * HD), q_norm=f32(L["q_norm"]), k_norm=f32(L["k_norm"]),
                         Kc=torch.zeros(B, max_ctx, nkv, HD, device=dev), Vc=torch.zeros(B, max_ctx, nkv, HD, device=dev))
            m = fn.moe_create(T.get("gate_up", cfg["gate_up"]), T.get("down", cfg["down"]), ne, cfg["k"], ffe, d, *L["moe"])
            self.moes.append(m)
            o["moe"] = m
            self.layers.append(o)
        z = lambda *n: torch.zeros(*n, device=dev)  # noqa: E731
        self.h, self.x, self.proj = z(B, d), z(B, d), z(B, max(self.n_in, self.n_qkv))
        self.core, self.Q, self.att, self.lr = z(B, nvh * DS), z(B, nh * HD), z(B, nh * HD), z(B, ne + 1)
        self.logits = z(B, cfg["vocab"])
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.next = torch.zeros(B, dtype=torch.int32, device=dev)
        self.tokens = torch.zeros(B, max_ctx, dtype=torch.int32, device=dev)
        self.plen = torch.zeros(1, dtype=torch.int32, device=dev)
        self.graph = None

    def _tc(self, qtype, raw, rows, cols):
        h = self.fn.tc_create(qtype, raw, rows, cols)
        self.tcs.append(h)
        return h

    def launches_per_step(self) -> int:
        """The embedding; per layer two norms, the input GEMV, the DeltaNet core or the two attention kernels, the output
        GEMV, the router GEMV and the MoE layer's three kernels; the final norm, the lm_head, the argmax and the step
        counter."""
        moe = 3
        return 1 + sum(2 + 1 + (1 if L["kind"] == "G" else 2) + 1 + 1 + moe for L in self.layers) + 4

    def launch_step(self, s: int):
        """One decode step of every sequence on stream s (device pointers only; capturable)."""
        fn, cfg, B = self.fn, self.cfg, self.B
        d, nvh, nh, nkv, eps, ne1 = cfg["D"], cfg["nvh"], cfg["nh"], cfg["nkv"], cfg["eps"], cfg["ne"] + 1
        p = lambda t: t.data_ptr()  # noqa: E731
        h, x, pr = p(self.h), p(self.x), p(self.proj)
        ps = self.proj.shape[1]
        fn.embed_batch(cfg["embed"], p(self.E), d, p(self.tokens), self.max_ctx, p(self.pos), h, B, s)
        for L in self.layers:
            fn.rmsnorm_rows(h, p(L["norm1"]), x, d, B, eps, s)
            if L["kind"] == "G":
                fn.tc_gemv(L["w_in"], x, d, pr, ps, B, 0, s)
                fn.gdn_run_batch(L["gdn"], pr, ps, pr + 4 * self.convch, ps, pr + 4 * (self.convch + nvh * DS), ps,
                                 p(self.core), nvh * DS, 1, s)
                fn.tc_gemv(L["w_out"], p(self.core), nvh * DS, h, d, B, 1, s)  # h += W_out core
            else:
                fn.tc_gemv(L["w_qkv"], x, d, pr, ps, B, 0, s)
                fn.attn_decode_batch(pr, pr + 4 * nh * 2 * HD, pr + 4 * (nh * 2 * HD + nkv * HD), ps, p(L["q_norm"]),
                                     p(L["k_norm"]), p(self.inv_freq), p(self.Q), p(L["Kc"]), p(L["Vc"]), p(self.att),
                                     p(self.pos), nh, nkv, self.max_ctx, B, eps, s)
                fn.tc_gemv(L["w_o"], p(self.att), nh * HD, h, d, B, 1, s)  # h += W_o o
            fn.rmsnorm_rows(h, p(L["norm2"]), x, d, B, eps, s)
            fn.tc_gemv(L["router"], x, d, p(self.lr), ne1, B, 0, s)
            fn.moe_run(L["moe"], p(self.lr), ne1, x, h, B, 1, s)  # every sequence's token in one call; h += moe(x)
        fn.rmsnorm_rows(h, p(self.final_norm), x, d, B, eps, s)
        vocab = cfg["vocab"]
        fn.tc_gemv(self.head, x, d, p(self.logits), vocab, B, 0, s)
        fn.argmax_dev(p(self.logits), vocab, vocab, B, p(self.next), s)
        fn.step_advance_batch(p(self.pos), p(self.tokens), p(self.next), p(self.plen), self.max_ctx, B, s)

    def start(self, prompts, stream):
        """New sequences: prompts [B][P] (one length for all), the position at 0, every DeltaNet state zeroed."""
        import torch
        prompts = np.asarray(prompts, np.int32)
        if prompts.shape[0] != self.B or not 1 <= prompts.shape[1] <= self.max_ctx:
            raise ValueError("prompts must be [batch][1..max_ctx]")
        with torch.cuda.stream(stream):
            self.tokens.zero_()
            self.tokens[:, :prompts.shape[1]] = torch.from_numpy(prompts).to(self.tokens.device)
            self.pos.zero_()
            self.plen.fill_(prompts.shape[1])
        for g in self.gdns:
            self.fn.gdn_reset(g, stream.cuda_stream)

    def capture(self, stream):
        """Capture one step as a CUDA graph (one eager step runs first, to set the kernels' attributes)."""
        import torch
        self.start(np.zeros((self.B, 1), np.int32), stream)
        self.launch_step(stream.cuda_stream)
        self.fn.sync(stream.cuda_stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
            self.launch_step(torch.cuda.current_stream().cuda_stream)
        self.graph = g

    def generate(self, prompts, n_new, stream, marks=None):
        """Greedy decode of every sequence; returns ids [B][P + n_new]. marks: optional CUDA events recorded after the
        reset, after the last prompt-only step and after the last step."""
        import torch
        if self.graph is None:
            raise RuntimeError("capture() the step first")
        P = np.asarray(prompts).shape[1]
        if P + n_new > self.max_ctx or n_new < 1:
            raise ValueError("prompt + new tokens exceed the context")
        self.start(prompts, stream)
        with torch.cuda.stream(stream):
            if marks:
                marks[0].record(stream)
            for i in range(P + n_new - 1):
                if marks and i == P - 1:
                    marks[1].record(stream)
                self.graph.replay()
            if marks:
                marks[2].record(stream)
        self.fn.sync(stream.cuda_stream)
        return self.tokens[:, :P + n_new].cpu().numpy()

    def free(self):
        self.graph = None
        for h in self.tcs:
            self.fn.tc_free(h)
        for m in self.moes:
            self.fn.moe_free(m)
        for g in self.gdns:
            self.fn.gdn_free(g)
        self.tcs, self.moes, self.gdns = [], [], []
