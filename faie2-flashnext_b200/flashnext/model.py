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
    def __init__(self, fn, cfg: dict, W: dict, max_ctx: int = 512, logits: bool = False):
        import torch
        self.fn, self.cfg, self.max_ctx = fn, cfg, max_ctx
        dev = torch.device("cuda", torch.cuda.current_device())
        f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
        d, nkh, nvh, nh, nkv = cfg["D"], cfg["nkh"], cfg["nvh"], cfg["nh"], cfg["nkv"]
        self.convch = 2 * nkh * DS + nvh * DS
        ne, ffe, P = cfg["ne"], cfg["ffe"], cfg["proj"]
        self.handles, self.moes, self.gdns = [], [], []
        self.E = torch.from_numpy(np.ascontiguousarray(W["embed"]).reshape(-1)).to(dev)
        self.head = self._w(cfg["head"], W["head"], cfg["vocab"], d)
        self.final_norm = f32(W["final_norm"])
        self.inv_freq = f32(rope_inv_freq(cfg["rope_base"]))
        self.layers = []
        for L in W["layers"]:
            o = dict(kind=L["kind"], norm1=f32(L["norm1"]), norm2=f32(L["norm2"]),
                     router=self._w(cfg["router"], L["router"], ne + 1, d))
            if L["kind"] == "G":
                o.update(w_in=self._w(P, L["w_in"], self.convch + nvh * DS, d), w_ab=self._w(P, L["w_ab"], 2 * nvh, d),
                         w_out=self._w(P, L["w_out"], d, nvh * DS))
                g = fn.gdn_create(nkh, nvh, L["conv_w"], L["dt_bias"], L["ssm_a"], L["gnorm"],
                                  np.zeros((nvh, DS, DS), np.float32), np.zeros((3, self.convch), np.float32))
                self.gdns.append(g)
                o["gdn"] = g
            else:
                o.update(w_q=self._w(P, L["w_q"], nh * 2 * HD, d), w_k=self._w(P, L["w_k"], nkv * HD, d),
                         w_v=self._w(P, L["w_v"], nkv * HD, d), w_o=self._w(P, L["w_o"], d, nh * HD),
                         q_norm=f32(L["q_norm"]), k_norm=f32(L["k_norm"]),
                         Kc=torch.zeros(max_ctx, nkv, HD, device=dev), Vc=torch.zeros(max_ctx, nkv, HD, device=dev))
            m = fn.moe_create(cfg["gate_up"], cfg["down"], ne, cfg["k"], ffe, d, *L["moe"])
            self.moes.append(m)
            o["moe"] = m
            self.layers.append(o)
        z = lambda n: torch.zeros(n, device=dev)  # noqa: E731
        self.h, self.x, self.qkvz, self.ab = z(d), z(d), z(self.convch + nvh * DS), z(2 * nvh)
        self.core, self.qg, self.k, self.v = z(nvh * DS), z(nh * 2 * HD), z(nkv * HD), z(nkv * HD)
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

    def launch_step(self, s: int):
        """Launch one decode step on stream s (device pointers only; capturable)."""
        fn, cfg = self.fn, self.cfg
        d, nvh, nh, nkv, eps = cfg["D"], cfg["nvh"], cfg["nh"], cfg["nkv"], cfg["eps"]
        p = lambda t: t.data_ptr()  # noqa: E731
        fn.embed(cfg["embed"], p(self.E), d, p(self.tokens), p(self.pos), p(self.h), s)
        for L in self.layers:
            fn.rmsnorm(p(self.h), p(L["norm1"]), p(self.x), d, eps, s)
            if L["kind"] == "G":
                fn.w_gemv(L["w_in"], p(self.x), d, p(self.qkvz), 0, 1, 0, s)
                fn.w_gemv(L["w_ab"], p(self.x), d, p(self.ab), 0, 1, 0, s)
                # the layer's previous core launch is a whole step back: its state is read before the wait
                fn.gdn_run(L["gdn"], p(self.qkvz), self.convch, p(self.qkvz) + 4 * self.convch, nvh * DS, p(self.ab),
                           2 * nvh, p(self.core), nvh * DS, 1, 1, s)
                fn.w_gemv(L["w_out"], p(self.core), nvh * DS, p(self.h), 0, 1, 1, s)  # h += W_out core
            else:
                fn.w_gemv(L["w_q"], p(self.x), d, p(self.qg), 0, 1, 0, s)
                fn.w_gemv(L["w_k"], p(self.x), d, p(self.k), 0, 1, 0, s)
                fn.w_gemv(L["w_v"], p(self.x), d, p(self.v), 0, 1, 0, s)
                fn.attn_decode(p(self.qg), p(self.k), p(self.v), p(L["q_norm"]), p(L["k_norm"]), p(self.inv_freq),
                               p(self.Q), p(L["Kc"]), p(L["Vc"]), p(self.att), p(self.pos), nh, nkv, self.max_ctx, eps, s)
                fn.w_gemv(L["w_o"], p(self.att), nh * HD, p(self.h), 0, 1, 1, s)  # h += W_o o
            fn.rmsnorm(p(self.h), p(L["norm2"]), p(self.x), d, eps, s)
            fn.w_gemv(L["router"], p(self.x), d, p(self.lr), 0, 1, 0, s)
            fn.moe_run(L["moe"], p(self.lr), cfg["ne"] + 1, p(self.x), p(self.h), 1, 1, s)  # h += moe(x)
        fn.rmsnorm(p(self.h), p(self.final_norm), p(self.x), d, eps, s)
        fn.w_gemv_argmax(self.head, p(self.x), d, p(self.logits) if self.logits is not None else 0, 0, 1, 0, 0,
                         p(self.next), 0, s)
        fn.step_advance(p(self.pos), p(self.tokens), p(self.next), p(self.plen), self.max_ctx, s)

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

    def generate(self, prompt, n_new, stream):
        """Greedy decode: the prompt, then n_new tokens; returns the token ids of all positions (device replays only)."""
        import torch
        if len(prompt) + n_new > self.max_ctx:
            raise ValueError("prompt + new tokens exceed the context")
        self.start(prompt, stream)
        with torch.cuda.stream(stream):  # replays go to the current stream
            for _ in range(len(prompt) + n_new - 1):
                self.graph.replay()
        self.fn.sync(stream.cuda_stream)
        return self.tokens[:len(prompt) + n_new].cpu().numpy()

    def free(self):
        self.graph = None
        for h in self.handles:
            self.fn.w_free(h)
        for m in self.moes:
            self.fn.moe_free(m)
        for g in self.gdns:
            self.fn.gdn_free(g)
        self.handles, self.moes, self.gdns = [], [], []
