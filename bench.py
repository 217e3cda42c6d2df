"""Benchmark of the B200 decode hot path: dequant-fused GEMV throughput (the format sweep) with the
config-3 MoE layer, at one fixed total workload on 1..N GPUs.

A step is one batch-1 pass of: the 13 graded GGUF formats x (2048x4096, 4096x2048, 512x2048) (out x in), the
config-3 MoE layer (512 experts, top-10, width 512, IQ3_XXS gate/up, Q4_K down, shared expert) and the Q6_K lm_head
151936x2048 with its fused argmax; 400 MB of weights per step, larger than the 126 MB L2, so every step streams its
weights from HBM. Weights are seeded synthetic GGUF blocks (uniform random bytes, fp16 scales |N(0,1)|*1e-3), x is
N(0,1), router logits 2 N(0,1): the reference's real model tensors are not shipped.

  value  device-resident throughput: the step's algorithmic bytes (GGUF weight bytes + 4*cols x + 4*rows y per GEMV;
         the MoE layer: the k routed and the shared experts' rows) / the max over ranks of the CUDA-event time of K
         steps, each step one replay of the captured CUDA graphs: the 39 independent sweep GEMVs as 8 concurrent
         chains (programmatic dependent launch inside a chain), the MoE layer, the lm_head
  e2e    the same metric with host buffers: each step copies every input (the GEMVs' x, the MoE layer's x and router
         logits) in from pinned memory, runs the step's library launches and copies every output (the GEMVs' y, the
         MoE output, the token id) out, inside the timed region; two input / output buffer pairs alternate so the
         copies overlap the neighbouring steps' kernels
  roofline  the dominant kernel (the lm_head GEMV): its algorithmic bytes / its mean CUDA-event duration inside the
         timed region, against the measured HBM copy bandwidth
  cpu_baseline  the reference's CPU path (gguf-py dequant + float64 numpy GEMV) on a bounded row sample, 1 core

N > 1 (torchrun, one rank per GPU): the same total step split the north star's way (strong scaling): every GEMV and
the lm_head by rows (rank g owns rows [g R / N, (g + 1) R / N); the lm_head's argmax is combined in-kernel from the
ranks' keys over NVLink), the MoE layer by experts (the slot outputs combined in-kernel over NVLink).
`--impl reference` times the CPU path with every host core instead (rank 0 only; other ranks exit 0).
`--components` (1 GPU) prints one JSON line per component instead of the bench line: every sweep GEMV alone with cold
weights (fn_bench_gemv), the tensor-core batched GEMV at 8 and 32 tokens against the CUDA-core batched GEMV, the
config-3 MoE layer and the config-4 DeltaNet layer step, each timed with CUDA events over a CUDA graph of back-to-back
calls whose weights alternate between copies (together larger than L2).
`--workload decode` prints the config-5 decode line instead (tok/s; see run_decode). `--workload kernel` runs one
kernel family alone for an ncu capture (run_kernel). `--workload lm_head` runs the lm_head alone.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "faie2-flashnext_b200")
for _p in (ROOT, PKG, os.path.join(PKG, "flashnext")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "decode tok/s (bs=1) and quant-GEMV achieved HBM GB/s vs B200 peak"
SWEEP13 = ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ2_XXS", "IQ3_XXS", "IQ4_XS"]
SHAPES = [(2048, 4096), (4096, 2048), (512, 2048)]
LM_HEAD = ("Q6_K", 151936, 2048)
FALLBACK_HBM_GBS = 6650.0
PROFILE_TRAFFIC = os.path.join(ROOT, "profiles", "gemv_q6k_lm_head_151936x2048.txt")


def workload():
    from synth import BY_NAME
    w = [(BY_NAME[n], r, c, n) for n in SWEEP13 for (r, c) in SHAPES]
    w.append((BY_NAME[LM_HEAD[0]], LM_HEAD[1], LM_HEAD[2], LM_HEAD[0]))
    return w


def alg_bytes(qtype, rows, cols):
    from synth import row_bytes
    return rows * row_bytes(qtype, cols) + 4 * cols + 4 * rows


class ClockSampler:
    """NVML SM clock, power and throttle reasons of one GPU, sampled in a thread while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, torch_dev: int):
        self.samples, self.stop_evt, self.th, self.h, self.max_mhz = [], threading.Event(), None, None, None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(torch_dev).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid.encode() if isinstance(uuid, str) else uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # clocks are reported as unavailable, the run itself is unaffected
            self.err = f"{type(e).__name__}: {e}"

    def _loop(self):
        while not self.stop_evt.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, rs))
            except Exception:
                pass
            time.sleep(0.002)

    def start(self):
        if self.h is not None:
            self.th = threading.Thread(target=self._loop, daemon=True)
            self.th.start()

    def stop(self):
        if self.th:
            self.stop_evt.set()
            self.th.join()
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": getattr(self, "err", "no samples")}
        mhz = [s[0] for s in self.samples]
        seen = set()
        for _, rs in self.samples:
            for name, bit in self.REASONS.items():
                if rs & bit:
                    seen.add(name)
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": sorted(seen),
                "samples": len(mhz), "source": "nvml"}


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic():
    """DRAM bytes per lm_head launch from the committed ncu summary (a 'dram_bytes_per_launch: N' line), or None."""
    try:
        for line in open(PROFILE_TRAFFIC):
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


def cpu_baseline_sample(work, target_s=12.0, workers=1):
    from oracle.ref_path import CPUSweep  # the checker's CPU path: baseline only
    probe = CPUSweep([(q, r, c) for q, r, c, _ in work], 1 / 256, workers)
    t = min(probe.step() for _ in range(2))
    probe.close()
    frac = min(1.0, (1 / 256) * target_s / max(t, 1e-3))
    s = CPUSweep([(q, r, c) for q, r, c, _ in work], frac, workers)
    dt = s.step()
    s.close()
    return s.bytes / dt / 1e9, frac, dt


def run_components():
    """Per-component device times on GPU 0 (see the module docstring); one JSON line each on stdout."""
    import torch
    from fn import FN
    from synth import BY_NAME, TYPES, random_blocks

    f = FN()
    f.set_device(0)
    torch.cuda.set_device(0)

    def emit(d):
        print(json.dumps(d), flush=True)

    for name, r, c in [(n, r, c) for n in SWEEP13 for r, c in SHAPES] + [LM_HEAD]:
        q = BY_NAME[name]
        ms = f.bench_gemv(q, r, c, 1, 40 if r < 100000 else 10)
        emit({"component": "gemv", "format": name, "rows": r, "cols": c, "us": round(ms * 1e3, 2),
              "tb_per_s": round(alg_bytes(q, r, c) / (ms / 1e3) / 1e12, 3)})

    # batched decode: the tensor-core GEMV (fn_bench_tc_gemv) against the CUDA-core batched GEMV (8 tokens per call)
    for name, r, c in [("Q4_K", 4096, 2048), ("IQ3_XXS", 4096, 2048), ("Q8_0", 2048, 4096), LM_HEAD]:
        q = BY_NAME[name]
        it = 200 if r < 100000 else 20
        cc8 = f.bench_gemv(q, r, c, 8, it)
        for nt in (8, 32):
            ms = f.bench_tc_gemv(q, r, c, nt, it)
            emit({"component": "tc_gemv", "format": name, "rows": r, "cols": c, "tokens": nt, "us": round(ms * 1e3, 2),
                  "cuda_core_us": round(cc8 * 1e3 * (nt // 8), 2), "speedup": round(cc8 * (nt // 8) / ms, 2),
                  "tflop_per_s": round(2.0 * r * c * nt / (ms / 1e3) / 1e12, 2),
                  "weight_tb_per_s": round(alg_bytes(q, r, c) / (ms / 1e3) / 1e12, 3)})

    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    K = 200

    def timed(one):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for i in range(K):
                one(i, torch.cuda.current_stream().cuda_stream)
        g.replay()
        torch.cuda.synchronize()
        best = 1e30
        for _ in range(3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            g.replay()
            b.record(st)
            torch.cuda.synchronize()
            best = min(best, a.elapsed_time(b) / K * 1e3)
        del g
        return best

    # config 3: 512 experts, top-10, width 512, hidden 2048, IQ3_XXS gate/up, Q4_K down, shared expert
    gu, dn, ne, k, ffe, d = BY_NAME["IQ3_XXS"], BY_NAME["Q4_K"], 512, 10, 512, 2048
    rng = np.random.default_rng(3)
    W = [random_blocks(gu, ne * ffe, d, rng), random_blocks(gu, ne * ffe, d, rng), random_blocks(dn, ne * d, ffe, rng),
         random_blocks(gu, ffe, d, rng), random_blocks(gu, ffe, d, rng), random_blocks(dn, d, ffe, rng)]
    hs = [f.moe_create(gu, dn, ne, k, ffe, d, *W) for _ in range(2)]
    del W
    x = torch.randn(16, d, device="cuda")
    lg = torch.randn(16, ne + 1, device="cuda") * 2
    y = torch.zeros(8, d, device="cuda")
    moe_bytes = (k + 1) * (2 * ffe * row_bytes_of(gu, d) + d * row_bytes_of(dn, ffe))
    for nt in (1, 8):
        us = timed(lambda i, cs: f.moe_run(hs[i % 2], lg[i % 16].data_ptr(), ne + 1, x[i % 16].data_ptr(), y.data_ptr(),
                                           nt, 2, cs))
        emit({"component": "moe_layer_config3", "tokens": nt, "us": round(us, 2), "kernels": 3,
              "weight_bytes_per_token": moe_bytes})
    for h in hs:
        f.moe_free(h)

    # config 4: Q5_K in-projection 2048 -> 8192 + 4096, Q8_0 alpha/beta 2048 -> 64, the core, Q5_K out 4096 -> 2048
    NKH, NVH, DS = 16, 32, 128
    CONVCH = 2 * NKH * DS + NVH * DS
    q5, q8 = BY_NAME["Q5_K"], BY_NAME["Q8_0"]
    hw = []
    for _ in range(2):
        w_in = f.w_create(q5, random_blocks(q5, CONVCH + NVH * DS, d, rng), CONVCH + NVH * DS, d)
        w_ab = f.w_create(q8, random_blocks(q8, 2 * NVH, d, rng), 2 * NVH, d)
        w_out = f.w_create(q5, random_blocks(q5, d, NVH * DS, rng), d, NVH * DS)
        conv_w = (rng.standard_normal((CONVCH, 4)) * 0.5).astype(np.float32)
        hg = f.gdn_create(NKH, NVH, conv_w, (rng.standard_normal(NVH) * 0.5).astype(np.float32),
                          (-np.exp(rng.standard_normal(NVH) * 0.5)).astype(np.float32),
                          (1 + 0.1 * rng.standard_normal(DS)).astype(np.float32),
                          (rng.standard_normal((NVH, DS, DS)) * 0.02).astype(np.float32),
                          rng.standard_normal((3, CONVCH)).astype(np.float32))
        hw.append((w_in, w_ab, w_out, hg))
    qkvz = torch.empty(CONVCH + NVH * DS, device="cuda")
    ab = torch.empty(2 * NVH, device="cuda")
    core = torch.empty(NVH * DS, device="cuda")
    yo = torch.empty(d, device="cuda")

    def gdn_core(i, cs):
        f.gdn_run(hw[i % 2][3], qkvz.data_ptr(), CONVCH, qkvz.data_ptr() + 4 * CONVCH, NVH * DS, ab.data_ptr(),
                  2 * NVH, core.data_ptr(), NVH * DS, 1, 0, cs)

    def gdn_layer(i, cs):
        w_in, w_ab, w_out, hg = hw[i % 2]
        xp = x[i % 16].data_ptr()
        f.w_gemv(w_in, xp, d, qkvz.data_ptr(), CONVCH + NVH * DS, 1, 0, cs)
        f.w_gemv(w_ab, xp, d, ab.data_ptr(), 2 * NVH, 1, 2, cs)
        f.gdn_run(hg, qkvz.data_ptr(), CONVCH, qkvz.data_ptr() + 4 * CONVCH, NVH * DS, ab.data_ptr(), 2 * NVH,
                  core.data_ptr(), NVH * DS, 1, 1, cs)
        f.w_gemv(w_out, core.data_ptr(), NVH * DS, yo.data_ptr(), d, 1, 0, cs)

    emit({"component": "gdn_core_config4", "tokens": 1, "us": round(timed(gdn_core), 2),
          "state_bytes_read_and_written": 2 * NVH * DS * DS * 4})
    emit({"component": "gdn_layer_config4", "tokens": 1, "us": round(timed(gdn_layer), 2), "kernels": 4,
          "weight_bytes": row_bytes_of(q5, d) * (CONVCH + NVH * DS) + row_bytes_of(q8, d) * 2 * NVH
          + row_bytes_of(q5, NVH * DS) * d})
    for w_in, w_ab, w_out, hg in hw:
        for h in (w_in, w_ab, w_out):
            f.w_free(h)
        f.gdn_free(hg)


def decode_step_bytes(cfg, ctx_mean):
    """Algorithmic bytes of one config-5 decode step: every GGUF weight the step reads once (the embedding row, the
    projections, the routers, k routed experts and the shared expert per layer, the lm_head), each DeltaNet state
    read and written (fp32 [nvh][128][128]), and the attention caches read over ctx_mean positions on average."""
    from synth import TYPES, row_bytes
    D, ne, k, ffe = cfg["D"], cfg["ne"], cfg["k"], cfg["ffe"]
    nkh, nvh, nh, nkv, P = cfg["nkh"], cfg["nvh"], cfg["nh"], cfg["nkv"], cfg["proj"]
    convch = 2 * nkh * 128 + nvh * 128
    rg, rd = row_bytes(cfg["gate_up"], D), row_bytes(cfg["down"], ffe)
    expert = 2 * ffe * rg + D * rd
    total = row_bytes(cfg["embed"], D) + cfg["vocab"] * row_bytes(cfg["head"], D)
    for l in range(cfg["layers"]):
        kind = cfg["pattern"][l % len(cfg["pattern"])]
        if kind == "G":
            total += (convch + nvh * 128 + 2 * nvh) * row_bytes(P, D) + D * row_bytes(P, nvh * 128)
            total += 2 * nvh * 128 * 128 * 4
        else:
            total += (nh * 512 + 2 * nkv * 256) * row_bytes(P, D) + D * row_bytes(P, nh * 256)
            total += 2 * ctx_mean * nkv * 256 * 4
        total += (ne + 1) * row_bytes(cfg["router"], D) + (k + 1) * expert
    return int(total)


def cpu_decode_sample(cfg, seed=0, tokens=4):
    """The reference's CPU forward (dequantised weights, float64, ref_fn.py pattern) on one thread, on a bounded sample:
    the model's first 4 layers (3 DeltaNet + 1 attention) at full width with a vocabulary of 8192, each token run twice
    (the first pass dequantises the experts it selects, as the reference's load does; the second is timed). Per token
    of the full model: 12 x (the 4 layers) + the lm_head matvec scaled to 151936 rows. Returns (tok/s, description)."""
    from threadpoolctl import threadpool_limits
    from oracle.model import OracleModel
    from synth import model_weights, rope_inv_freq
    sub = dict(cfg, layers=4, vocab=8192)
    with threadpool_limits(1):
        W = model_weights(sub, seed)
        o = OracleModel(sub, W, rope_inv_freq(sub["rope_base"]))
        toks = np.random.default_rng(seed).integers(0, sub["vocab"], tokens)
        for t in toks:
            o.step(int(t))
        o.reset()
        t0 = time.perf_counter()
        for t in toks:
            o.step(int(t))
        t4 = (time.perf_counter() - t0) / tokens
        x = np.random.default_rng(1).standard_normal(cfg["D"])
        t0 = time.perf_counter()
        for _ in range(5):
            o.Hd @ x
        th = (time.perf_counter() - t0) / 5
    per_token = cfg["layers"] / 4 * (t4 - th) + th * cfg["vocab"] / sub["vocab"]
    return 1.0 / per_token, (f"4 layers (GGGA) at full width, vocab 8192, {tokens} tokens, float64 numpy on 1 thread: "
                             f"{t4 * 1e3:.0f} ms per token; x12 layers + lm_head matvec scaled to {cfg['vocab']} rows")


def run_decode(f, args, rank, with_cpu=True):
    """greedy decode of 256 tokens from a seeded 64-token prompt at batch 1 on the synthetic
    48-layer hybrid MoE, one decode step = one CUDA graph replay. Returns a dict of the figures."""
    import torch
    from model import DecodeModel
    from synth import model_config, model_weights
    cfg = model_config()
    n_prompt, n_new = 64, 256
    t0 = time.perf_counter()
    W = model_weights(cfg, seed=0, pooled=True)
    m = DecodeModel(f, cfg, W, max_ctx=n_prompt + n_new)
    del W
    build_s = time.perf_counter() - t0
    s = torch.cuda.Stream()
    m.capture(s)
    prompt = torch.from_numpy(np.random.default_rng(0).integers(0, cfg["vocab"], n_prompt).astype(np.int32)).pin_memory()
    out = torch.zeros(n_new, dtype=torch.int32).pin_memory()
    if args.profile_steps:  # the launch list of a few eager steps (an NVTX range "decode_steps" for ncu)
        m.generate_host(prompt, 1, out, s)
        f.sync(s.cuda_stream)
        torch.cuda.nvtx.range_push("decode_steps")
        for _ in range(args.profile_steps):
            m.launch_step(s.cuda_stream)
        f.sync(s.cuda_stream)
        torch.cuda.nvtx.range_pop()
        n = m.launches_per_step()
        m.free()
        return {"profile_steps": args.profile_steps, "gpu_launches_per_step": n, "build_s": round(build_s, 1)}
    for _ in range(max(1, args.warmup // 20)):  # each warm-up generation is 319 decode steps
        m.generate_host(prompt, n_new, out, s)
    f.sync(s.cuda_stream)
    reps = max(1, min(4, args.steps // n_new))
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(reps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ids = []
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    clocks.start()
    for r in range(reps):
        if r == 0:
            e0.record(s)
        m.generate_host(prompt, n_new, out, s, marks=ev[r])
        if r == reps - 1:
            e1.record(s)
        f.sync(s.cuda_stream)
        ids.append(out.numpy().copy())
    clk = clocks.stop()
    gen_ms = [ev[r][1].elapsed_time(ev[r][2]) for r in range(reps)]
    all_ms = [ev[r][0].elapsed_time(ev[r][2]) for r in range(reps)]
    e2e_ms = e0.elapsed_time(e1) / reps  # prompt copy in, resets, 319 steps, ids copied out
    steps_all = n_prompt + n_new - 1
    ms_tok = statistics.median(gen_ms) / n_new
    ctx_mean = (n_prompt + n_new) / 2
    nbytes = decode_step_bytes(cfg, ctx_mean)
    peak, peak_kind = measured_peak()
    d = {
        "tok_s": round(1e3 / ms_tok, 2), "ms_per_token": round(ms_tok, 4),
        "tok_s_all_steps": round(steps_all * 1e3 / statistics.median(all_ms), 2),
        "e2e_tok_s": round(n_new * 1e3 / e2e_ms, 2), "e2e_ms_per_generation": round(e2e_ms, 3),
        "generations": reps, "bytes_per_step": nbytes,
        "roofline": {"bound": "hbm", "achieved": round(nbytes / (ms_tok / 1e3) / 1e9, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(nbytes / (ms_tok / 1e3) / 1e9 / peak, 4), "peak_kind": peak_kind,
                     "scope": "whole decode step (algorithmic bytes / step time)"},
        "ids_repeatable": bool(all(np.array_equal(ids[0], i) for i in ids)),
        "distinct_ids": int(len(np.unique(ids[0]))),
        "gpu_launches_per_step": m.launches_per_step(),
        "build_s": round(build_s, 1), "clocks": clk,
        "config": "config5: 48 layers GGGA (gated DeltaNet 16/32 heads x 128, gated attention 16/2 heads x 256, "
                  "RoPE 1e7), MoE 512 experts top-10 + shared on every layer (IQ3_XXS gate/up, Q4_K down), Q4_K "
                  "projections, BF16 router, Q6_K lm_head 151936 with fused argmax; 64-token prompt, 256 greedy tokens",
    }
    if with_cpu and rank == 0:
        tps, desc = cpu_decode_sample(cfg)
        d["cpu_baseline"] = {"value": round(tps, 5), "unit": "tok/s", "cores": 1, "kind": "port", "sample": desc}
    m.free()
    return d


def run_decode_batch(f, args, batch):
    """Config 5 at batch `batch` on the tensor-core path: `batch` seeded 64-token prompts, 256 greedy tokens each, one
    step = one CUDA graph replay for all sequences. tok/s = batch x 256 / the CUDA-event time of the 256 steps."""
    import torch
    from model import BatchDecodeModel
    from synth import model_config, model_weights
    cfg = model_config()
    n_prompt, n_new = 64, 256
    t0 = time.perf_counter()
    m = BatchDecodeModel(f, cfg, model_weights(cfg, seed=0, pooled=True), batch, max_ctx=n_prompt + n_new)
    build_s = time.perf_counter() - t0
    s = torch.cuda.Stream()
    m.capture(s)
    prompts = np.random.default_rng(0).integers(0, cfg["vocab"], (batch, n_prompt))
    m.generate(prompts, 16, s)  # warm-up
    if args.profile_steps:  # the launch list of a few eager steps (an NVTX range "decode_steps" for ncu)
        torch.cuda.nvtx.range_push("decode_steps")
        for _ in range(args.profile_steps):
            m.launch_step(s.cuda_stream)
        f.sync(s.cuda_stream)
        torch.cuda.nvtx.range_pop()
        n = m.launches_per_step()
        m.free()
        return {"batch": batch, "profile_steps": args.profile_steps, "gpu_launches_per_step": n,
                "build_s": round(time.perf_counter() - t0, 1)}
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    clocks.start()
    ids = m.generate(prompts, n_new, s, marks=ev)
    clk = clocks.stop()
    gen_ms = ev[1].elapsed_time(ev[2])
    ms_step = gen_ms / n_new
    d = {"batch": batch, "tok_s": round(batch * n_new * 1e3 / gen_ms, 2), "ms_per_step": round(ms_step, 4),
         "tok_s_per_sequence": round(1e3 / ms_step, 2), "gpu_launches_per_step": m.launches_per_step(),
         "distinct_ids": int(len(np.unique(ids[:, n_prompt:]))), "build_s": round(build_s, 1), "clocks": clk,
         "path": "projections, routers and lm_head on fn_tc_gemv (tcgen05.mma, bf16 hi/lo), the MoE layer for the whole batch in one call"}
    m.free()
    return d


def decode_line(f, args):
    """`--workload decode`: the config-5 decode as its own bench line (tok/s)."""
    if args.batch > 1:
        d = run_decode_batch(f, args, args.batch)
        if args.profile_steps:
            return d
        return {"metric": METRIC, "value": d["tok_s"], "unit": "tok/s", "n_gpus": 1, "steps": 256, "warmup": 16,
                "ms_per_step": d["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32 (bf16 hi/lo tensor-core products)", "data": "synthetic",
                "config": {"workload": f"config5 batched decode, batch {args.batch}: 64-token prompts, 256 greedy tokens "
                                       "each", "parallelism": "1 GPU"},
                "gpu_launches": d["gpu_launches_per_step"] * 256, "clocks": d["clocks"], "decode_batch": d}
    d = run_decode(f, args, 0, with_cpu=not args.no_cpu_baseline)
    if args.profile_steps:
        return d
    gen = d["generations"]
    line = {
        "metric": METRIC, "value": d["tok_s"], "unit": "tok/s", "n_gpus": 1, "steps": 256 * gen,
        "warmup": args.warmup, "ms_per_step": d["ms_per_token"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": d["config"], "bytes_per_step": d["bytes_per_step"], "parallelism": "1 GPU",
                   "l2": "inputs larger than L2 (about 2 GB of weights and states per step)"},
        "e2e": {"value": d["e2e_tok_s"], "unit": "tok/s", "h2d_bytes_per_step": round(64 * 4 / 256, 3),
                "d2h_bytes_per_step": 4, "note": "per generation: the 64-token prompt copied in (256 B), 256 ids "
                "copied out (1 KiB), the resets and all 319 steps inside the timed region"},
        "roofline": d["roofline"], "gpu_launches": d["gpu_launches_per_step"] * (64 + 256 - 1) * gen,
        "clocks": d["clocks"], "decode": d,
    }
    if "cpu_baseline" in d:
        line["cpu_baseline"] = d["cpu_baseline"]
    return line


def row_bytes_of(qtype, cols):
    from synth import TYPES
    _, qk, tb = TYPES[qtype]
    return cols // qk * tb


def run_reference(args, rank):
    """`--impl reference`: the reference's CPU path (gguf-py dequant + float64 GEMV) on every host core."""
    if rank != 0:
        return
    from oracle.ref_path import CPUSweep
    work = workload() + moe3_gemvs()
    cores = os.cpu_count() or 1
    steps, warm = args.steps, args.warmup
    budget = 150.0  # seconds for the whole run
    probe = CPUSweep([(q, r, c) for q, r, c, _ in work], 1 / 512, cores)
    t = min(probe.step() for _ in range(2))
    probe.close()
    per_step = max(0.02, min(3.0, budget / max(1, steps + warm)))
    frac = min(1.0, (1 / 512) * per_step / max(t, 1e-4))
    s = CPUSweep([(q, r, c) for q, r, c, _ in work], frac, cores)
    for _ in range(warm):
        s.step()
    times = [s.step() for _ in range(steps)]
    s.close()
    total = sum(times)
    gbs = s.bytes * steps / total / 1e9
    sample = (f"every GEMV of the step (the MoE layer as its 33 expert GEMVs) cut to {frac:.4g} of its rows "
              f"({s.bytes / 1e6:.1f} MB of GGUF weights per step)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": warm, "ms_per_step": round(1e3 * total / steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "config2 format sweep (13 formats x 3 shapes + Q6_K lm_head 151936x2048) + config-3 "
                               "MoE layer, bs=1",
                   "path": "gguf-py 0.19.0 quants.dequantize -> float64 numpy x . W^T (flashnext/ref_fn.py:44-53, "
                           "flashnext/test_fn_quants.py:34)"},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_kernel(args):
    """`--workload kernel`: one kernel family alone, `steps` eager launches on one stream (PDL as set by FN_PDL) with
    two weight copies alternating, for ncu captures of a single kernel (-k / -c) from a committed command; prints one
    JSON line with the mean time per call. --kernel gemv / tc_gemv: --format, --rows, --cols, --tokens; moe: BASELINE
    config 3 (IQ3_XXS gate/up, Q4_K down, 512 experts, top-10, --tokens tokens; --moe-var selects the MoE variant); gdn: the
    config-4 DeltaNet core step (--tokens B > 1: a batch of B sequences, one token each)."""
    import torch
    from fn import FN
    from synth import BY_NAME, random_blocks
    f = FN()
    f.set_device(0)
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(3)
    s = torch.cuda.Stream()
    cs = s.cuda_stream
    frees = []
    if args.kernel in ("gemv", "tc_gemv"):
        q, r, c, nt = BY_NAME[args.format], args.rows, args.cols, args.tokens
        if args.warps >= 0:  # the decode step plans its GEMVs with 16 warps per CTA (DecodeModel)
            f.gemv_tune(args.warps)
        f.qmma(1 if args.qmma is None else args.qmma)
        mk = f.w_create if args.kernel == "gemv" else f.tc_create
        hs = [mk(q, random_blocks(q, r, c, rng), r, c) for _ in range(2)]
        frees = [(f.w_free if args.kernel == "gemv" else f.tc_free, h) for h in hs]
        x = torch.randn(nt, c, device=dev)
        y = torch.zeros(nt, r, device=dev)
        call = (lambda i: f.w_gemv(hs[i % 2], x.data_ptr(), c, y.data_ptr(), r, nt, 0, cs)) if args.kernel == "gemv" \
            else (lambda i: f.tc_gemv(hs[i % 2], x.data_ptr(), c, y.data_ptr(), r, nt, 0, cs))
        what = {"kernel": args.kernel, "format": args.format, "rows": r, "cols": c, "tokens": nt, "warps": args.warps,
                "qmma": 1 if args.qmma is None else args.qmma}
    elif args.kernel == "moe":
        gu, dn, ne, k, ffe, d = BY_NAME["IQ3_XXS"], BY_NAME["Q4_K"], 512, 10, 512, 2048
        f.moe_var(args.moe_var or 0)
        hs = [f.moe_create(gu, dn, ne, k, ffe, d, random_blocks(gu, ne * ffe, d, rng), random_blocks(gu, ne * ffe, d, rng),
                           random_blocks(dn, ne * d, ffe, rng), random_blocks(gu, ffe, d, rng),
                           random_blocks(gu, ffe, d, rng), random_blocks(dn, d, ffe, rng)) for _ in range(2)]
        frees = [(f.moe_free, h) for h in hs]
        nt = args.tokens
        lg = torch.randn(nt, ne + 1, device=dev) * 2
        x = torch.randn(nt, d, device=dev)
        y = torch.zeros(nt, d, device=dev)
        call = lambda i: f.moe_run(hs[i % 2], lg.data_ptr(), ne + 1, x.data_ptr(), y.data_ptr(), nt, 2, cs)  # noqa: E731
        what = {"kernel": "moe", "config": "config3", "moe_var": args.moe_var or 0, "tokens": nt}
    elif args.tokens > 1:  # gdn, a batch of --tokens sequences at one token each (the batched decode's core)
        NKH, NVH, DS, B = 16, 32, 128, args.tokens
        CONVCH = 2 * NKH * DS + NVH * DS
        hs = [f.gdn_create_batch(NKH, NVH, (rng.standard_normal((CONVCH, 4)) * 0.5).astype(np.float32),
                                 (rng.standard_normal(NVH) * 0.5).astype(np.float32),
                                 (-np.exp(rng.standard_normal(NVH) * 0.5)).astype(np.float32),
                                 (1 + 0.1 * rng.standard_normal(DS)).astype(np.float32), B) for _ in range(2)]
        frees = [(f.gdn_free, h) for h in hs]
        qkvz = torch.randn(B, CONVCH + NVH * DS, device=dev)
        ab = torch.randn(B, 2 * NVH, device=dev)
        out = torch.zeros(B, NVH * DS, device=dev)
        rs = CONVCH + NVH * DS
        call = lambda i: f.gdn_run_batch(hs[i % 2], qkvz.data_ptr(), rs, qkvz.data_ptr() + 4 * CONVCH, rs,  # noqa: E731
                                         ab.data_ptr(), 2 * NVH, out.data_ptr(), NVH * DS, 1, cs)
        what = {"kernel": "gdn", "config": f"config4 core, a batch of {B} sequences", "tokens": B}
    else:  # gdn
        NKH, NVH, DS = 16, 32, 128
        CONVCH = 2 * NKH * DS + NVH * DS
        hs = []
        for _ in range(2):
            hs.append(f.gdn_create(NKH, NVH, (rng.standard_normal((CONVCH, 4)) * 0.5).astype(np.float32),
                                   (rng.standard_normal(NVH) * 0.5).astype(np.float32),
                                   (-np.exp(rng.standard_normal(NVH) * 0.5)).astype(np.float32),
                                   (1 + 0.1 * rng.standard_normal(DS)).astype(np.float32),
                                   (rng.standard_normal((NVH, DS, DS)) * 0.02).astype(np.float32),
                                   rng.standard_normal((3, CONVCH)).astype(np.float32)))
        frees = [(f.gdn_free, h) for h in hs]
        qkvz = torch.randn(CONVCH + NVH * DS, device=dev)
        ab = torch.randn(2 * NVH, device=dev)
        out = torch.zeros(NVH * DS, device=dev)
        call = lambda i: f.gdn_run(hs[i % 2], qkvz.data_ptr(), CONVCH, qkvz.data_ptr() + 4 * CONVCH, NVH * DS,  # noqa: E731
                                   ab.data_ptr(), 2 * NVH, out.data_ptr(), NVH * DS, 1, 1, cs)
        what = {"kernel": "gdn", "config": "config4 core"}
    for i in range(max(3, args.warmup)):
        call(i)
    f.sync(cs)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for i in range(args.steps):
        call(i)
    b.record(s)
    f.sync(cs)
    print(json.dumps(dict(what, steps=args.steps, us_per_call=round(a.elapsed_time(b) * 1e3 / args.steps, 3))), flush=True)
    f.moe_var(0)
    for fr, h in frees:
        fr(h)


MOE3 = ("IQ3_XXS", "Q4_K", 512, 10, 512, 2048)  # gate/up, down, experts, top-k, width, hidden


def moe3_gemvs():
    """The config-3 MoE layer of one token as the GEMVs it reads (the k routed experts and the shared expert: gate and
    up over the hidden size, down over the width): the CPU arms' restatement of its weight traffic."""
    from synth import BY_NAME
    gu, dn, ne, k, ffe, d = MOE3
    return [(BY_NAME[gu], ffe, d, gu)] * (2 * (k + 1)) + [(BY_NAME[dn], d, ffe, dn)] * (k + 1)


def moe3_bytes():
    """Algorithmic bytes of one config-3 MoE layer for one token: the k routed experts' and the shared expert's
    gate, up and down rows, each read once."""
    from synth import BY_NAME
    gu, dn, ne, k, ffe, d = MOE3
    return (k + 1) * (2 * ffe * row_bytes_of(BY_NAME[gu], d) + d * row_bytes_of(BY_NAME[dn], ffe))


class SweepStep:
    """The bench step on this rank: the 39 sweep GEMVs, the config-3 MoE layer (one token) and the lm_head with its
    fused argmax. One GPU: everything here. N ranks (one per GPU): the north star's partitions at a fixed total
    workload (strong scaling): every GEMV split by rows (rank g owns rows [g R / N, (g + 1) R / N): each row's sum is
    the one-GPU sum), the lm_head split by vocabulary rows with its argmax combined in-kernel over NVLink
    (parallel.LmHeadSplit), the MoE layer split by experts with the slot outputs exchanged in-kernel
    (fn_moe_ep_create / fn_moe_ep_run). Every input (the GEMVs' x, the MoE layer's x and router logits) is a view of
    one device buffer X and every output (the GEMVs' y slices, the MoE output, the argmax) of one buffer Y, so a
    step's host round trip is one copy each way."""

    def __init__(self, f, work, rank, world, group, with_moe=True):
        import torch
        from parallel import LmHeadSplit, expert_range, row_range
        from synth import BY_NAME, random_blocks
        self.f, self.work, self.world, self.group, self.with_moe = f, work, world, group, with_moe
        dev = torch.device("cuda", torch.cuda.current_device())
        gu, dn, ne, k, ffe, d = MOE3
        self.gu, self.dn = BY_NAME[gu], BY_NAME[dn]
        # inputs: every GEMV's x, then the MoE layer's x and its router logits (the same values on every rank)
        xlen = [c for _, _, c, _ in work] + [d, ne + 1]
        self.xoff = np.concatenate([[0], np.cumsum(xlen)]).astype(int)
        X = torch.empty(int(self.xoff[-1]), device=dev)
        for i, n in enumerate(xlen):
            g = torch.Generator("cuda").manual_seed(i)
            X[self.xoff[i]:self.xoff[i + 1]] = torch.randn(n, device=dev, generator=g) * (2.0 if i == len(xlen) - 1 else 1.0)
        self.X = X
        self.buf = 0  # which input / output buffer pair the launches use (the e2e pipeline alternates two)
        self.rows = [row_range(r, world, rank) for _, r, _, _ in work]
        ylen = [r1 - r0 for r0, r1 in self.rows] + [d, 4]  # y slices, the MoE output, the argmax (one int32 slot)
        self.yoff = np.concatenate([[0], np.cumsum(ylen)]).astype(int)
        self.Y = torch.zeros(int(self.yoff[-1]), device=dev)
        self.X2, self.Y2 = self.X.clone(), torch.zeros_like(self.Y)  # the second pair
        self.hs, self.head = [], None
        self.step_bytes = sum(alg_bytes(q, r, c) for q, r, c, _ in work) + (moe3_bytes() if with_moe else 0)
        self.head_rows = self.rows[-1][1] - self.rows[-1][0]
        self.head_bytes = alg_bytes(work[-1][0], self.head_rows, work[-1][2])
        for i, (q, r, c, name) in enumerate(work):
            raw = random_blocks(q, r, c, np.random.default_rng(i))  # the same matrix on every rank
            r0, r1 = self.rows[i]
            if i == len(work) - 1 and world > 1:
                self.head = LmHeadSplit(f, group, q, raw, r, c)
            else:
                self.hs.append(f.w_create(q, np.ascontiguousarray(raw[r0:r1]), r1 - r0, c))
            del raw
        self.moe = 0
        self.launches_per_step = len(work) + (1 if world > 1 else 0)  # the split lm_head adds its key combine
        if not with_moe:
            return
        rng = np.random.default_rng(77)  # config-3 weights, the same on every rank
        Wg, Wu = random_blocks(self.gu, ne * ffe, d, rng), random_blocks(self.gu, ne * ffe, d, rng)
        Wd = random_blocks(self.dn, ne * d, ffe, rng)
        sh = [random_blocks(self.gu, ffe, d, rng), random_blocks(self.gu, ffe, d, rng), random_blocks(self.dn, d, ffe, rng)]
        if world > 1:
            e0, e1 = expert_range(ne, world, rank)
            self.moe = f.moe_ep_create(self.gu, self.dn, ne, k, ffe, d, group.id, np.ascontiguousarray(Wg[e0 * ffe:e1 * ffe]),
                                       np.ascontiguousarray(Wu[e0 * ffe:e1 * ffe]), np.ascontiguousarray(Wd[e0 * d:e1 * d]),
                                       *sh)
        else:
            self.moe = f.moe_create(self.gu, self.dn, ne, k, ffe, d, Wg, Wu, Wd, *sh)
        del Wg, Wu, Wd
        self.launches_per_step += 3 if world == 1 else 4  # routing, gate/up, down (+ the combine across ranks)

    def bufs(self, b):
        """Input and output buffers of pair b (0: the device-timed step's; 1: the e2e pipeline's second pair)."""
        return (self.X, self.Y) if b == 0 else (self.X2, self.Y2)

    def x(self, i):
        return self.bufs(self.buf)[0].data_ptr() + 4 * int(self.xoff[i])

    def y(self, i):
        return self.bufs(self.buf)[1].data_ptr() + 4 * int(self.yoff[i])

    def launch_gemv(self, i, s, early=True):
        q, r, c, _ = self.work[i]
        r0, r1 = self.rows[i]
        if i == len(self.work) - 1:  # the lm_head: logits slice and the vocabulary-wide argmax
            amax = self.y(len(self.work) + 1)
            if self.head is not None:
                self.head.run(self.x(i), c, amax, 1, self.y(i), 2 if early else 0, s)
            else:
                self.f.w_gemv_argmax(self.hs[i], self.x(i), c, self.y(i), r, 1, 2 if early else 0, 0, amax, 0, s)
        else:
            self.f.w_gemv(self.hs[i], self.x(i), c, self.y(i), r1 - r0, 1, 2 if early else 0, s)

    def launch_moe(self, s):
        ne, n = MOE3[2], len(self.work)
        run = self.f.moe_ep_run if self.world > 1 else self.f.moe_run
        run(self.moe, self.x(n + 1), ne + 1, self.x(n), self.y(n), 1, 0, s)

    def host_buffers(self):
        """Pinned host copies of X and Y (the e2e path's inputs and outputs)."""
        import torch
        return self.X.cpu().pin_memory(), torch.empty(self.Y.numel(), dtype=torch.float32).pin_memory()

    def free(self):
        for h in self.hs:
            self.f.w_free(h)
        if self.head is not None:
            self.head.close()
        if self.moe:
            self.f.moe_free(self.moe)


def run_sweep(f, args, rank, world, local, dist):
    """The default step (SweepStep) on this rank: device-timed value with the inputs resident, then the e2e value with
    the inputs copied in from pinned host memory and the outputs copied out every step. Returns the JSON line."""
    import torch
    from parallel import PeerGroup

    work = workload() if args.workload == "sweep" else workload()[-1:]
    group = None
    if world > 1:
        def gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out
        group = PeerGroup(f, rank, world, gather, dist.barrier)
    st = SweepStep(f, work, rank, world, group, with_moe=args.workload == "sweep")
    n = len(work)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    s0 = stream.cuda_stream
    # first launches outside capture (kernel attributes, error-word address); every rank makes the same group calls
    for i in range(n):
        st.launch_gemv(i, s0, early=False)
    if st.with_moe:
        st.launch_moe(s0)
    f.sync(s0)

    # the sweep's GEMVs are independent (own weights, inputs and outputs): each is launched early (it reads its x
    # without waiting for the kernel before it, the reference's early-GEMV protocol) and they run as BRANCHES
    # concurrent chains of one graph (a fork and a join on the capture stream), so several are resident on an SM
    # at once; the MoE layer and the lm_head with its argmax are graphs of their own on the main stream
    side = [torch.cuda.Stream() for _ in range(args.branches)]

    def capture(b):
        """The step's graphs (sweep, MoE layer, lm_head) over input / output buffer pair b."""
        st.buf = b
        g_small = torch.cuda.CUDAGraph() if n > 1 else None
        g_moe = torch.cuda.CUDAGraph() if st.with_moe else None
        g_head = torch.cuda.CUDAGraph()
        if g_small is not None:
            with torch.cuda.graph(g_small, stream=stream, capture_error_mode="thread_local"):
                main_s = torch.cuda.current_stream()
                for sd in side:
                    sd.wait_stream(main_s)
                for i in range(n - 1):
                    st.launch_gemv(i, side[i % len(side)].cuda_stream)
                for sd in side:
                    main_s.wait_stream(sd)
        if g_moe is not None:
            with torch.cuda.graph(g_moe, stream=stream, capture_error_mode="thread_local"):
                st.launch_moe(torch.cuda.current_stream().cuda_stream)
        with torch.cuda.graph(g_head, stream=stream, capture_error_mode="thread_local"):
            st.launch_gemv(n - 1, torch.cuda.current_stream().cuda_stream, early=False)
        st.buf = 0
        return [g for g in (g_small, g_moe, g_head) if g is not None]

    graphs = capture(0)
    sets = [graphs, capture(1)]  # the second over buffer pair 1, which holds the same inputs
    g_small = graphs[0] if n > 1 else None
    g_moe = graphs[1 if n > 1 else 0] if st.with_moe else None

    def step():
        for g in graphs:
            g.replay()

    def max_over_ranks(v):
        if dist:
            t = torch.tensor([v], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
        return v

    for w in range(args.warmup):
        for g in sets[w & 1]:
            g.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    K = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(graphs) + 1)] for _ in range(K)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    # `value`: K steps timed by events at the ends only, the two graph sets alternating and each step ordered after the
    # previous one through an event, as in the e2e pipeline below (measured on 2 GPUs: 2160 -> 2256 GB/s; no change on
    # one); then the same K steps again with an event between the graphs, for the per-component split and the
    # lm_head's launch time (the events between graphs add small gaps)
    evs = [torch.cuda.Event(), torch.cuda.Event()]
    e0.record(stream)
    for k in range(K):
        if k >= 1:
            stream.wait_event(evs[(k - 1) & 1])
        for g in sets[k & 1]:
            g.replay()
        evs[k & 1].record(stream)
    e1.record(stream)
    for k in range(K):
        ev[k][0].record(stream)
        for j, g in enumerate(graphs):
            g.replay()
            ev[k][j + 1].record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    seg = [sum(ev[k][j].elapsed_time(ev[k][j + 1]) for k in range(K)) / K for j in range(len(graphs))]
    head_ms = seg[-1]
    value = st.step_bytes * K / (ms / 1e3) / 1e9

    # e2e: every step copies all inputs in from pinned host memory, runs the step's library launches (the captured
    # graphs of the same calls) and copies every output out (the GEMVs' y slices, the MoE output, the token id). Two
    # input / output buffer pairs alternate, with a copy stream each way, so a step's copies overlap the kernels of the
    # steps beside it: step k's input copy waits for step k - 2's kernels (the same input buffer), its kernels for that
    # copy and for step k - 2's output copy (the same output buffer), its output copy for its kernels.
    xh, yh = st.host_buffers()
    h2d, d2h = xh.numel() * 4, yh.numel() * 4
    Ke = max(3, min(K, 200))
    pairs = [st.bufs(0), st.bufs(1)]
    yhs = [yh, torch.empty_like(yh).pin_memory()]
    cs_in, cs_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in, ev_done, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

    def e2e_run(nsteps, start, end):
        start.record(stream)
        cs_in.wait_event(start)
        cs_out.wait_event(start)
        for k in range(nsteps):
            bb = k & 1
            X, Y = pairs[bb]
            if k >= 2:
                cs_in.wait_event(ev_done[bb])
            with torch.cuda.stream(cs_in):
                X.copy_(xh, non_blocking=True)
            ev_in[bb].record(cs_in)
            stream.wait_event(ev_in[bb])
            if k >= 2:
                stream.wait_event(ev_out[bb])
            for g in sets[bb]:
                g.replay()
            ev_done[bb].record(stream)
            cs_out.wait_event(ev_done[bb])
            with torch.cuda.stream(cs_out):
                yhs[bb].copy_(Y, non_blocking=True)
            ev_out[bb].record(cs_out)
        stream.wait_stream(cs_out)
        end.record(stream)
        torch.cuda.synchronize()

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_run(4, a, b)  # warm-up
    if dist:
        dist.barrier()
    e2e_run(Ke, a, b)
    e2e_ms = max_over_ranks(a.elapsed_time(b))
    e2e = st.step_bytes * Ke / (e2e_ms / 1e3) / 1e9
    yh = yhs[(Ke - 1) & 1]
    yv = yh.numpy()
    tok = int(yv[-4:].view(np.int32)[0])
    ok = bool(np.isfinite(yv[:-4]).all()) and 0 <= tok < work[-1][1]

    peak, peak_kind = measured_peak()
    achieved = st.head_bytes / (head_ms / 1e3) / 1e9
    traffic = profile_traffic()
    if traffic is not None:  # the capture is of the whole 151936-row head; a rank's slice reads its share
        traffic = round(traffic * st.head_rows / work[-1][1])
    names = (["39 sweep GEMVs"] if g_small is not None else []) + (["config-3 MoE layer"] if g_moe is not None else [])
    names.append("lm_head" + (" slice + argmax combine" if world > 1 else " + argmax"))
    part = ("1 GPU" if world == 1 else f"{world} GPUs: every GEMV and the lm_head split by rows (argmax combined "
            f"in-kernel over NVLink), the MoE layer split by experts (outputs combined in-kernel over NVLink)")
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(ms / K, 5), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2 format sweep: 13 formats x (2048x4096, 4096x2048, 512x2048) + Q6_K lm_head "
                               "151936x2048 with fused argmax" + (" + config-3 MoE layer (512 experts, top-10, width "
                               "512, IQ3_XXS/Q4_K, shared expert)" if st.with_moe else "") + ", bs=1, one fixed "
                               "total workload split over the GPUs",
                   "bytes_per_step": st.step_bytes, "l2": "inputs larger than L2 (400 MB of weights per step over "
                   "all GPUs, each read once per step)", "parallelism": part,
                   "frac_of_measured_peak": round(value / world / peak, 4)},
        "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": Ke, "outputs_finite": bool(ok), "path": "pinned host -> device copy of every input, the "
                "step's library launches (as captured graphs), device -> pinned host copy of every output, per step; "
                "two input / output buffer pairs alternate with a copy stream each way, so the copies overlap the "
                "neighbouring steps' kernels"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                     "kernel": f"k_gemv<Q6_K> lm_head {st.head_rows}x2048 + fused argmax",
                     "mean_launch_us": round(head_ms * 1e3, 2), "alg_bytes_per_launch": st.head_bytes},
        "split_ms_per_step": {k: round(v, 5) for k, v in zip(names, seg)},
        "gpu_launches": 2 * K * st.launches_per_step,  # the value pass and the split pass
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, frac, dt = cpu_baseline_sample(work + (moe3_gemvs() if st.with_moe else []))
        line["cpu_baseline"] = {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                                "sample": f"every GEMV of the step (the MoE layer as its 33 expert GEMVs) cut to "
                                          f"{frac:.3g} of its rows, one pass ({dt:.1f} s), gguf-py dequant + float64 "
                                          f"numpy GEMV, 1 thread"}
    del graphs, sets, g_small, g_moe
    torch.cuda.synchronize()
    st.free()
    if group is not None:
        group.close()
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--components", action="store_true",
                    help="per-component device times (sweep GEMVs alone, config-3 MoE layer, config-4 DeltaNet layer)")
    ap.add_argument("--workload", default="sweep", choices=["sweep", "lm_head", "decode", "kernel"],
                    help="lm_head: only the dominant kernel (the small case the ncu capture profiles); decode: only "
                         "the config-5 greedy decode (its own line, tok/s); kernel: one kernel family alone (--kernel)")
    ap.add_argument("--kernel", default="gemv", choices=["gemv", "tc_gemv", "moe", "gdn"])
    ap.add_argument("--format", default="Q4_K")
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--cols", type=int, default=2048)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--moe-var", type=int, default=None,
                    help="the MoE variant (fn_moe_var; default: 0 with --kernel moe, the library's default elsewhere)")
    ap.add_argument("--qmma", type=int, default=None,
                    help="Q4_K / Q6_K GEMVs of up to 2048 columns on the tensor cores as integer products (fn_qmma); "
                         "default: on for --workload kernel, the library's default elsewhere")
    ap.add_argument("--warps", type=int, default=-1,
                    help="with --kernel gemv: warps per CTA of the plan (fn_gemv_tune; 0 = by weight size)")
    ap.add_argument("--no-decode", action="store_true", help="leave the config-5 decode out of the sweep line")
    ap.add_argument("--branches", type=int, default=8, help="concurrent graph chains of the sweep's independent GEMVs")
    ap.add_argument("--batch", type=int, default=1,
                    help="with --workload decode: that many sequences at once on the tensor-core path (2..32)")
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="with --workload decode (any --batch): run this many eager decode steps in an NVTX range and exit")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.components:
        if rank == 0:
            run_components()
        return
    if args.workload == "kernel":
        run_kernel(args)
        return
    if args.warmup < 3:
        args.warmup = 3

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        # NCCL carries only host plumbing here (handle exchange, barriers, the max over ranks): no NVLink multicast
        # objects are needed, and none are bound to the ranks' memory
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))

    from fn import FN
    from synth import random_blocks

    f = FN()
    f.set_device(local)
    if args.qmma is not None:
        f.qmma(args.qmma)
    if args.moe_var is not None:
        f.moe_var(args.moe_var)
    if args.workload == "decode":
        if world > 1:
            raise SystemExit("--workload decode runs on one GPU")
        print(json.dumps(decode_line(f, args)), flush=True)
        return
    line = run_sweep(f, args, rank, world, local, dist)
    if world == 1 and args.workload == "sweep" and not args.no_decode:
        line["decode"] = run_decode(f, args, rank, with_cpu=not args.no_cpu_baseline)
        line["gpu_launches"] += line["decode"]["gpu_launches_per_step"] * (64 + 256 - 1) * line["decode"]["generations"]
        # batched decode on the tensor-core path (BASELINE config 5's batch 8 and 32)
        line["decode"]["batched"] = []
        for b in (8, 32):
            db = run_decode_batch(f, args, b)
            line["decode"]["batched"].append(db)
            line["gpu_launches"] += db["gpu_launches_per_step"] * (64 + 16 - 1 + 64 + 256 - 1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
