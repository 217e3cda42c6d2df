/* C ABI of libfaie2fn.so, the B200 (sm_100a) decode hot path of FAIE2-FlashNext.
 *
 * Every entry point mirrors one the reference exports from engine/faie2fn.cu (built there as faie2fn.dll with
 * __declspec(dllexport), :34) and binds through the same ctypes layer (flashnext/fn.py). Conventions, as in the
 * reference: int results are 0 on success and -1 on error, with the message in fn_error() (:114-118, :2495); the
 * caller owns every host buffer (C-contiguous); the fn_test_* and fn_bench_* hooks are synchronous and use the device
 * named by fn_set_device (default: env FN_DEVICE, else 0). Not thread-safe: one caller thread.
 *
 * Type ids are ggml's: Q4_0=2 Q4_1=3 Q5_0=6 Q5_1=7 Q8_0=8 Q2_K=10 Q3_K=11 Q4_K=12 Q5_K=13 Q6_K=14 IQ2_XXS=16
 * IQ2_XS=17 IQ3_XXS=18 IQ4_NL=20 IQ3_S=21 IQ2_S=22 IQ4_XS=23 BF16=30 Q2_0=42.
 *
 * The reference's model hooks (fn_load, fn_reset, fn_forward, fn_debug_layers, fn_use_graphs, fn_n_past,
 * fn_last_ms, fn_dev_gb, fn_split, fn_free; engine/faie2fn.cu:2466-2743) are symbols here too, with the same
 * signatures: a GGUF file (qwen3next tensor names) loaded into the decode step below on the current GPU.
 */
#ifndef FAIE2FN_H
#define FAIE2FN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- errors and settings ---------------------------------------------------------------------------------- */

/* Message of the last failed call. Replaces fn_error (engine/faie2fn.cu:2495). */
const char *fn_error(void);

/* Device used by the test / bench hooks; also made current. New: the reference hard-codes devices 0 and 1
 * (engine/faie2fn.cu:2757, 2826). */
int fn_set_device(int dev);

/* Programmatic dependent launch on/off. Replaces fn_pdl (engine/faie2fn.cu:2800). */
void fn_pdl(int on);
/* GEMVs marked early run beside the kernel before them, on/off. Replaces fn_early (engine/faie2fn.cu:2802). */
void fn_early(int on);
/* 1: fn_bench_gemv replays one hot copy without an L2 flush. Replaces fn_bench_hot (engine/faie2fn.cu:2822). */
void fn_bench_hot(int on);
/* The reference's GEMV plan override for weights planned from now on (engine/faie2fn.cu:2786-2791), same arguments:
 * tb = threads per CTA (0: automatic), warps_per_sm = target warps per SM (default 16). wpt and ks (weights per
 * thread, split-K) have no counterpart in this plan (a row never spans warps): accepted and ignored. */
void fn_gemv_override(int wpt, int ks, int tb, int warps_per_sm);
/* This plan's own knobs for sweeps: warps per CTA (0: automatic by weight size, < 0 keeps), shared-memory ring KiB
 * (all warps' rings), stage KiB (unused by the per-warp rings), CTAs per SM (> 0 sets). No reference counterpart. */
void fn_gemv_tune(int warps, int ring_kb, int stage_kb, int ctas_per_sm);
/* MoE layer variant, the reference's A/B switch (engine/faie2fn.cu:2799): 0 (default) = a routing kernel before
 * gate/up, 1 = one token on one GPU routed inside the gate/up and down kernels, 2 = one token on one GPU in one fused
 * gate/up + down kernel. */
void fn_moe_var(int v);
/* Q4_K / Q6_K GEMVs of 1..4 tokens with rows of up to 2048 columns: 1 = exact integer products on the tensor cores
 * (tcgen05.mma kind::i8), 0 (default) = the CUDA-core GEMV. No reference counterpart (this build's A/B switch). */
void fn_qmma(int on);
/* The reference's routed-expert launch shapes (engine/faie2fn.cu:2801-2806); the B200 MoE kernels size themselves
 * from the layer's shape and the SM count: accepted and ignored. */
void fn_moe_override(int gu_wpt, int gu_tb, int dn_wpt, int dn_tb);
/* CTAs per SM of the GEMV grid. Replaces fn_gemv_waves (engine/faie2fn.cu:2793). */
void fn_gemv_waves(int ctas_per_sm);
/* Plan of a rows x cols weight: out[7] = {lanes per row, groups per lane, rows per stage, ring slots, CTAs,
 * threads, row stride bytes}. Replaces fn_gemv_plan (engine/faie2fn.cu:2809-2815). */
int fn_gemv_plan(uint32_t type, int rows, int cols, int *out);

/* ---- model-free test / bench hooks ------------------------------------------------------------------------ */

/* out[r][c] = dequant(W)[r][c]: W is rows GGUF rows of `type` (rows x row_bytes), out rows x cols fp32.
 * Bit-identical to gguf-py 0.19.0. Replaces fn_test_dequant (engine/faie2fn.cu:2751-2782). */
int fn_test_dequant(uint32_t type, const uint8_t *W, int rows, int cols, float *out);

/* y[t][r] = sum_c dequant(W)[r][c] x[t][c] for t < nt <= 8; x nt x cols, y nt x rows, fp32.
 * Replaces fn_test_gemv (engine/faie2fn.cu:2914-2935). */
int fn_test_gemv(uint32_t type, const uint8_t *W, int rows, int cols, const float *x, int nt, float *y);

/* ms per GEMV call, weights cold in L2 (rotating copies, L2 flushed, iters calls replayed as one CUDA graph).
 * Replaces fn_bench_gemv (engine/faie2fn.cu:2823-2866). */
int fn_bench_gemv(uint32_t type, int rows, int cols, int nt, int iters, float *ms);

/* ---- resident weights (device-pointer interface; new, the engine-internal QW of engine/faie2fn.cu:1940-1948
 * exposed so callers that own device memory and streams can drive the GEMV) ---------------------------------- */

/* Upload GGUF rows to the current device; returns a handle >= 1 or -1. Replaces load_qw
 * (engine/faie2fn.cu:2125-2142) for one tensor. */
int fn_w_create(uint32_t type, const uint8_t *W, int rows, int cols);
int fn_w_free(int h);
/* GGUF bytes of the weight (rows x row_bytes), the bytes one GEMV must read. */
double fn_w_bytes(int h);
/* Launch y[t][r] (+)= W[r] . x[t] for t < nt <= 8 on a CUDA stream (device pointers, token strides xs, ys in
 * floats; x 16-byte aligned). flags: bit 0 adds into y; bit 1 = early (x was complete before the previous kernel in
 * the stream started, and the previous kernel does not read y: read x without waiting, wait for the previous kernel
 * before exiting). Replaces gemv()
 * (engine/faie2fn.cu:2250-2281) and its acc / early arguments. */
int fn_w_gemv(int h, const float *x, int xs, float *y, int ys, int nt, int flags, void *stream);
/* The same with host buffers x (nt x cols) and y (nt x rows), copied on the stream; does not synchronise. */
int fn_w_gemv_host(int h, const float *x, int nt, float *y, void *stream);
/* A decode step's GEMVs, one token each, on host buffers: x = the inputs of handles[0..n) back to back (cols_i floats
 * each), y = the outputs back to back (rows_i floats each, the lm_head's left out); head (-1: none) = the position in
 * handles of the lm_head, whose argmax goes to *index instead of its logits. One host->device copy, the GEMVs as one
 * CUDA graph (built on the first call for a list of handles, then replayed), one device->host copy; does not
 * synchronise. New: the reference's fn_forward (engine/faie2fn.cu:2733) runs a whole step per call; this is that
 * call's shape for the GEMV path. */
int fn_w_step_host(int n, const int *handles, const float *x, float *y, int head, int *index, void *stream);
/* ---- the rest of a decode step (device pointers, on a stream) --------------------------------
 * h = dequant(E[tokens[*pos]]) (GGUF rows). Replaces k_embed (engine/faie2fn.cu:1334-1347). */
int fn_embed(uint32_t type, const uint8_t *E, int D, const int *tokens, const int *pos, float *h, void *stream);
/* out = x * rsqrt(mean(x^2) + eps) * w. Replaces k_groupnorm (engine/faie2fn.cu:1222-1235) for one stream. */
int fn_rmsnorm(const float *x, const float *w, float *out, int D, float eps, void *stream);
/* Gated attention of one token at position *pos (head dim 256, RoPE on the first 64 dims): q / k head RMSNorm, RoPE,
 * k / v appended to the caches [max_ctx][nkv][256], out [nh][256] = softmax(q.k / 16) v * sigmoid(gate). Replaces
 * k_qk_norm_rope + k_attn_split + k_attn_combine (engine/faie2fn.cu:1452-1478, 1598-1690), without the QSA indexer. */
int fn_attn_decode(const float *qg, const float *k, const float *v, const float *wq, const float *wk,
                   const float *inv_freq, float *Q, float *Kc, float *Vc, float *out, const int *pos, int nh, int nkv,
                   int max_ctx, float eps, void *stream);
/* *pos += 1 and, once the prompt tokens[0..*prompt_len) is consumed, tokens[*pos] = *next (all device memory).
 * Replaces k_advance (engine/faie2fn.cu:1905) and the host's token feedback, so a decode step replays as one CUDA
 * graph for any prompt. */
int fn_step_advance(int *pos, int *tokens, const int *next, const int *prompt_len, int max_ctx, void *stream);

/* Synchronise a stream and report any device-side error (a bounded wait that ran out). */
int fn_sync(void *stream);

/* ---- lm_head argmax (k_argmax, engine/faie2fn.cu:1910-1935; lm_head + argmax at :2446-2447) ----------------
 * Selection rule everywhere: the largest value wins, the lowest index among equal values; NaN never wins; -0 ranks
 * as +0; index 0 when no value exceeds -inf. */

/* The lm_head GEMV with the argmax fused into its epilogue (device pointers, on a stream). y nullable (logits not
 * written); index[t] nullable = winning global row (row0 + local row); keys[t] nullable (may be a peer GPU's memory)
 * = the winner's 64-bit ordering key, for combining the row slices of a split lm_head by max. flags as fn_w_gemv.
 * One such call at a time per handle. Replaces gemv(e.head) followed by k_argmax. */
int fn_w_gemv_argmax(int h, const float *x, int xs, float *y, int ys, int nt, int flags, int row0, int *index,
                     unsigned long long *keys, void *stream);
/* The same with host buffers (x [nt][cols] in; y nullable [nt][rows] and index [nt] out); does not synchronise. */
int fn_w_gemv_argmax_host(int h, const float *x, int nt, float *y, int *index, void *stream);
/* Stand-alone argmax of logits [nt][n] (token stride ls, device pointers; nt <= 1024) into out[nt]. Replaces
 * k_argmax. Its scratch is file-scope device memory: one stand-alone argmax at a time per device. */
int fn_argmax(const float *logits, int ls, int n, int nt, int *out, void *stream);
/* out[t] = winning index among keys [nranks][nt] (device pointers) of the slices of a row-split lm_head. New: the
 * reference has no multi-GPU lm_head. */
int fn_argmax_keys(const unsigned long long *keys, int nranks, int nt, int *out, void *stream);
/* ---- multi-GPU: peer-memory groups (one process per GPU, CUDA IPC over NVLink) -------------------------------
 * New: the reference runs on at most two GPUs with host-staged copies. Setup per rank: fn_ipc_alloc (this rank's
 * buffer + a 64-byte handle), exchange the handles between the ranks' processes, fn_ipc_open every peer handle,
 * fn_group_create(rank, n, bases) with bases[rank] = the own buffer. Teardown: fn_group_free, a barrier between the
 * processes, fn_ipc_close the peers, fn_ipc_free the own buffer. */
int fn_ipc_alloc(size_t bytes, void **ptr, uint8_t *handle64);
int fn_ipc_open(const uint8_t *handle64, void **ptr);
int fn_ipc_close(void *ptr);
int fn_ipc_free(void *ptr);
int fn_group_create(int rank, int n, void *const *bases, size_t bytes);
int fn_group_free(int group);
/* Row-split lm_head (vocabulary rows [row0, row0 + rows of h) on this rank): the GEMV with fused argmax publishes the
 * slice's winning keys into every rank's buffer and counts its arrival with a release atomic; a one-warp kernel waits
 * (bounded, ~1 s; a timeout gives index -1 and an error at fn_sync) for all ranks and writes the vocabulary-wide
 * winner to index[t] on every rank. y nullable (the rank's logit slice). Every rank makes the same calls in the
 * same order. Replaces gemv(e.head) + k_argmax (engine/faie2fn.cu:2446-2447) when the lm_head is split by rows. */
int fn_w_gemv_argmax_group(int h, int group, const float *x, int xs, float *y, int ys, int nt, int flags, int row0,
                           int *index, void *stream);

/* Expert-parallel MoE layer on a peer group: rank g holds routed experts [g ne / n, (g + 1) ne / n) (Wg / Wu: their
 * ffe GGUF rows each, Wd: their d rows each) and the whole shared expert. Every rank routes every token; a routed
 * slot is computed by its expert's rank, the shared slot by the rank with the fewest routed slots of the token; the
 * down kernel stores its slot outputs into every rank's buffer over NVLink and counts its arrival; a combine kernel
 * waits (bounded) and adds the k + 1 slots in slot order, bit-identical to the one-GPU layer, on every rank.
 * New: the reference has no expert parallelism. Run: device pointers, logits [nt][ls], x, y [nt][d] replicated;
 * acc flags as fn_moe_run. */
int fn_moe_ep_create(uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d, int group, const uint8_t *Wg,
                     const uint8_t *Wu, const uint8_t *Wd, const uint8_t *Wsg, const uint8_t *Wsu, const uint8_t *Wsd);
int fn_moe_ep_run(int h, const float *logits, int ls, const float *x, float *y, int nt, int acc, void *stream);

/* Synchronous hooks on host buffers: k_argmax over logits [nt][n]; the fused lm_head GEMV + argmax on GGUF rows
 * (as fn_test_gemv; y nullable), run twice on the same scratch so the second launch checks the ticket reset. */
int fn_test_argmax(const float *logits, int n, int nt, int *out);
int fn_test_gemv_argmax(uint32_t type, const uint8_t *W, int rows, int cols, const float *x, int nt, float *y,
                        int *index);

/* ---- MoE layer ------------------------------------------------------------------------ */

/* One MoE layer on host buffers: y[t] = sum_{s<k} w[t][s] down_e . (silu(gate_e . x[t]) * (up_e . x[t])) with
 * (sel, w) the top-k routing of logits[t][0..ne) (probability descending, ties to the lower index, renormalised),
 * plus sigmoid(logits[t][ne]) times the shared expert. Routed weights are expert-stacked GGUF rows (gate/up:
 * ne * ffe rows of d columns; down: ne * d rows of ffe columns); shared: ffe (gate/up) and d (down) rows in the same
 * formats. nt <= 32. sel / wsel ([nt][k] int32 / fp32) may be NULL. New hook with the conventions of fn_test_gemv;
 * replaces the per-layer MoE of layer_forward (engine/faie2fn.cu:2406-2420: k_route, moe_gu, moe_down, k_hc_add). */
int fn_test_moe(uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d, int nt, const uint8_t *Wg,
                const uint8_t *Wu, const uint8_t *Wd, const uint8_t *Wsg, const uint8_t *Wsu, const uint8_t *Wsd,
                const float *logits, const float *x, float *y, int *sel, float *wsel);
/* Resident MoE weights on the current device (arguments as fn_test_moe); a handle >= 1 or -1. Replaces the expert
 * loads of fn_load (engine/faie2fn.cu:2651-2668). */
int fn_moe_create(uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d, const uint8_t *Wg,
                  const uint8_t *Wu, const uint8_t *Wd, const uint8_t *Wsg, const uint8_t *Wsu, const uint8_t *Wsd);
int fn_moe_free(int h);
/* Launch one MoE layer on device pointers: logits [nt][ls] (ls >= ne + 1), x [nt][d] -> y [nt][d], nt <= 32 (three kernels:
 * routing, gate/up, down + combine). acc flags: bit 0 adds into y; bit 1 = x early: x was complete before the kernel
 * before this call started (e.g. the router GEMV's predecessor wrote it), so the gate/up kernel reads it beside the
 * routing kernel, as an early GEMV does (engine/faie2fn.cu:2247-2249). */
int fn_moe_run(int h, const float *logits, int ls, const float *x, float *y, int nt, int acc, void *stream);
/* Routing of router outputs given as split-K partials part[ks][8][528] (512 experts, top 10): sel / wsel [nt][10],
 * ms per call over iters graph-replayed calls. variant 0 counts the reference's order out expert by expert (as
 * k_route_ref), 1 runs the engine's routing (as k_route); both rank by fp32 expf(l - max) with ties to the lower
 * index. Replaces fn_bench_route (engine/faie2fn.cu:2873-2912). */
int fn_bench_route(int variant, int nt, int ks, const float *part, int iters, int *sel, float *wsel, float *ms);

/* ---- gated-DeltaNet core ------------------------------------------------------------- */

/* nt tokens of one DeltaNet layer's core on host buffers, tokens_per_launch tokens per kernel launch (1 = decode):
 * conv (kernel 4) + silu, l2norm of q and k, beta = sigmoid(b), decay = exp(ssm_a * softplus(a + dt_bias)), the delta
 * rule S = decay S + k ((v - decay S^T k) beta)^T, o = S^T q / sqrt(ds), out = o rsqrt(mean o^2 + 1e-6) norm_w
 * sigmoid(z); value head h reads key head h % nkh. qkv [nt][2 nkh ds + nvh ds] (q | k | v), z [nt][nvh ds], ab
 * [nt][2 nvh] (alpha | beta), conv_w [convch][4] (oldest input first), dt_bias, ssm_a [nvh], norm_w [ds]; S
 * [nvh][ds][ds] and conv_state [3][convch] are read and updated in place; out [nt][nvh ds]. ds must be 128.
 * Replaces k_gdn's per-layer use (engine/faie2fn.cu:1349-1431, 2386-2389) as a model-free hook. */
int fn_test_gdn(int nkh, int nvh, int ds, int nt, int tokens_per_launch, const float *qkv, const float *z,
                const float *ab, const float *conv_w, const float *dt_bias, const float *ssm_a, const float *norm_w,
                float *S, float *conv_state, float *out);
/* Resident DeltaNet state + parameters on the current device (arguments as fn_test_gdn; S0, conv0 initial state);
 * a handle >= 1 or -1. Replaces the DeltaNet loads and state of fn_load / fn_reset (engine/faie2fn.cu:2617-2640,
 * 2703-2717). */
int fn_gdn_create(int nkh, int nvh, int ds, const float *conv_w, const float *dt_bias, const float *ssm_a,
                  const float *norm_w, const float *S0, const float *conv0);
/* Zero a handle's recurrent state and conv histories (a new sequence), on a stream. */
int fn_gdn_reset(int h, void *stream);
int fn_gdn_free(int h);
/* Launch nt tokens on device pointers (token strides qs, zs, abs_, os in floats); the handle's state advances.
 * prefetch_state = 1 only when this handle's previous launch is two or more kernels back in the stream (the state is
 * then read while the kernel before runs, under programmatic dependent launch); 0 for back-to-back launches. */
int fn_gdn_run(int h, const float *qkv, int qs, const float *z, int zs, const float *ab, int abs_, float *out, int os,
               int nt, int prefetch_state, void *stream);
/* Copy the state to host (S [nvh][ds][ds], conv [3][convch]; either may be NULL); synchronises the device. */
int fn_gdn_get_state(int h, float *S, float *conv);

/* The MoE layer of fn_moe_run for callers that cannot allocate device memory (a host whose memory is all owned by
 * its own pool, or a decode loop that must not pay cudaFree's device synchronisation). No counterpart in the
 * reference. Everything is a device pointer the caller owns: weights as in fn_test_moe, rows at a stride of
 * row_bytes rounded up to 16, 16-byte aligned; logits [nt][ls] (ls >= ne + 1); x, y [nt][d]. The only scratch (the
 * gate/up -> down activations) is a static 256 KiB device array inside the library: 1 <= nt <= 32 and
 * nt * (k + 1) * ffe <= 65536, larger calls fail. All calls share that array, so calls that overlap on the GPU race;
 * keep them in one stream. The first call on a device (and the first after its context is re-created) resolves the
 * array's address there; make it outside stream capture. Allocates nothing. */
int fn_moe_layer_static(uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d, const uint8_t *Wg,
                        const uint8_t *Wu, const uint8_t *Wd, const uint8_t *Wsg, const uint8_t *Wsu, const uint8_t *Wsd,
                        const float *logits, int ls, const float *x, float *y, int nt, void *stream);

/* ---- batched decode on the tensor cores (tcgen05) ------------------------------------------------------------ */
/* Resident weights for the tensor-core batched GEMV: GGUF rows Wh [rows][row_bytes] of any of the 19 formats (cols a
 * multiple of 128). Handle >= 1 or -1. The batched form of gemv() (engine/faie2fn.cu:2250-2281; the reference's k_tgemv
 * takes nt <= 8 on CUDA cores, :734-955). */
int fn_tc_create(uint32_t type, const uint8_t *Wh, int rows, int cols);
int fn_tc_free(int h);
/* y[t][r] = W[r] . x[t] for t < nt <= 32 on a stream (device pointers; token strides xs, ys in floats; x 16-byte
 * aligned): each weight tile dequantised once to bf16 hi/lo pairs and multiplied by all tokens with tcgen05.mma
 * (hi*hi + hi*lo + lo*hi, fp32 accumulation in tensor memory); within 1e-4 of float64 relative to max |y|,
 * deterministic; flags bit 0 adds into y. One call at a time per handle. */
int fn_tc_gemv(int h, const float *x, int xs, float *y, int ys, int nt, int flags, void *stream);
/* The same on host buffers (synchronous), as fn_test_gemv: x [nt][cols] -> y [nt][rows]. */
int fn_test_tc_gemv(uint32_t type, const uint8_t *Wh, int rows, int cols, const float *x, int nt, float *y);
/* Device ms per call of the tensor-core GEMV on random weights streamed from HBM (as fn_bench_gemv), nt tokens. */
int fn_bench_tc_gemv(uint32_t type, int rows, int cols, int nt, int iters, float *ms);

/* ---- batched decode: a batch of independent sequences at one position ---------------------------------------- */
/* h[b] = dequant(E row tokens[b * tstride + *pos]) for b < batch (k_embed per sequence). */
int fn_embed_batch(uint32_t type, const uint8_t *E, int D, const int *tokens, int tstride, const int *pos, float *h,
                   int batch, void *stream);
/* fn_rmsnorm of `rows` rows of D values (row b at b * D). */
int fn_rmsnorm_rows(const float *x, const float *w, float *out, int D, int rows, float eps, void *stream);
/* fn_attn_decode for `batch` sequences: sequence b's qg, k, v rows at b * ss floats after qg, k, v; its Q and out rows
 * at b * nh * 256; its caches at b * max_ctx * nkv * 256 floats into Kc, Vc. */
int fn_attn_decode_batch(const float *qg, const float *k, const float *v, int ss, const float *wq, const float *wk,
                         const float *inv_freq, float *Q, float *Kc, float *Vc, float *out, const int *pos, int nh,
                         int nkv, int max_ctx, int batch, float eps, void *stream);
/* fn_step_advance for `batch` sequences (token ids of sequence b at tokens + b * max_ctx, its argmax at next[b]). */
int fn_step_advance_batch(int *pos, int *tokens, const int *next, const int *prompt_len, int max_ctx, int batch,
                          void *stream);
/* A gated-DeltaNet layer for `batch` independent sequences (zero states); fn_gdn_run_batch runs one token of each
 * (token row b of qkv / z / ab / out is sequence b's). fn_gdn_reset zeroes every sequence. Batched form of k_gdn
 * (engine/faie2fn.cu:1349-1431). */
int fn_gdn_create_batch(int nkh, int nvh, int ds, const float *conv_w, const float *dt_bias, const float *ssm_a,
                        const float *norm_w, int batch);
int fn_gdn_run_batch(int h, const float *qkv, int qs, const float *z, int zs, const float *ab, int abs_, float *out,
                     int os, int prefetch_state, void *stream);

/* ---- L2 prefetch hints for a decode chain (no counterpart in the reference, whose decode reads every weight cold) -- */
/* Device address and byte size of a resident weight (rows at the handle's 16-byte stride). */
int fn_w_weights(int h, const void **ptr, uint64_t *bytes);
/* From now on every launch of GEMV handle h, or the down kernel of MoE handle h, also prefetches [ptr, ptr + bytes) of
 * device memory into L2, spread over its CTAs, before its wait for the previous kernel: read-only data that a later
 * kernel of the chain reads (the next weight of a decode step). ptr 16-byte aligned (NULL clears); bytes rounded
 * down to 16. */
int fn_w_prefetch_after(int h, const void *ptr, uint64_t bytes);
int fn_moe_prefetch_after(int h, const void *ptr, uint64_t bytes);
/* RMSNorm folded into the consumer (the reference launches k_groupnorm before each normed GEMV / MoE layer,
 * engine/faie2fn.cu:1222-1235 and its callers :2380-2447): from now on GEMV handle h computes
 * y[t] = rsqrt(mean x[t]^2 + eps) (W . (x[t] * w)) from the raw x, and MoE layer h takes rmsnorm(x) * w as its input.
 * w: the norm weight (cols / d floats of device memory, 16-byte aligned, kept by reference); NULL turns it off. */
int fn_w_norm(int h, const float *w, float eps);
int fn_moe_norm(int h, const float *w, float eps);

/* ---- the decode step (the reference's layer_forward + forward, engine/faie2fn.cu:2370-2490) --------------------
 * One step of the hybrid MoE decoder over resident handles (fn_w_create, fn_gdn_create, fn_moe_create) and device
 * buffers the caller owns: the embedding row of tokens[*pos], per layer the input projection, the gated-DeltaNet core
 * or the gated attention, the output projection adding into the residual, the router and the MoE layer adding into the
 * residual; the lm_head with its fused argmax into *next; *pos += 1 and, past the prompt, tokens[*pos] = *next. */
typedef struct fn_layer_t {
    int kind;                      /* 0: gated DeltaNet layer, 1: gated attention layer */
    int w_in[3];                   /* input projection GEMV handle(s), outputs one after another (unused: 0):
                                    * DeltaNet [q k v z | alpha beta], attention [q gate | k | v] */
    int w_in_rows[3];              /* rows of each */
    int w_out;                     /* output projection (its result is added into the residual) */
    int gdn;                       /* DeltaNet core (kind 0) */
    int router;                    /* router GEMV: ne expert rows, then the shared-expert gate row */
    int moe;                       /* MoE layer */
    const float *norm1, *norm2;    /* RMSNorm weights before the mixer and before the MoE layer [D] */
    const float *q_norm, *k_norm;  /* attention q / k head norms [256] (kind 1) */
    float *Kc, *Vc;                /* attention caches [max_ctx][nkv][256] (kind 1) */
} fn_layer_t;
typedef struct fn_model_t {
    int D, nkh, nvh, nh, nkv, ne, vocab, max_ctx;
    float eps;
    uint32_t embed_type;
    const uint8_t *embed;          /* token embedding, GGUF rows [vocab] */
    int head;                      /* lm_head GEMV handle */
    const float *final_norm;       /* [D] */
    const float *inv_freq;         /* RoPE inverse frequencies [32] (attention layers) */
    int fuse_norm;                 /* 1: every RMSNorm folded into its consumers (fn_w_norm / fn_moe_norm); 0: launched */
    int prefetch;                  /* 1: L2 prefetch hints along the chain (fn_w_prefetch_after) */
    float *hidden, *xnorm;         /* residual [D]; normed input [D] (fuse_norm 0 only) */
    float *proj, *core, *Q, *att;  /* input projection output, DeltaNet output [nvh 128], attention q / output [nh 256] */
    float *router_out;             /* [ne + 1] */
    float *logits;                 /* [vocab], nullable (not written) */
    int *tokens, *pos, *next, *prompt_len;  /* [max_ctx], position, argmax, prompt length */
} fn_model_t;
/* Create a step (validates, and sets the norm folding and prefetch hints on the handles, which must belong to this
 * step alone); a handle >= 1 or -1. No reference counterpart as a symbol (the reference's step is inside fn_forward). */
int fn_decoder_create(const fn_model_t *m, const fn_layer_t *layers, int n_layers);
int fn_decoder_free(int h);
/* One step on a stream (capturable). dbg (host, nullable): the residual after layer l copied to dbg + l * dbg_stride. */
int fn_decoder_step(int h, void *stream, float *dbg, int64_t dbg_stride);
/* Kernel launches of one step. */
int fn_decoder_launches(int h);

/* ---- the reference's model hooks (engine/faie2fn.cu:2497-2743) ------------------------------------------------
 * fn_load reads a GGUF v3 model (shard2 nullable: one file; otherwise the tensors of both) with the qwen3next tensor
 * names onto the current GPU (split is accepted and every layer stays on this GPU; fn_split reads back the layer count)
 * and builds the decode step with its CUDA graph. fn_forward runs nt (1..8) tokens at n_past: argmax[i] = the greedy
 * next id after token i, logits (nullable) [nt][vocab]; errors "not loaded", "nt out of range", "context full". */
int fn_load(const char *shard1, const char *shard2, int max_ctx, int split);
int fn_forward(const int *tokens, int nt, float *logits, int *argmax);
int fn_reset(void);
void fn_free(void);
/* The residual after every layer of the following forwards into out [layers][nt][D] (host; kept until reset with
 * NULL); those forwards then step eagerly. */
int fn_debug_layers(float *out);
/* CUDA graph replay on / off (the graph is recaptured at the next forward either way). */
int fn_use_graphs(int on);
int fn_n_past(void);
double fn_last_ms(void);
/* Weight GB on device dv (this GPU: all of them; -1 when not loaded). */
double fn_dev_gb(int dv);
int fn_split(void);
/* Sizes of the loaded model: out[4] = {vocab, hidden size, layers, max_ctx} (the reference's fn.py keeps these as
 * module constants, flashnext/fn.py:11-13; no counterpart symbol). */
int fn_model_dims(int *out);

#ifdef __cplusplus
}
#endif

#endif /* FAIE2FN_H */
