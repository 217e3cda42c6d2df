// The kernels a whole decode step needs besides the GEMV, MoE and DeltaNet ones: token embedding, RMSNorm, the gated
// attention layer's q/k norm + RoPE + KV-cache append and its decode attention, and the step counter. With them the
// engine runs the synthetic hybrid MoE of BASELINE config 5 end to end (flashnext/model.py builds the step).
//
// Reference behaviour: k_embed (engine/faie2fn.cu:1334-1347: one GGUF row of the token embedding, dequantised),
// k_groupnorm (:1222-1235: x * rsqrt(mean x^2 + eps) * w), k_qk_norm_rope (:1452-1478: per head RMSNorm over the head
// dim, times the shared q / k weights, RoPE on the first NROT dims as pairs (i, i + NROT/2) with angle pos * inv_freq[i],
// keys and values appended to the cache at the position held in device memory), k_attn_split / k_attn_combine
// (:1598-1690: softmax(q . k / sqrt(head dim)) v over the cached positions, q head h reading kv head h / (NH / NKV),
// the output times sigmoid(gate), the gate being the second half of the head's q projection). The QSA indexer that
// prunes the reference's attention is not part of this path.
//
// B200 design: the step's position and token ids live in device memory, so one decode step is one CUDA graph replayed
// once per token with no host work in between; every kernel is a single small grid chained by programmatic launch.
// Reductions run in a fixed order (warp shuffles, then the warps in order), so a step's result does not depend on the
// launch or the token.
#include "fn_engine.h"
#include "fn_rowdot.cuh"

namespace fn {

constexpr int ATT_HD = 256;   // attention head dim (one thread per dim)
constexpr int ATT_NROT = 64;  // rotary dims

// fixed-order block sum: warp butterflies, then warp 0 adds the warp partials in order; every thread gets the sum
template <int NW> __device__ __forceinline__ float block_sum_fixed(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) s += red[w];
    __syncthreads();
    return s;
}
template <int NW> __device__ __forceinline__ float block_max_fixed(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) s = fmaxf(s, red[w]);
    __syncthreads();
    return s;
}

// ---- embedding: h = dequant(E[tokens[*pos]]), one CTA
template <uint32_t TY>
__global__ void k_embed(const uint8_t *__restrict__ E, uint64_t rb, const int *__restrict__ tokens,
                        const int *__restrict__ pos, float *__restrict__ h, int D, int tstride) {
    pdl_wait();
    pdl_trigger();
    // CTA b: sequence b of a batch (its token ids at b * tstride, its row of h at b * D)
    h += (size_t)blockIdx.x * D;
    const int tok = after_wait(tokens)[(size_t)blockIdx.x * tstride + *after_wait(pos)];
    const uint8_t *row = E + (size_t)tok * rb;
    const uint32_t *grid = dev_grid<TY>();
    for (int g = threadIdx.x; g < D / 32; g += blockDim.x) {
        const auto v = load_group<TY>(row, g, grid);
#pragma unroll
        for (int j = 0; j < 32; j += 4) *(float4 *)(h + g * 32 + j) = v.quad(j);
    }
}

// ---- RMSNorm: out = x * rsqrt(mean x^2 + eps) * w, one CTA of 256 threads, D % 1024 == 0 ... any D % 4 == 0
__global__ void __launch_bounds__(256) k_rmsnorm(const float *__restrict__ x, const float *__restrict__ w,
                                                 float *__restrict__ out, int D, float eps) {
    __shared__ float red[8];
    pdl_wait();
    pdl_trigger();
    const float *xp = after_wait(x) + (size_t)blockIdx.x * D;  // CTA b: row b
    out += (size_t)blockIdx.x * D;
    float ss = 0.0f;
    for (int i = threadIdx.x * 4; i < D; i += 1024) {
        const float4 v = *(const float4 *)(xp + i);
        ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(v.x * v.x, v.y * v.y), __fadd_rn(v.z * v.z, v.w * v.w)));
    }
    const float r = rsqrtf(block_sum_fixed<8>(ss, red) / (float)D + eps);
    for (int i = threadIdx.x * 4; i < D; i += 1024) {
        const float4 v = *(const float4 *)(xp + i), wv = *(const float4 *)(w + i);
        *(float4 *)(out + i) = make_float4(v.x * r * wv.x, v.y * r * wv.y, v.z * r * wv.z, v.w * r * wv.w);
    }
}

// ---- attention, part 1: q heads (NH), k heads (NKV), v heads (NKV); one CTA of ATT_HD threads each
struct AttnQkvArgs {
    const float *qg;  // [NH][2 HD]: q, then the gate
    const float *k, *v;  // [NKV][HD]
    const float *wq, *wk;  // [HD]
    const float *inv_freq;  // [NROT / 2]
    float *Q;               // [NH][HD]
    float *Kc, *Vc;         // [max_ctx][NKV][HD]
    const int *pos;
    int nh, nkv, max_ctx;
    float eps;
    int ss;  // a batch of sequences (gridDim.y): floats between sequence b's qg, k and v rows
};

__global__ void __launch_bounds__(ATT_HD) k_attn_qkv(const AttnQkvArgs a) {
    __shared__ float red[ATT_HD / 32];
    __shared__ float buf[ATT_HD];
    pdl_wait();
    pdl_trigger();
    const int j = blockIdx.x, d = threadIdx.x, p = *after_wait(a.pos), b = blockIdx.y;
    if (p >= a.max_ctx) return;  // past the cache: the host checks the length first
    const size_t cache = (size_t)b * a.max_ctx * a.nkv * ATT_HD, row = (size_t)b * a.ss;
    float *Kc = a.Kc + cache, *Vc = a.Vc + cache;
    if (j >= a.nh + a.nkv) {     // values
        const int kv = j - a.nh - a.nkv;
        Vc[((size_t)p * a.nkv + kv) * ATT_HD + d] = after_wait(a.v)[row + kv * ATT_HD + d];
        return;
    }
    const bool isq = j < a.nh;
    const float x = isq ? after_wait(a.qg)[row + (size_t)j * 2 * ATT_HD + d] : after_wait(a.k)[row + (j - a.nh) * ATT_HD + d];
    const float ss = block_sum_fixed<ATT_HD / 32>(x * x, red);
    buf[d] = x * rsqrtf(ss / (float)ATT_HD + a.eps) * (isq ? a.wq[d] : a.wk[d]);
    __syncthreads();
    float y = buf[d];
    if (d < ATT_NROT) {
        const int i = d % (ATT_NROT / 2);
        // the angle reaches thousands of radians at long contexts: formed and reduced in double, so the rotation
        // keeps fp32 accuracy at every position (64 threads of one CTA per head: the cost is nil)
        double sd, cd;
        sincos((double)p * (double)a.inv_freq[i], &sd, &cd);
        const float cs = (float)cd, sn = (float)sd;
        const float x0 = buf[i], x1 = buf[i + ATT_NROT / 2];
        y = d < ATT_NROT / 2 ? x0 * cs - x1 * sn : x1 * cs + x0 * sn;
    }
    if (isq) a.Q[((size_t)b * a.nh + j) * ATT_HD + d] = y;
    else Kc[((size_t)p * a.nkv + (j - a.nh)) * ATT_HD + d] = y;
}

// ---- attention, part 2: one CTA per q head over the positions 0..pos; out = softmax(q . k / 16) v * sigmoid(gate)
struct AttnArgs {
    const float *Q, *Kc, *Vc, *qg;
    float *out;  // [NH][HD] per sequence
    const int *pos;
    int nh, nkv, max_ctx;
    int ss;  // a batch of sequences (gridDim.y): floats between sequence b's qg rows
};

__global__ void __launch_bounds__(ATT_HD) k_attn_decode(const AttnArgs a) {
    extern __shared__ float sc[];  // [max_ctx] scores
    __shared__ float q[ATT_HD];
    __shared__ float red[ATT_HD / 32];
    pdl_wait();
    pdl_trigger();
    const int h = blockIdx.x, d = threadIdx.x, warp = d >> 5, lane = d & 31, b = blockIdx.y;
    const int n = min(*after_wait(a.pos), a.max_ctx - 1) + 1, kv = h / (a.nh / a.nkv);
    q[d] = after_wait(a.Q)[((size_t)b * a.nh + h) * ATT_HD + d];
    __syncthreads();
    const size_t cache = (size_t)b * a.max_ctx * a.nkv * ATT_HD;
    const float *Kc = after_wait(a.Kc) + cache, *Vc = after_wait(a.Vc) + cache;
    // scores: keys t = warp, warp + 8, .. by one warp each, 8 dims per lane; a warp loads its next 4 keys at once (one
    // memory round trip for four keys), each key's sum in the same order as one at a time
    float qr[ATT_HD / 32];
#pragma unroll
    for (int i = 0; i < ATT_HD / 32; ++i) qr[i] = q[lane + 32 * i];
    constexpr int KB = 4, WS = ATT_HD / 32;
    for (int t0 = warp; t0 < n; t0 += KB * WS) {
        float kv_[KB][ATT_HD / 32];
#pragma unroll
        for (int u = 0; u < KB; ++u) {
            const int t = t0 + u * WS;
            const float *kr = Kc + ((size_t)min(t, n - 1) * a.nkv + kv) * ATT_HD;
#pragma unroll
            for (int i = 0; i < ATT_HD / 32; ++i) kv_[u][i] = kr[lane + 32 * i];
        }
#pragma unroll
        for (int u = 0; u < KB; ++u) {
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < ATT_HD / 32; ++i) s = __fmaf_rn(qr[i], kv_[u][i], s);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            const int t = t0 + u * WS;
            if (lane == 0 && t < n) sc[t] = s * 0.0625f;  // 1 / sqrt(256)
        }
    }
    __syncthreads();
    float m = -INFINITY;
    for (int t = d; t < n; t += ATT_HD) m = fmaxf(m, sc[t]);
    m = block_max_fixed<ATT_HD / 32>(m, red);
    for (int t = d; t < n; t += ATT_HD) sc[t] = expf(sc[t] - m);
    __syncthreads();
    float l = 0.0f, o = 0.0f;
    const float *vp = Vc + (size_t)kv * ATT_HD + d;
    const size_t vs = (size_t)a.nkv * ATT_HD;
#pragma unroll 8
    for (int t = 0; t < n; ++t) {  // every thread the same order: l is identical in all threads
        const float e = sc[t];
        l += e;
        o = __fmaf_rn(e, vp[(size_t)t * vs], o);
    }
    const float gate = after_wait(a.qg)[(size_t)b * a.ss + (size_t)h * 2 * ATT_HD + ATT_HD + d];
    a.out[((size_t)b * a.nh + h) * ATT_HD + d] = (o / l) * sigm(gate);
}

// ---- the step counter: the token the step predicted becomes the next input once the prompt is consumed
// thread b: sequence b of a batch (its token ids at b * max_ctx); one position for all
__global__ void k_step_advance(int *pos, int *tokens, const int *next, const int *prompt_len, int max_ctx, int batch) {
    pdl_wait();
    pdl_trigger();
    const int p = *pos, b = threadIdx.x;
    if (b < batch && p + 1 < max_ctx && p + 1 >= *prompt_len) tokens[(size_t)b * max_ctx + p + 1] = next[b];
    __syncthreads();
    if (b == 0) *pos = p + 1;
}

int launch_embed(uint32_t type, const uint8_t *E, uint64_t rb, const int *tokens, const int *pos, float *h, int D,
                 cudaStream_t s, int batch = 1, int tstride = 0) {
    if (D % 32 || row_bytes(type, D) != rb) return fail("embed: bad type/width");
    if (batch < 1 || batch > 65535) return fail("embed: batch out of range");
    cudaError_t e = cudaSuccess;
    const bool known = dispatch_type(type, [&]<uint32_t TY>() {
        e = launch_k(k_embed<TY>, dim3(batch), dim3(256), 0, s, E, rb, tokens, pos, h, D, tstride);
    });
    if (!known) return fail("embed: unsupported type");
    if (e != cudaSuccess) return fail(std::string("embed launch: ") + cudaGetErrorString(e));
    return 0;
}

}  // namespace fn

using namespace fn;

// ---- C ABI (device pointers, on a stream; no synchronisation) ------------------------------------------------------

// h[0..D) = dequant(E row tokens[*pos]) for GGUF rows E (row stride row_bytes(type, D)). Replaces k_embed
// (engine/faie2fn.cu:1334-1347).
FN_API int fn_embed(uint32_t type, const uint8_t *E, int D, const int *tokens, const int *pos, float *h, void *stream) {
    return launch_embed(type, E, row_bytes(type, D), tokens, pos, h, D, (cudaStream_t)stream);
}

// out = x * rsqrt(mean(x^2) + eps) * w over D values (D % 4 == 0, 16-byte aligned). Replaces k_groupnorm
// (engine/faie2fn.cu:1222-1235) for one stream.
// h[b][0..D) = dequant(E row tokens[b * tstride + *pos]) for b < batch (batched decode: one position for all).
FN_API int fn_embed_batch(uint32_t type, const uint8_t *E, int D, const int *tokens, int tstride, const int *pos,
                          float *h, int batch, void *stream) {
    return launch_embed(type, E, row_bytes(type, D), tokens, pos, h, D, (cudaStream_t)stream, batch, tstride);
}

// fn_rmsnorm of `rows` rows of D values each (row b at b * D floats of x and out).
FN_API int fn_rmsnorm_rows(const float *x, const float *w, float *out, int D, int rows, float eps, void *stream) {
    if (D < 4 || D % 4 || rows < 1 || rows > 65535) return fail("rmsnorm: bad width / rows");
    const cudaError_t e = launch_k(k_rmsnorm, dim3(rows), dim3(256), 0, (cudaStream_t)stream, x, w, out, D, eps);
    if (e != cudaSuccess) return fail(std::string("rmsnorm launch: ") + cudaGetErrorString(e));
    return 0;
}

FN_API int fn_rmsnorm(const float *x, const float *w, float *out, int D, float eps, void *stream) {
    if (D < 4 || D % 4) return fail("rmsnorm: D must be a positive multiple of 4");
    const cudaError_t e = launch_k(k_rmsnorm, dim3(1), dim3(256), 0, (cudaStream_t)stream, x, w, out, D, eps);
    if (e != cudaSuccess) return fail(std::string("rmsnorm launch: ") + cudaGetErrorString(e));
    return 0;
}

// Gated attention for one token at position *pos (head dim 256, RoPE on the first 64 dims): qg [nh][512] (q then gate
// per head), k, v [nkv][256] -> the q heads normed and rotated into Q [nh][256], k (normed, rotated) and v appended to
// the caches Kc, Vc [max_ctx][nkv][256] at *pos, then out [nh][256] = softmax(q . k / 16) v * sigmoid(gate) over the
// positions 0..*pos. inv_freq [32] = rope_base^(-2i / 64). Replaces k_qk_norm_rope + k_attn_split + k_attn_combine
// (engine/faie2fn.cu:1452-1478, 1598-1690) without the QSA indexer.
static int attn_launch(const float *qg, const float *k, const float *v, int ss, const float *wq, const float *wk,
                       const float *inv_freq, float *Q, float *Kc, float *Vc, float *out, const int *pos, int nh, int nkv,
                       int max_ctx, int batch, float eps, cudaStream_t s) {
    if (nh < 1 || nkv < 1 || nh % nkv || max_ctx < 1 || max_ctx > 12288) return fail("attn: bad head counts / context");
    if (batch < 1 || batch > 65535) return fail("attn: batch out of range");
    AttnQkvArgs a{qg, k, v, wq, wk, inv_freq, Q, Kc, Vc, pos, nh, nkv, max_ctx, eps, ss};
    cudaError_t e = launch_k(k_attn_qkv, dim3(nh + 2 * nkv, batch), dim3(ATT_HD), 0, s, a);
    if (e != cudaSuccess) return fail(std::string("attn qkv launch: ") + cudaGetErrorString(e));
    AttnArgs b{Q, Kc, Vc, qg, out, pos, nh, nkv, max_ctx, ss};
    const size_t smem = (size_t)max_ctx * 4;
    static bool attr = false;
    if (!attr) {
        e = cudaFuncSetAttribute(k_attn_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, 48 * 1024);
        if (e != cudaSuccess) return fail(std::string("attn attribute: ") + cudaGetErrorString(e));
        attr = true;
    }
    e = launch_k(k_attn_decode, dim3(nh, batch), dim3(ATT_HD), smem, s, b);
    if (e != cudaSuccess) return fail(std::string("attn launch: ") + cudaGetErrorString(e));
    return 0;
}

// Gated attention for one token at position *pos (head dim 256, RoPE on the first 64 dims): qg [nh][512] (q then gate
// per head), k, v [nkv][256] -> the q heads normed and rotated into Q [nh][256], k (normed, rotated) and v appended to
// the caches Kc, Vc [max_ctx][nkv][256] at *pos, then out [nh][256] = softmax(q . k / 16) v * sigmoid(gate) over the
// positions 0..*pos. inv_freq [32] = rope_base^(-2i / 64). Replaces k_qk_norm_rope + k_attn_split + k_attn_combine
// (engine/faie2fn.cu:1452-1478, 1598-1690) without the QSA indexer.
FN_API int fn_attn_decode(const float *qg, const float *k, const float *v, const float *wq, const float *wk,
                          const float *inv_freq, float *Q, float *Kc, float *Vc, float *out, const int *pos, int nh,
                          int nkv, int max_ctx, float eps, void *stream) {
    return attn_launch(qg, k, v, 0, wq, wk, inv_freq, Q, Kc, Vc, out, pos, nh, nkv, max_ctx, 1, eps,
                       (cudaStream_t)stream);
}

// fn_attn_decode for `batch` independent sequences at the same position: sequence b's qg, k and v rows at b * ss floats
// after qg, k, v; its Q and out rows at b * nh * 256; its caches at b * max_ctx * nkv * 256 floats into Kc, Vc.
FN_API int fn_attn_decode_batch(const float *qg, const float *k, const float *v, int ss, const float *wq,
                                const float *wk, const float *inv_freq, float *Q, float *Kc, float *Vc, float *out,
                                const int *pos, int nh, int nkv, int max_ctx, int batch, float eps, void *stream) {
    return attn_launch(qg, k, v, ss, wq, wk, inv_freq, Q, Kc, Vc, out, pos, nh, nkv, max_ctx, batch, eps,
                       (cudaStream_t)stream);
}

// After a step at position *pos: *pos += 1 and, once the prompt (tokens[0..*prompt_len)) is consumed, tokens[*pos] =
// *next (the step's argmax). Every argument lives in device memory, so a captured step serves any prompt. Replaces
// k_advance (engine/faie2fn.cu:1905) and the host's token feedback.
FN_API int fn_step_advance(int *pos, int *tokens, const int *next, const int *prompt_len, int max_ctx, void *stream) {
    const cudaError_t e = launch_k(k_step_advance, dim3(1), dim3(1), 0, (cudaStream_t)stream, pos, tokens, next,
                                   prompt_len, max_ctx, 1);
    if (e != cudaSuccess) return fail(std::string("step advance launch: ") + cudaGetErrorString(e));
    return 0;
}

// fn_step_advance for `batch` sequences at one position: sequence b's token ids at tokens + b * max_ctx, its argmax at
// next[b] (batch <= 1024).
FN_API int fn_step_advance_batch(int *pos, int *tokens, const int *next, const int *prompt_len, int max_ctx, int batch,
                                 void *stream) {
    if (batch < 1 || batch > 1024) return fail("step advance: batch out of range (1..1024)");
    const cudaError_t e = launch_k(k_step_advance, dim3(1), dim3(batch), 0, (cudaStream_t)stream, pos, tokens, next,
                                   prompt_len, max_ctx, batch);
    if (e != cudaSuccess) return fail(std::string("step advance launch: ") + cudaGetErrorString(e));
    return 0;
}
