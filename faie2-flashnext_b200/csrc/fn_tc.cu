// Batched decode GEMV on the 5th-generation tensor cores (tcgen05): y[t][r] = W[r] . x[t] for t < nt <= 32 tokens.
//
// At batch 8..32 the quantised GEMV becomes a dense contraction (rows x cols x nt), so this path dequantises each
// weight tile once and lets tcgen05.mma multiply it by all tokens at once, where the CUDA-core GEMV would repeat the
// FMA work per token (its batched form, k_gemv<.., NT = 8, ..>, runs 8 tokens per call). The reference has no batched
// path (its k_tgemv takes nt <= 8 on CUDA cores, engine/faie2fn.cu:734-955); the operator contract is the same as
// fn_w_gemv's.
//
// Precision: the tensor cores take bf16 operands, so every weight value v (the exact GGUF dequantisation, load_group) and
// every x value is split into v_hi = bf16(v) and v_lo = bf16(v - v_hi), and the products hi*hi + hi*lo + lo*hi are
// accumulated in fp32 in tensor memory: each keeps about 16 mantissa bits (the lo*lo term is below 2^-16 of it), so y
// is within about 3e-5 of float64, relative to max |y| (the stated tolerance is 1e-4). BF16 weights are exact in bf16
// (v_lo = 0), so they take one MMA per step.
//
// Weights on the device: GGUF rows cut into raw chunks of 256 columns (128 for the formats whose 256 columns exceed
// 240 bytes), each chunk padded to a 16-byte multiple and stored tile-major (a chunk of a tile's 128 rows is one
// contiguous run, one bulk copy), so that a chunk starts on a block boundary and a 16-byte boundary (a K-quant block's
// fields then sit 16-byte aligned in shared memory).
//
// One CTA per SM streams its tiles (128 rows) chunk by chunk; warps meet only at mbarriers (no block barrier in the
// loop), and every wait parks the warp in the hardware (try_wait with a suspend-time hint):
//   * one lane issues the raw chunk copies into a ring of up to 8 slots (100-200 KB in flight per SM);
//   * 16 decoder warps turn a step's 128 columns (4 groups of 32) into bf16 hi / lo and store them straight into
//     tensor memory (tcgen05.st; warp w holds lanes 32 (w % 4) .. and group w / 4), which the MMAs read as their A
//     operand, so the weights never pass through shared memory after the copy;
//   * one warp copies each step's x columns of every token into a 4-slot fp32 staging ring (one 512-byte bulk copy per
//     token, one token per lane), and 4 warps convert them into the B operand: x_hi of the N tokens, then x_lo, as
//     2 N rows in the canonical K-major layout without swizzle (8-row x 16-byte core matrices, 8-row groups 128 bytes
//     apart, 8-column groups 2 N x 16 bytes apart);
//   * one lane issues two MMAs per 16-deep step (M = 128, K = 16): A_hi [x_hi | x_lo] with N = 2 npad, and A_lo x_hi
//     with N = npad (the operand's first npad rows), into a tile's accumulators in tensor memory (double-buffered
//     across tiles), and commits them to the buffers' mbarriers; an MMA costs about the same at N = 32 as at N = 64,
//     so the x halves share one instruction;
//   * 4 warps read a finished tile's accumulators (tcgen05.ld), add A_hi x_hi + A_hi x_lo + A_lo x_hi in that order
//     and store y (or the split's partial) while the next tile runs.
// Matrices with fewer tiles than SMs split K instead (one tile per CTA); the tile's last CTA adds the partials in split
// order (release / acquire ticket), so y is deterministic. Every wait is bounded: a wait that runs out records
// DEV_WAIT_TIMEOUT, the CTA waits (bounded) for the copies and MMAs it issued, frees its tensor memory and returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "fn_engine.h"
#include "fn_rowdot.cuh"

namespace fn {

constexpr int TC_M = 128;       // rows per tile (one MMA's M)
constexpr int TC_KC = 128;      // columns per decode step (4 groups of 32, 8 MMA steps of 16)
constexpr int TC_NMAX = 32;     // tokens per call
constexpr int TC_DEC = 16;      // decoder warps: tensor-memory lane quarter w % 4, group w / 4 of a step
constexpr int TC_XW = 4;        // warps staging x (the B operand)
constexpr int TC_EPI = 4;       // read-back warps, one per tensor-memory lane quarter
constexpr int W_X0 = TC_DEC, W_EPI0 = W_X0 + TC_XW, W_COPY = W_EPI0 + TC_EPI, W_XCOPY = W_COPY + 1, W_MMA = W_XCOPY + 1;
constexpr int TC_THREADS = 32 * (W_MMA + 1);  // 864
constexpr int TC_RS_MAX = 8;                  // raw chunk slots at most
constexpr int TC_XS = 4;                      // x staging slots (fp32, every token's 128 columns of a step)
// tensor memory: A buffers [2][hi 64 | lo 64 columns] (bf16 pairs, 128 values of a row), then per tile parity the
// accumulators D1 (A_hi [x_hi | x_lo]: 2 N columns) and D2 (A_lo x_hi: N columns), 128 columns per parity
constexpr uint32_t TC_TA = 0, TC_TACC = 256, TC_TMEM_COLS = 512;
// shared memory: mbarriers, B buffers [2] (x_hi tokens then x_lo tokens: 2 N x 128 bf16, sized for N = 32), x staging
// [TC_XS][32 tokens]
// (rows of 128 fp32 padded to 528 bytes: the converting threads read 8 tokens' rows without bank conflicts), then the
// raw ring
constexpr uint32_t TC_B_BUF = 2 * TC_NMAX * TC_KC * 2;
constexpr uint32_t TC_XROW = TC_KC * 4 + 16, TC_XSLOT = TC_NMAX * TC_XROW;
constexpr uint32_t TC_B_OFF = 1024, TC_X_OFF = TC_B_OFF + 2 * TC_B_BUF, TC_RAW_OFF = TC_X_OFF + TC_XS * TC_XSLOT;
constexpr size_t TC_SMEM_MAX = 227 * 1024 - 2048;  // less the static shared memory

static size_t tc_align(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct TcArgs {
    const uint8_t *W;  // tile-major: raw chunk c of tile T = 128 rows x wbytes at (T * nr + c) * 128 * wbytes
    int rows, nt, npad;  // npad: the MMA's N (16 or 32)
    const float *x;
    int xs;
    float *y;
    int ys, acc;       // acc 1: y += W x (the residual add of a projection)
    int tiles, nr, spr;  // tiles of the matrix; raw chunks per row; decode steps per raw chunk (1 or 2)
    int splits, nr_split;  // K splits (then one tile per CTA), raw chunks per split
    int rs;            // raw ring slots
    uint32_t wbytes;   // bytes of a padded raw chunk of a row (16-byte multiple)
    float *part;        // [splits][32][rows] when splits > 1
    uint32_t *tickets;  // [tiles], zero between launches
    uint32_t *err;
};

// sm_100 shared-memory matrix descriptor: start address, leading / stride byte offsets (>> 4), version 1, no swizzle
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
           (1ull << 46);
}
// instruction descriptor of kind::f16: fp32 accumulator, bf16 A and B, both K-major, N >> 3 and M >> 4
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
// D (+)= A B with A in tensor memory (row i in lane i, two bf16 per 32-bit column along K) and B in shared memory
__device__ __forceinline__ void umma_bf16_tmem_a(uint32_t dtmem, uint32_t atmem, uint64_t b, uint32_t idesc,
                                                 uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(dtmem),
        "r"(atmem), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void async_proxy_fence() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void tc_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// 16 consecutive fp32 columns of this warp's 32 tensor-memory lanes
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 16 consecutive 32-bit columns into this warp's 32 tensor-memory lanes (one row per lane)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};\n" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// the bf16 pair (hi, lo) of 4 values as two 8-byte words
__device__ __forceinline__ void split4(float a, float b, float c, float d, uint2 &hi, uint2 &lo) {
    const __nv_bfloat162 h01 = __floats2bfloat162_rn(a, b), h23 = __floats2bfloat162_rn(c, d);
    const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
    const __nv_bfloat162 l01 = __floats2bfloat162_rn(a - f01.x, b - f01.y), l23 = __floats2bfloat162_rn(c - f23.x, d - f23.y);
    hi = make_uint2(*(const uint32_t *)&h01, *(const uint32_t *)&h23);
    lo = make_uint2(*(const uint32_t *)&l01, *(const uint32_t *)&l23);
}

// two values as bf16 hi / lo words: hi = bf16(v), lo = bf16(v - hi) (v - hi is exact in fp32: one FMA by -1)
__device__ __forceinline__ void split2(float2 v, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
    const uint32_t hw = *(const uint32_t *)&h;
    const float2 hf = make_float2(__uint_as_float(hw << 16), __uint_as_float(hw & 0xFFFF0000u));
    const float2 d = __ffma2_rn(hf, make_float2(-1.0f, -1.0f), v);
    const __nv_bfloat162 l = __floats2bfloat162_rn(d.x, d.y);
    hi = hw;
    lo = *(const uint32_t *)&l;
}
// bytes k, k+1 of w (unsigned) as the floats 2^23 + byte
__device__ __forceinline__ float2 tc_mag2(uint32_t w, int k) {
    return make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u + k)),
                       __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441u + k)));
}
// values v = A (q - off) (+ B) of the four unsigned codes q of word w, as split words 2i, 2i + 1 of hi / lo; the
// same two float32 roundings as gguf-py ((A q) then + B), B = -0 where a format has no offset
template <bool HAS_B>
__device__ __forceinline__ void tc_word(uint32_t w, float off, float A, float B, uint32_t *hi, uint32_t *lo) {
    const float2 mo = make_float2(-(8388608.0f + off), -(8388608.0f + off)), a2 = make_float2(A, A);
    float2 v01 = __fmul2_rn(a2, __fadd2_rn(tc_mag2(w, 0), mo)), v23 = __fmul2_rn(a2, __fadd2_rn(tc_mag2(w, 2), mo));
    if constexpr (HAS_B) {
        v01 = __fadd2_rn(v01, make_float2(B, B));
        v23 = __fadd2_rn(v23, make_float2(B, B));
    }
    split2(v01, hi[0], lo[0]);
    split2(v23, hi[1], lo[1]);
}

// Group g of a staged raw chunk as 16 hi and 16 lo words (values 2i, 2i + 1 in word i). Q4_K and Q6_K decode their
// 16-byte-aligned block fields directly (the values of load_group, bit for bit); the other formats go through
// load_group.
template <uint32_t TY>
__device__ __forceinline__ void tc_group_words(const uint8_t *row, int g, const uint32_t *grid, uint32_t (&hi)[16],
                                               uint32_t (&lo)[16]) {
    if constexpr (TY == T_Q6_K) {
        // a 256-column chunk is one block: ql [128] at 0, qh [64] at 128, int8 scales [16] at 192, fp16 d at 208
        const int s = g & 7, H = s >> 2, sp = s & 3;
        const uint4 l0 = *(const uint4 *)(row + 64 * H + 32 * (sp & 1)), l1 = *(const uint4 *)(row + 64 * H + 32 * (sp & 1) + 16);
        const uint4 h0 = *(const uint4 *)(row + 128 + 32 * H), h1 = *(const uint4 *)(row + 144 + 32 * H);
        const uint32_t sc = u16_at(row + 192 + 2 * s);
        const float d = f16_at(row + 208);
        const float A0 = __fmul_rn(d, (float)(int8_t)(sc & 255u)), A1 = __fmul_rn(d, (float)(int8_t)(sc >> 8));
        const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const int lsh = 4 * (sp >> 1), hsh = 2 * sp;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t th = (hsh <= 4 ? hw[i] << (4 - hsh) : hw[i] >> (hsh - 4)) & 0x30303030u;
            tc_word<false>(((lw[i] >> lsh) & LOW4) | th, 32.0f, i < 4 ? A0 : A1, 0.0f, hi + 2 * i, lo + 2 * i);
        }
    } else if constexpr (TY == T_Q4_K) {
        const uint8_t *blk = row + (g >> 3) * 144;
        const int s = g & 7;
        const uint4 h = *(const uint4 *)blk;  // d, dmin | the 12 packed scale and min bytes
        uint32_t sc, mn;
        kq_scale_min(s, h.y, h.z, h.w, sc, mn);
        const float A = __fmul_rn(f16_of(h.x, 0), __uint2float_rn(sc)), B = -__fmul_rn(f16_of(h.x, 1), __uint2float_rn(mn));
        const uint4 q0 = *(const uint4 *)(blk + 16 + 32 * (s >> 1)), q1 = *(const uint4 *)(blk + 32 + 32 * (s >> 1));
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const int sh = 4 * (s & 1);
#pragma unroll
        for (int i = 0; i < 8; ++i) tc_word<true>((qw[i] >> sh) & LOW4, 0.0f, A, B, hi + 2 * i, lo + 2 * i);
    } else {
        const auto G = load_group<TY>(row, g, grid);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float4 v = G.quad(4 * k);
            split2(make_float2(v.x, v.y), hi[2 * k], lo[2 * k]);
            split2(make_float2(v.z, v.w), hi[2 * k + 1], lo[2 * k + 1]);
        }
    }
}

template <uint32_t TY>
__global__ void __launch_bounds__(TC_THREADS, 1) k_tc_gemv(const __grid_constant__ TcArgs a) {
    constexpr bool EXACT = TY == T_BF16;  // weights exact in bf16: no lo part, one MMA per step
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_fail;
    __shared__ int s_last;
    uint64_t *rfull = (uint64_t *)sm, *rempty = rfull + TC_RS_MAX, *aready = rempty + TC_RS_MAX, *afree = aready + 2,
             *bready = afree + 2, *bfree = bready + 2, *accdone = bfree + 2, *accfree = accdone + 2,
             *xfull = accfree + 2, *xempty = xfull + TC_XS;
    uint8_t *Bs = sm + TC_B_OFF, *xst = sm + TC_X_OFF, *raw = sm + TC_RAW_OFF;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // this CTA's work: tiles [t0, t1), raw chunks [c0, c1) of each of their rows
    int t0, t1, c0, c1, split = 0;
    if (a.splits > 1) {
        t0 = blockIdx.x / a.splits;
        t1 = t0 + 1;
        split = blockIdx.x - t0 * a.splits;
        c0 = split * a.nr_split;
        c1 = min(a.nr, c0 + a.nr_split);
    } else {
        t0 = (int)((long long)blockIdx.x * a.tiles / gridDim.x);
        t1 = (int)((long long)(blockIdx.x + 1) * a.tiles / gridDim.x);
        c0 = 0;
        c1 = a.nr;
    }
    const int nrc = c1 - c0, ntile = t1 - t0, NI = ntile * nrc, NS = NI * a.spr, sps = nrc * a.spr;
    const uint32_t n = (uint32_t)a.npad;
    // a bounded wait that gives up at once when another role already failed
    auto wt = [&](uint64_t *bar, uint32_t par) {
        if (s_fail) return false;
        if (mbar_park(bar, par)) return true;
        s_fail = 1;
        return false;
    };

    if (tid == 0) {
        for (int i = 0; i < TC_RS_MAX; ++i) {
            mbar_init(&rfull[i], 1);
            mbar_init(&rempty[i], TC_DEC);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&aready[i], TC_DEC);
            mbar_init(&afree[i], 1);
            mbar_init(&bready[i], TC_XW);
            mbar_init(&bfree[i], 1);
            mbar_init(&accdone[i], 1);
            mbar_init(&accfree[i], TC_EPI);
        }
        for (int i = 0; i < TC_XS; ++i) {
            mbar_init(&xfull[i], 1);
            mbar_init(&xempty[i], TC_XW);
        }
        mbar_fence_init();
        s_fail = 0;
    }
    if (warp == W_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&s_tmem)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    int n_raw = 0, n_mma = 0, n_x = 0;  // raw chunks / steps / x steps issued by the copy, MMA and x-copy lanes

    if (warp == W_COPY) {
        // ---- raw chunk copies, tile-major; the weights are read-only, so the first ring's copies go before the wait
        // for the previous kernel; every lane then takes part in the wait and the trigger
        auto issue = [&](int i) {
            const int sl = i % a.rs;
            if (i >= a.rs && !wt(&rempty[sl], (uint32_t)((i / a.rs) - 1) & 1u)) return false;
            mbar_arrive_tx(&rfull[sl], (uint32_t)TC_M * a.wbytes);
            bulk_g2s(raw + (size_t)sl * TC_M * a.wbytes,
                     a.W + ((size_t)(t0 + i / nrc) * a.nr + c0 + i % nrc) * TC_M * a.wbytes, (uint32_t)TC_M * a.wbytes,
                     &rfull[sl]);
            n_raw = i + 1;
            return true;
        };
        const int first = min(NI, a.rs);
        if (lane == 0)
            for (int i = 0; i < first; ++i) issue(i);
        __syncwarp();
        pdl_wait();
        pdl_trigger();
        if (lane == 0)
            for (int i = first; i < NI && !s_fail; ++i)
                if (!issue(i)) break;
    } else {
        pdl_wait();
        pdl_trigger();
    }

    if (warp < TC_DEC) {
        // ---- decode: group gl of every step, rows 32 q + lane, into A buffer j & 1 of tensor memory
        const int q = warp & 3, gl = warp >> 2, r = 32 * q + lane;
        const uint32_t *grid = dev_grid<TY>();
        for (int j = 0; j < NS; ++j) {
            const int i = j / a.spr, sub = j - i * a.spr, sl = i % a.rs, b = j & 1;
            bool ok = true;
            if (sub == 0) ok = wt(&rfull[sl], (uint32_t)(i / a.rs) & 1u);
            if (ok && j >= 2) ok = wt(&afree[b], (uint32_t)((j >> 1) - 1) & 1u);
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.st is warp-collective
            if (ok) {
                const int tile = t0 + i / nrc;
                uint32_t hi[16], lo[16];
                if (tile * TC_M + r < a.rows) {
                    tc_group_words<TY>(raw + ((size_t)sl * TC_M + r) * a.wbytes, sub * 4 + gl, grid, hi, lo);
                } else {  // rows past the matrix: zeros (their accumulator lanes are never read)
#pragma unroll
                    for (int k = 0; k < 16; ++k) hi[k] = lo[k] = 0u;
                }
                const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + TC_TA + (uint32_t)b * 128u + 16u * (uint32_t)gl;
                tmem_st16(ta, hi);
                if constexpr (!EXACT) tmem_st16(ta + 64u, lo);
                tmem_wait_st();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                tc_arrive(&aready[b]);
                if (sub == a.spr - 1) tc_arrive(&rempty[sl]);
            }
        }
    } else if (warp < W_EPI0) {
        // ---- x: the step's columns of every token (staged fp32 by the x copies) as bf16 hi / lo into B buffer j & 1;
        // a thread's items are (token t, 8-column group kc) = xi + 128 m; tokens >= nt are zero
        constexpr int XI = TC_NMAX * (TC_KC / 8) / (32 * TC_XW);  // items per thread at N = 32
        const int xi = tid - 32 * W_X0, nitems = (int)n * (TC_KC / 8);
        for (int j = 0; j < NS; ++j) {
            const int b = j & 1, xsl = j % TC_XS;
            bool ok = wt(&xfull[xsl], (uint32_t)(j / TC_XS) & 1u);
            if (ok && j >= 2) ok = wt(&bfree[b], (uint32_t)((j >> 1) - 1) & 1u);
            if (ok) {
                uint8_t *Bb = Bs + (size_t)b * TC_B_BUF;
                const uint8_t *xs_ = xst + (size_t)xsl * TC_XSLOT;
#pragma unroll
                for (int m = 0; m < XI; ++m) {
                    const int it = xi + 32 * TC_XW * m, t = it % (int)n, kc = it / (int)n;
                    if (it >= nitems) break;
                    float4 p = make_float4(0.f, 0.f, 0.f, 0.f), p2 = p;
                    if (t < a.nt) {
                        const float4 *src = (const float4 *)(xs_ + (size_t)t * TC_XROW + 32 * kc);
                        p = src[0];
                        p2 = src[1];
                    }
                    uint2 h0, l0, h1, l1;
                    split4(p.x, p.y, p.z, p.w, h0, l0);
                    split4(p2.x, p2.y, p2.z, p2.w, h1, l1);
                    // K-major, 2 N rows: 8-column groups 2 N x 16 bytes apart, 8-row groups 128 bytes apart
                    const uint32_t kofs = (uint32_t)kc * (2u * n * 16u), tl = (uint32_t)t + n;
                    *(uint4 *)(Bb + kofs + (uint32_t)(t >> 3) * 128u + (uint32_t)(t & 7) * 16u) = make_uint4(h0.x, h0.y, h1.x, h1.y);
                    *(uint4 *)(Bb + kofs + (tl >> 3) * 128u + (tl & 7) * 16u) = make_uint4(l0.x, l0.y, l1.x, l1.y);
                }
            }
            async_proxy_fence();  // the generic-proxy stores before the tensor cores read them
            __syncwarp();
            if (lane == 0) {
                tc_arrive(&bready[b]);
                tc_arrive(&xempty[xsl]);
            }
        }
    } else if (warp == W_XCOPY) {
        // ---- x copies: step j's 128 columns of each of the nt tokens (one 512-byte bulk copy per token), TC_XS steps
        // ahead of the conversion
        // (lane t issues token t's copy after lane 0 set the slot's expected bytes)
        const float *x = after_wait(a.x);
        for (int j = 0; j < NS; ++j) {
            const int xsl = j % TC_XS, i = j / a.spr, sub = j - i * a.spr;
            bool ok = !s_fail;
            if (ok && j >= TC_XS) ok = wt(&xempty[xsl], (uint32_t)((j / TC_XS) - 1) & 1u);
            if (!__all_sync(0xffffffffu, ok)) break;
            const int col0 = (c0 + i % nrc) * (a.spr * TC_KC) + sub * TC_KC;
            if (lane == 0) mbar_arrive_tx(&xfull[xsl], (uint32_t)a.nt * (TC_KC * 4));
            __syncwarp();
            if (lane < a.nt)
                bulk_g2s(xst + (size_t)xsl * TC_XSLOT + (size_t)lane * TC_XROW, x + (size_t)lane * a.xs + col0, TC_KC * 4,
                         &xfull[xsl]);
            n_x = j + 1;
        }
    } else if (warp < W_COPY) {
        // ---- read-back: tile k's accumulator (lanes = its rows) -> y or this split's partial
        const int q = warp & 3, rl = 32 * q + lane;
        for (int k = 0; k < ntile; ++k) {
            const int ab = k & 1;
            bool ok = wt(&accdone[ab], (uint32_t)(k >> 1) & 1u);
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
            tc_fence_after();
            const int r = (t0 + k) * TC_M + rl;
            if (ok) {
                for (int c = 0; c < a.npad; c += 16) {
                    // y = A_hi x_hi + A_hi x_lo + A_lo x_hi, added in that order
                    const uint32_t tb = tmem + ((uint32_t)(32 * q) << 16) + TC_TACC + (uint32_t)ab * 128u + (uint32_t)c;
                    float v[16], w[16];
                    tmem_ld16(tb, v);
                    tmem_ld16(tb + n, w);
#pragma unroll
                    for (int qq = 0; qq < 16; ++qq) v[qq] += w[qq];
                    if constexpr (!EXACT) {
                        tmem_ld16(tb + 2u * n, w);
#pragma unroll
                        for (int qq = 0; qq < 16; ++qq) v[qq] += w[qq];
                    }
                    if (r < a.rows)
#pragma unroll
                        for (int qq = 0; qq < 16; ++qq) {
                            const int t = c + qq;
                            if (t < a.nt) {
                                if (a.splits == 1) {
                                    float *o = a.y + (size_t)t * a.ys + r;
                                    *o = a.acc ? __fadd_rn(*o, v[qq]) : v[qq];
                                } else {
                                    a.part[((size_t)split * TC_NMAX + t) * a.rows + r] = v[qq];
                                }
                            }
                        }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) tc_arrive(&accfree[ab]);
        }
        if (a.splits > 1) __threadfence();  // this split's partials, before the tile's ticket below
    } else if (warp == W_MMA) {
        // ---- MMAs: step j reads A buffer j & 1 and B buffer j & 1 into tile k's accumulator k & 1
        if (lane == 0) {
            // one MMA A_hi [x_hi | x_lo] (N = 2 npad) and one A_lo x_hi (N = npad, the operand's first npad rows) per
            // 16-deep step: few, wide MMAs (an MMA's issue costs about the same at N = 32 as at N = 64)
            const uint32_t id2 = umma_idesc_bf16(TC_M, 2 * a.npad), id1 = umma_idesc_bf16(TC_M, a.npad);
            const uint32_t bbase = smem_u32(Bs);
            const uint64_t binc = (2u * 2u * n * 16u) >> 4;  // a 16-deep step: two core-matrix columns of 2 N rows
            for (int j = 0; j < NS; ++j) {
                const int b = j & 1, k = j / sps, js = j - k * sps;
                if (!wt(&aready[b], (uint32_t)(j >> 1) & 1u) || !wt(&bready[b], (uint32_t)(j >> 1) & 1u)) break;
                if (js == 0 && k >= 2 && !wt(&accfree[k & 1], (uint32_t)((k >> 1) - 1) & 1u)) break;
                tc_fence_after();
                const uint32_t d1 = tmem + TC_TACC + (uint32_t)(k & 1) * 128u, d2 = d1 + 2u * n;
                const uint32_t ah = tmem + TC_TA + (uint32_t)b * 128u, al = ah + 64u;
                uint64_t db = umma_desc(bbase + (uint32_t)b * TC_B_BUF, 2u * n * 16u, 128u);
#pragma unroll
                for (int ks = 0; ks < TC_KC / 16; ++ks) {
                    const uint32_t acc = (js > 0 || ks > 0) ? 1u : 0u;
                    umma_bf16_tmem_a(d1, ah + 8u * ks, db, id2, acc);
                    if constexpr (!EXACT) umma_bf16_tmem_a(d2, al + 8u * ks, db, id1, acc);
                    db += binc;
                }
                umma_commit(&afree[b]);
                umma_commit(&bfree[b]);
                if (js == sps - 1) umma_commit(&accdone[k & 1]);
                n_mma = j + 1;
            }
        }
    }

    // ---- wind down: what this CTA issued completes before its shared and tensor memory are released
    if (s_fail) {
        if (warp == W_COPY && lane == 0) {
            dev_fail(a.err, DEV_WAIT_TIMEOUT);
            for (int k = max(0, n_raw - a.rs); k < n_raw; ++k) mbar_wait(&rfull[k % a.rs], (uint32_t)(k / a.rs) & 1u, 1u << 16);
        }
        if (warp == W_XCOPY && lane == 0)
            for (int k = max(0, n_x - TC_XS); k < n_x; ++k) mbar_wait(&xfull[k % TC_XS], (uint32_t)(k / TC_XS) & 1u, 1u << 16);
        if (warp == W_MMA && lane == 0 && n_mma > 0) {  // the last commit covers every MMA issued before it
            const int j = n_mma - 1;
            mbar_wait(&afree[j & 1], (uint32_t)(j >> 1) & 1u, 1u << 16);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TC_TMEM_COLS) : "memory");
    }
    if (a.splits == 1) return;
    // ---- split K (one tile per CTA): the tile's last CTA adds the partials in split order (release / acquire
    // ticket); every thread takes up to 5 of the tile's 128 x 32 outputs and has all of their splits' loads in flight
    if (tid == 0) {
        uint32_t tk;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(tk) : "l"(a.tickets + t0) : "memory");
        s_last = tk == (uint32_t)a.splits - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    constexpr int PER = (TC_M * TC_NMAX + TC_THREADS - 1) / TC_THREADS, SPL = 8;
    float v[PER][SPL];
#pragma unroll
    for (int m = 0; m < PER; ++m) {
        const int o = tid + TC_THREADS * m, t = o / TC_M, r = t0 * TC_M + (o % TC_M);
        const bool live = o < TC_M * TC_NMAX && t < a.nt && r < a.rows;
#pragma unroll
        for (int p = 0; p < SPL; ++p)
            v[m][p] = live && p < a.splits ? __ldcg(a.part + ((size_t)p * TC_NMAX + t) * a.rows + r) : 0.0f;
    }
#pragma unroll
    for (int m = 0; m < PER; ++m) {
        const int o = tid + TC_THREADS * m, t = o / TC_M, r = t0 * TC_M + (o % TC_M);
        if (o < TC_M * TC_NMAX && t < a.nt && r < a.rows && !s_fail) {
            float sum = 0.0f;
#pragma unroll
            for (int p = 0; p < SPL; ++p)
                if (p < a.splits) sum += v[m][p];
            float *dst = a.y + (size_t)t * a.ys + r;
            *dst = a.acc ? __fadd_rn(*dst, sum) : sum;
        }
    }
    if (tid == 0) a.tickets[t0] = 0u;
}

// ---- resident weights for the tensor-core path: padded raw chunks, plus the split-K scratch -------------------------

struct TcH {
    uint32_t type = 0;
    int rows = 0, cols = 0, dev = 0, tiles = 0, nr = 0, spr = 1, splits = 1, nr_split = 1, rs = 2, grid = 1;
    uint32_t wbytes = 0, cb = 0;  // padded / GGUF bytes of a raw chunk of a row
    size_t smem = 0;
    uint64_t rb = 0;
    DevBuf W, part, tickets;
};
static std::vector<TcH *> g_tc;
static std::mutex g_tc_mu;

static TcH *tc_get(int h) {
    std::lock_guard<std::mutex> l(g_tc_mu);
    return h >= 1 && h <= (int)g_tc.size() ? g_tc[h - 1] : nullptr;
}

// raw chunk width: 256 columns where its bytes fit a 240-byte box (a K-quant block, eight 32-value blocks), else 128
static int tc_plan(TcH &w) {
    int qk = 0, tb = 0;
    type_info(w.type, qk, tb);
    auto bytes = [&](int c) { return (uint64_t)(c / qk) * (uint64_t)tb; };
    int rc = 0;
    if (w.cols % 256 == 0 && 256 % qk == 0 && bytes(256) <= 240) rc = 256;
    else if (w.cols % 128 == 0 && 128 % qk == 0 && bytes(128) <= 256) rc = 128;
    if (!rc) return fail("tc: unsupported type or shape (cols a multiple of 128, 256 for 256-value blocks)");
    w.spr = rc / TC_KC;
    w.nr = w.cols / rc;
    w.cb = (uint32_t)bytes(rc);
    w.wbytes = (uint32_t)tc_align(w.cb, 16);
    const size_t slot = (size_t)TC_M * w.wbytes;
    w.rs = (int)std::min<size_t>(TC_RS_MAX, (TC_SMEM_MAX - TC_RAW_OFF) / slot);
    if (w.rs < 2) return fail("tc: rows too wide for the raw chunk ring");
    w.smem = TC_RAW_OFF + (size_t)w.rs * slot;
    w.tiles = (w.rows + TC_M - 1) / TC_M;
    const int nsm = num_sms();
    if (w.tiles < nsm) {  // fewer tiles than SMs: split K (at most 8 partials per row)
        w.splits = std::max(1, std::min(std::min(8, nsm / w.tiles), w.nr));
        w.nr_split = (w.nr + w.splits - 1) / w.splits;
        w.splits = (w.nr + w.nr_split - 1) / w.nr_split;  // no empty split
    } else {
        w.splits = 1;
        w.nr_split = w.nr;
    }
    w.grid = w.splits > 1 ? w.tiles * w.splits : std::min(w.tiles, nsm);
    return 0;
}

int launch_tc_gemv(const TcH &w, const float *x, int xs, float *y, int ys, int nt, cudaStream_t s, bool acc = false) {
    if (nt < 1 || nt > TC_NMAX) return fail("tc gemv: nt out of range (1..32)");
    if (((uintptr_t)x & 15) || (xs & 3)) return fail("tc gemv: x must be 16-byte aligned, xs % 4 == 0");
    TcArgs a;
    a.W = w.W.as<uint8_t>();
    a.rows = w.rows;
    a.nt = nt;
    a.npad = nt <= 16 ? 16 : 32;
    a.x = x;
    a.xs = xs;
    a.y = y;
    a.ys = ys;
    a.acc = acc ? 1 : 0;
    a.tiles = w.tiles;
    a.nr = w.nr;
    a.spr = w.spr;
    a.splits = w.splits;
    a.nr_split = w.nr_split;
    a.rs = w.rs;
    a.wbytes = w.wbytes;
    a.part = w.part.as<float>();
    a.tickets = w.tickets.as<uint32_t>();
    a.err = dev_error_ptr();
    cudaError_t e = cudaSuccess;
    const bool known = dispatch_type(w.type, [&]<uint32_t TY>() {
        e = allow_max_dynamic_smem(k_tc_gemv<TY>);
        if (e == cudaSuccess) e = launch_k(k_tc_gemv<TY>, dim3(w.grid), dim3(TC_THREADS), w.smem, s, a);
    });
    if (!known) return fail("tc gemv: unsupported type");
    if (e != cudaSuccess) return fail(std::string("tc gemv launch: ") + cudaGetErrorString(e));
    return 0;
}

static TcH *tc_build(uint32_t type, const uint8_t *Wh, int rows, int cols) {
    const uint64_t rb = row_bytes(type, cols);
    if (!rb || rows < 1 || cols < TC_KC || cols % TC_KC) {
        fail("tc: unsupported type or shape (cols a multiple of 128)");
        return nullptr;
    }
    TcH *w = new TcH();
    w->type = type;
    w->rows = rows;
    w->cols = cols;
    w->rb = rb;
    cudaGetDevice(&w->dev);
    if (tc_plan(*w)) {
        delete w;
        return nullptr;
    }
    // tile-major padded raw chunks: chunk c of tile T holds its 128 rows' GGUF bytes of columns [c rc, (c + 1) rc) at
    // a row stride of wbytes (zeros after each row's bytes and for rows past the matrix), at (T nr + c) 128 wbytes, so
    // a chunk is one contiguous bulk copy
    const size_t chunk = (size_t)TC_M * w->wbytes, total = (size_t)w->tiles * w->nr * chunk;
    std::vector<uint8_t> host(total, 0);
    for (int r = 0; r < rows; ++r) {
        const int T = r / TC_M, rr = r % TC_M;
        for (int c = 0; c < w->nr; ++c)
            std::memcpy(host.data() + ((size_t)T * w->nr + c) * chunk + (size_t)rr * w->wbytes, Wh + (size_t)r * rb + (size_t)c * w->cb,
                        w->cb);
    }
    bool ok = cudaMalloc(&w->W.p, total) == cudaSuccess &&
              cudaMemcpy(w->W.p, host.data(), total, cudaMemcpyHostToDevice) == cudaSuccess;
    ok = ok && cudaMalloc(&w->part.p, (size_t)w->splits * TC_NMAX * rows * 4) == cudaSuccess &&
         cudaMalloc(&w->tickets.p, (size_t)w->tiles * 4) == cudaSuccess &&
         cudaMemset(w->tickets.p, 0, (size_t)w->tiles * 4) == cudaSuccess;
    if (!ok) {
        delete w;
        fail("tc: device allocation / copy failed");
        return nullptr;
    }
    return w;
}

}  // namespace fn

using namespace fn;

// ---- C ABI --------------------------------------------------------------------------------------------------------

// Resident weights for the tensor-core batched path on the current device: GGUF rows Wh [rows][row_bytes(type, cols)]
// (any of the 19 formats; cols a multiple of 128). Returns a handle >= 1 or -1. Counterpart of fn_w_create for
// batches of 1..32 tokens.
FN_API int fn_tc_create(uint32_t type, const uint8_t *Wh, int rows, int cols) {
    TcH *w = tc_build(type, Wh, rows, cols);
    if (!w) return -1;
    std::lock_guard<std::mutex> l(g_tc_mu);
    g_tc.push_back(w);
    return (int)g_tc.size();
}

FN_API int fn_tc_free(int h) {
    TcH *w = tc_get(h);
    if (!w) return fail("fn_tc_free: bad handle");
    delete w;
    std::lock_guard<std::mutex> l(g_tc_mu);
    g_tc[h - 1] = nullptr;
    return 0;
}

// y[t][r] (+)= W[r] . x[t] for t < nt <= 32 on a stream (device pointers; token strides xs, ys in floats; x 16-byte
// aligned; flags bit 0 adds into y). One call at a time per handle (the split-K scratch belongs to the handle). The
// batched-decode form of gemv() (engine/faie2fn.cu:2250-2281) on the tensor cores; within 1e-4 of float64 relative to
// max |y|.
FN_API int fn_tc_gemv(int h, const float *x, int xs, float *y, int ys, int nt, int flags, void *stream) {
    TcH *w = tc_get(h);
    if (!w) return fail("fn_tc_gemv: bad handle");
    return launch_tc_gemv(*w, x, xs, y, ys, nt, (cudaStream_t)stream, (flags & 1) != 0);
}

// The same on host buffers (synchronous), the tensor-core counterpart of fn_test_gemv: W GGUF rows, x [nt][cols],
// y [nt][rows], nt <= 32.
FN_API int fn_test_tc_gemv(uint32_t type, const uint8_t *Wh, int rows, int cols, const float *xh, int nt, float *yh) {
    if (nt < 1 || nt > TC_NMAX) return fail("nt out of range (1..32)");
    FN_CK(cudaSetDevice(hook_device()));
    TcH *w = tc_build(type, Wh, rows, cols);
    if (!w) return -1;
    cudaStream_t s = hook_stream();
    DevBuf x, y;
    int rc = 0;
    if (cudaMalloc(&x.p, (size_t)nt * cols * 4) != cudaSuccess || cudaMalloc(&y.p, (size_t)nt * rows * 4) != cudaSuccess ||
        cudaMemcpyAsync(x.p, xh, (size_t)nt * cols * 4, cudaMemcpyHostToDevice, s) != cudaSuccess)
        rc = fail("fn_test_tc_gemv: allocation / copy failed");
    if (!rc) rc = launch_tc_gemv(*w, x.as<float>(), cols, y.as<float>(), rows, nt, s);
    if (!rc && (cudaMemcpyAsync(yh, y.p, (size_t)nt * rows * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
                cudaStreamSynchronize(s) != cudaSuccess))
        rc = fail("fn_test_tc_gemv: copy out failed");
    delete w;
    if (rc) return rc;
    return check_dev_error("fn_test_tc_gemv");
}

// Device time of one call (CUDA events over `iters` back-to-back calls in a CUDA graph, after a warm-up replay) on
// hash-random weights of a format, tokens nt; the weights of consecutive calls alternate between copies whose total
// exceeds twice the L2, so every call streams its weights from HBM (as fn_bench_gemv).
FN_API int fn_bench_tc_gemv(uint32_t type, int rows, int cols, int nt, int iters, float *ms) {
    if (nt < 1 || nt > TC_NMAX || iters < 1) return fail("nt/iters out of range");
    FN_CK(cudaSetDevice(hook_device()));
    const uint64_t rb = row_bytes(type, cols);
    if (!rb || cols % TC_KC) return fail("unsupported type/shape");
    int dev = 0, l2 = 0;
    FN_CK(cudaGetDevice(&dev));
    FN_CK(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev));
    const size_t wbytes = (size_t)tc_align(rb, 16) * rows;
    const int copies = (int)std::max<size_t>(2, (2 * (size_t)l2 + wbytes - 1) / wbytes + 1);
    std::vector<uint8_t> host(rb * (size_t)rows);
    uint32_t st = 0x9E3779B9u ^ type ^ (uint32_t)rows;
    for (auto &b : host) {  // xorshift bytes; the fp16 scale fields stay finite through the decoders' use of them
        st ^= st << 13;
        st ^= st >> 17;
        st ^= st << 5;
        b = (uint8_t)(st & 0x3B);
    }
    std::vector<TcH *> ws;
    for (int i = 0; i < copies; ++i) {
        TcH *w = tc_build(type, host.data(), rows, cols);
        if (!w) {
            for (TcH *q : ws) delete q;
            return -1;
        }
        ws.push_back(w);
    }
    cudaStream_t s = hook_stream();
    DevBuf x, y;
    int rc = 0;
    if (cudaMalloc(&x.p, (size_t)nt * cols * 4) != cudaSuccess || cudaMalloc(&y.p, (size_t)nt * rows * 4) != cudaSuccess ||
        cudaMemsetAsync(x.p, 0, (size_t)nt * cols * 4, s) != cudaSuccess)
        rc = fail("fn_bench_tc_gemv: allocation failed");
    for (int i = 0; !rc && i < copies; ++i) rc = launch_tc_gemv(*ws[i], x.as<float>(), cols, y.as<float>(), rows, nt, s);
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    if (!rc && cudaStreamSynchronize(s) == cudaSuccess &&
        cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
        for (int i = 0; !rc && i < iters; ++i)
            rc = launch_tc_gemv(*ws[i % copies], x.as<float>(), cols, y.as<float>(), rows, nt, s);
        if (cudaStreamEndCapture(s, &g) != cudaSuccess || rc) rc = rc ? rc : fail("fn_bench_tc_gemv: capture failed");
    } else if (!rc) {
        rc = fail("fn_bench_tc_gemv: capture failed");
    }
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (!rc && (cudaGraphInstantiate(&ge, g, 0) != cudaSuccess || cudaGraphLaunch(ge, s) != cudaSuccess ||
                cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess ||
                cudaEventRecord(e0, s) != cudaSuccess || cudaGraphLaunch(ge, s) != cudaSuccess ||
                cudaEventRecord(e1, s) != cudaSuccess || cudaEventSynchronize(e1) != cudaSuccess))
        rc = fail("fn_bench_tc_gemv: timing failed");
    float t = 0.0f;
    if (!rc) {
        cudaEventElapsedTime(&t, e0, e1);
        *ms = t / (float)iters;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    for (TcH *q : ws) delete q;
    if (rc) return rc;
    return check_dev_error("fn_bench_tc_gemv");
}
