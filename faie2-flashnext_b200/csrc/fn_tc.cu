// Batched decode GEMV on the 5th-generation tensor cores (tcgen05): y[t][r] = W[r] . x[t] for t < nt <= 32 tokens.
//
// At batch 8..32 the quantised GEMV becomes a dense contraction (rows x cols x nt), so this path dequantises each
// weight tile once into shared memory and lets tcgen05.mma multiply it by all tokens at once, where the CUDA-core GEMV
// would repeat the FMA work per token (its batched form, k_gemv<.., NT = 8, ..>, runs 8 tokens per call). The
// reference has no batched path (its k_tgemv takes nt <= 8 on CUDA cores, engine/faie2fn.cu:734-955); the operator
// contract is the same as fn_w_gemv's.
//
// Precision: the tensor cores take bf16 operands, so every weight value v (the exact GGUF dequantisation, load_group) and
// every x value is split into v_hi = bf16(v) and v_lo = bf16(v - v_hi), and each 16-deep step runs three MMAs,
// hi*hi + hi*lo + lo*hi, accumulated in fp32 in tensor memory: each product keeps about 16 mantissa bits (the lo*lo
// term is below 2^-16 of it), so y is within about 3e-5 of float64, relative to max |y| (the stated tolerance is 1e-4).
//
// Layout and schedule, per CTA (256 threads; one 128-row tile of W and a K range of its columns; CTAs split K when
// there are fewer tiles than SMs, the last CTA of a tile adding the partials in split order, so y is deterministic):
//   * K is walked in chunks of 128 columns, two chunk buffers in shared memory. For a chunk, warps decode the tile's
//     128 x 128 values (one lane per row and 32-value group, stored as whole 16-byte core-matrix rows, so the 8 lanes
//     of a store phase fill one core matrix) into A_hi / A_lo and
//     stage x's N x 128 values into B_hi / B_lo, all in the tensor cores' canonical K-major layout without swizzle:
//     8-row x 16-byte core matrices, the 8-row groups 128 bytes apart (SBO), the 8-column groups a whole M (or N)
//     extent apart (LBO).
//   * one thread issues the chunk's 8 x 3 MMAs (M = 128, N = 16 or 32, K = 16 each) and commits them to the buffer's
//     mbarrier; the warps then decode the next chunk into the other buffer while the tensor cores work, and wait for a
//     buffer's commit before they overwrite it.
//   * the accumulator (128 lanes x N fp32 columns of tensor memory) is read by warps 0-3 (lane 32w + l = row
//     32w + l) with tcgen05.ld and stored to y (or to the split's partial).
// Every wait is bounded: a wait that runs out records DEV_WAIT_TIMEOUT, the CTA still waits (bounded) for the MMAs it
// issued, frees its tensor memory and returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>
#include <vector>

#include "fn_engine.h"
#include "fn_rowdot.cuh"

namespace fn {

constexpr int TC_M = 128;       // rows per tile (one MMA's M)
constexpr int TC_KC = 128;      // columns per chunk
constexpr int TC_THREADS = 512;
constexpr int TC_NMAX = 32;     // tokens per call
constexpr int TC_TMEM_COLS = 32;

static size_t tc_align(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct TcArgs {
    CUtensorMap tmap;  // W as a 2-D byte array [rows][ldw]; box: 128 rows x raw_stride bytes
    const uint8_t *W;  // GGUF rows at stride ldw
    uint32_t ldw;
    int rows, cols;
    const float *x;
    int xs;
    float *y;
    int ys, nt, npad;  // npad: the MMA's N (16 or 32)
    int acc;           // 1: y += W x (the residual add of a projection)
    int chunks_per_split, splits;
    float *part;        // [splits][32][rows] when splits > 1
    uint32_t *tickets;  // [tiles], zero between launches
    uint32_t raw_stride;  // bytes per row of a raw chunk slot (16-byte multiple): the TMA box width
    uint32_t *err;
};

// shared memory (bytes): per buffer A_hi, A_lo [16 k-cores][16 m-groups][128 B], B_hi, B_lo [16 k-cores][N/8][128 B]
constexpr uint32_t TC_A_BYTES = TC_M * TC_KC * 2;        // 32 KiB
constexpr uint32_t TC_B_BYTES = TC_NMAX * TC_KC * 2;     // 8 KiB at N = 32
constexpr uint32_t TC_BUF_BYTES = 2 * TC_A_BYTES + 2 * TC_B_BYTES;
constexpr uint32_t TC_BARS = 2 * TC_BUF_BYTES;           // 4 mbarriers: MMA done per buffer, raw chunk landed per slot
constexpr uint32_t TC_RAW = TC_BARS + 128;              // two raw chunk slots of 128 rows x raw_stride
constexpr size_t TC_SMEM_MAX = 227 * 1024 - 1024;       // less the static shared memory

// bytes [start, end) of a row that chunk c (columns 128 c .. 128 c + 127) decodes from: whole blocks, widened to
// 16-byte boundaries for the bulk copy (the row stride is a 16-byte multiple, so end <= the stride)
__host__ __device__ inline void tc_chunk_bytes(int c, int qk, int tb, uint32_t &start, uint32_t &end) {
    const uint32_t b0 = (uint32_t)(c * TC_KC / qk), b1 = (uint32_t)(((c + 1) * TC_KC + qk - 1) / qk);
    start = (b0 * (uint32_t)tb) & ~15u;
    end = (b1 * (uint32_t)tb + 15u) & ~15u;
}

// sm_100 shared-memory matrix descriptor: start address, leading / stride byte offsets (>> 4), version 1, no swizzle
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
           (1ull << 46);
}
// instruction descriptor of kind::f16: fp32 accumulator, bf16 A and B, both K-major, N >> 3 and M >> 4
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void umma_bf16(uint32_t dtmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(dtmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void async_proxy_fence() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

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

// the bf16 pair (hi, lo) of 4 values as two 8-byte words
__device__ __forceinline__ void split4(float a, float b, float c, float d, uint2 &hi, uint2 &lo) {
    const __nv_bfloat162 h01 = __floats2bfloat162_rn(a, b), h23 = __floats2bfloat162_rn(c, d);
    const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
    const __nv_bfloat162 l01 = __floats2bfloat162_rn(a - f01.x, b - f01.y), l23 = __floats2bfloat162_rn(c - f23.x, d - f23.y);
    hi = make_uint2(*(const uint32_t *)&h01, *(const uint32_t *)&h23);
    lo = make_uint2(*(const uint32_t *)&l01, *(const uint32_t *)&l23);
}

// One 32-value group of a staged raw row, as load_group (the same values, bit for bit). Q4_K blocks sit 16-byte
// aligned in a row, so their header and quants are read with four 16-byte shared-memory loads; the other formats go
// through load_group.
template <uint32_t TY> __device__ __forceinline__ auto tc_load(const uint8_t *row, int g, const uint32_t *grid) {
    if constexpr (TY == T_Q4_K) {
        const uint8_t *blk = row + (g >> 3) * 144;
        const int s = g & 7;
        const uint4 h = *(const uint4 *)blk;  // d, dmin | the 12 packed scale and min bytes
        uint32_t sc, mn;
        kq_scale_min(s, h.y, h.z, h.w, sc, mn);
        Codes32 c;
        c.a[0] = c.a[1] = __fmul_rn(f16_of(h.x, 0), __uint2float_rn(sc));
        c.b[0] = c.b[1] = -__fmul_rn(f16_of(h.x, 1), __uint2float_rn(mn));
        const uint4 q0 = *(const uint4 *)(blk + 16 + 32 * (s >> 1)), q1 = *(const uint4 *)(blk + 32 + 32 * (s >> 1));
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const int sh = 4 * (s & 1);
#pragma unroll
        for (int i = 0; i < 8; ++i) c.q[i] = (qw[i] >> sh) & LOW4;
        return c;
    } else {
        return load_group<TY>(row, g, grid);
    }
}

template <uint32_t TY>
__global__ void __launch_bounds__(TC_THREADS, 1) k_tc_gemv(const __grid_constant__ TcArgs a) {
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail, s_last;
    uint64_t *mbars = (uint64_t *)(sm + TC_BARS);      // [2]: the MMAs reading buffer b are complete
    uint64_t *rbars = mbars + 2;                       // [2]: raw chunk slot s has landed
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x, split = blockIdx.y, row0 = tile * TC_M;
    const int nchunks = a.cols / TC_KC;
    const int c0 = split * a.chunks_per_split, c1 = min(nchunks, c0 + a.chunks_per_split);
    const int nrow = min(TC_M, a.rows - row0);
    const uint32_t n = (uint32_t)a.npad, bbytes = n * TC_KC * 2;  // B bytes per hi / lo
    const uint32_t idesc = umma_idesc_bf16(TC_M, a.npad);
    const uint32_t *grid = dev_grid<TY>();
    constexpr int QK = Gguf<TY>::qk, TB = Gguf<TY>::bytes;

    // the raw bytes of chunk c of the tile's rows into slot sl: one 2-D tensor copy of the box (128 rows x raw_stride
    // bytes from byte column st, a 16-byte multiple; rows past the matrix and bytes past the stride read as zero)
    auto issue_raw = [&](int c, int sl) {
        if (tid != 0) return;
        uint32_t st, en;
        tc_chunk_bytes(c, QK, TB, st, en);
        uint64_t *bar = &rbars[sl];
        mbar_arrive_tx(bar, (uint32_t)TC_M * a.raw_stride);
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
            ::"r"(smem_u32(sm + TC_RAW + (size_t)sl * TC_M * a.raw_stride)), "l"(&a.tmap), "r"((int)st), "r"(row0),
            "r"(smem_u32(bar))
            : "memory");
    };

    if (tid == 0) {
        for (int q = 0; q < 4; ++q) mbar_init(&mbars[q], 1);
        mbar_fence_init();
        s_fail = 0;
    }
    if (warp == 0) {  // tensor memory: TC_TMEM_COLS fp32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&s_tmem)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    // the weights are read-only: the first two chunks' copies fly before the wait for the previous kernel
    if (c0 < c1) issue_raw(c0, 0);
    if (c0 + 1 < c1) issue_raw(c0 + 1, 1);

    pdl_wait();
    pdl_trigger();
    const float *x = after_wait(a.x);
    // x: one (token, 8-column group) item per thread (n * 16 <= 512 items); the next chunk's values are loaded into
    // registers while this chunk is decoded
    const int xt = tid % (int)n, xkc = tid / (int)n;
    const bool xitem = tid < (int)n * (TC_KC / 8), xlive = xitem && xt < a.nt;
    auto load_x = [&](int c, float4 &p, float4 &q) {
        if (xlive) {
            const float4 *src = (const float4 *)(x + (size_t)xt * a.xs + c * TC_KC + xkc * 8);
            p = src[0];
            q = src[1];
        }
    };
    float4 xp = make_float4(0.f, 0.f, 0.f, 0.f), xq = xp, np_ = xp, nq_ = xp;
    if (c0 < c1) load_x(c0, xp, xq);

    int issued = 0;  // chunks whose MMAs were issued (the commit of chunk i arrives on mbars[i & 1])
    for (int c = c0; c < c1; ++c) {
        const int i = c - c0, b = i & 1;
        uint8_t *buf = sm + b * TC_BUF_BYTES;
        uint8_t *Ahi = buf, *Alo = buf + TC_A_BYTES, *Bhi = buf + 2 * TC_A_BYTES, *Blo = Bhi + bbytes;
        // the slot of chunk i + 1 held chunk i - 1, decoded before the barrier that ended that chunk's staging
        if (i >= 1 && c + 1 < c1) issue_raw(c + 1, (i + 1) & 1);
        bool ok = mbar_wait(&rbars[i & 1], (uint32_t)(i >> 1) & 1u);
        if (i >= 2) ok = ok && mbar_wait(&mbars[b], (uint32_t)((i - 2) >> 1) & 1u);  // chunk i - 2 read this buffer
        if (!ok) s_fail = 1;
        __syncthreads();
        if (s_fail) break;
        if (c + 1 < c1) load_x(c + 1, np_, nq_);
        // weights: one (row, group of 32) per thread, a warp on 32 consecutive rows, decoded from the raw slot (the
        // row pointer is shifted so that the decoder's block offsets of this chunk land in the slot)
        uint32_t st, en;
        tc_chunk_bytes(c, QK, TB, st, en);
        const uint8_t *raw = sm + TC_RAW + (size_t)(i & 1) * TC_M * a.raw_stride;
        for (int it = tid; it < TC_M * (TC_KC / 32); it += TC_THREADS) {
            const int r = it & (TC_M - 1), gl = it >> 7;
            const uint32_t roff = (uint32_t)(r >> 3) * 128u + (uint32_t)(r & 7) * 16u;
            if (r < nrow) {
                const uint8_t *rp = raw + (size_t)r * a.raw_stride - st;
                // the group's values as four 16-byte core-matrix rows each of hi and lo: the 8 lanes of a store
                // phase write one core matrix's 128 contiguous bytes (no bank conflict)
                const auto G = tc_load<TY>(rp, c * (TC_KC / 32) + gl, grid);
#pragma unroll
                for (int kc = 0; kc < 4; ++kc) {
                    uint2 h0, l0, h1, l1;
                    const float4 p = G.quad(8 * kc), q = G.quad(8 * kc + 4);
                    split4(p.x, p.y, p.z, p.w, h0, l0);
                    split4(q.x, q.y, q.z, q.w, h1, l1);
                    const uint32_t off = (uint32_t)(gl * 4 + kc) * (TC_M * 16u) + roff;
                    *(uint4 *)(Ahi + off) = make_uint4(h0.x, h0.y, h1.x, h1.y);
                    *(uint4 *)(Alo + off) = make_uint4(l0.x, l0.y, l1.x, l1.y);
                }
            } else {
#pragma unroll
                for (int kc = 0; kc < 4; ++kc) {
                    const uint32_t off = (uint32_t)(gl * 4 + kc) * (TC_M * 16u) + roff;
                    *(uint4 *)(Ahi + off) = make_uint4(0, 0, 0, 0);
                    *(uint4 *)(Alo + off) = make_uint4(0, 0, 0, 0);
                }
            }
        }
        // x: this thread's (token, 8-column group); tokens >= nt are zero
        if (xitem) {
            const uint32_t off = (uint32_t)xkc * (n * 16u) + (uint32_t)(xt >> 3) * 128u + (uint32_t)(xt & 7) * 16u;
            uint2 h0, l0, h1, l1;
            split4(xp.x, xp.y, xp.z, xp.w, h0, l0);
            split4(xq.x, xq.y, xq.z, xq.w, h1, l1);
            *(uint4 *)(Bhi + off) = make_uint4(h0.x, h0.y, h1.x, h1.y);
            *(uint4 *)(Blo + off) = make_uint4(l0.x, l0.y, l1.x, l1.y);
        }
        xp = np_;
        xq = nq_;
        async_proxy_fence();  // the generic-proxy stores (and reads of the raw slot) ordered before async-proxy use
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            // descriptors of step 0; a 16-deep step moves the start address by two core-matrix columns (the address
            // field is address >> 4 in the low 14 bits, and shared addresses stay below 2^18, so adding cannot carry)
            uint64_t dah = umma_desc(smem_u32(Ahi), TC_M * 16u, 128u), dal = umma_desc(smem_u32(Alo), TC_M * 16u, 128u);
            uint64_t dbh = umma_desc(smem_u32(Bhi), n * 16u, 128u), dbl = umma_desc(smem_u32(Blo), n * 16u, 128u);
            const uint64_t ainc = 2u * TC_M * 16u >> 4, binc = 2u * n * 16u >> 4;
#pragma unroll
            for (int j = 0; j < TC_KC / 16; ++j) {  // 16-deep steps: two 8-column core matrices each
                umma_bf16(tmem, dah, dbh, idesc, (i > 0 || j > 0) ? 1u : 0u);
                umma_bf16(tmem, dah, dbl, idesc, 1u);
                umma_bf16(tmem, dal, dbh, idesc, 1u);
                dah += ainc;
                dal += ainc;
                dbh += binc;
                dbl += binc;
            }
            umma_commit(&mbars[b]);
        }
        ++issued;
    }
    // the last commit covers every MMA this CTA issued; raw copies still in flight (a wait ran out) land first
    if (issued > 0) {
        const int i = issued - 1;
        if (!mbar_wait(&mbars[i & 1], (uint32_t)(i >> 1) & 1u) && tid == 0) s_fail = 1;
    }
    if (s_fail && tid == 0) {
        const int n_issued_raw = min(c1 - c0, issued + 2);
        for (int q = issued; q < n_issued_raw; ++q) mbar_wait(&rbars[q & 1], (uint32_t)(q >> 1) & 1u, 1u << 16);
    }
    tc_fence_after();
    __syncthreads();
    const bool ok = !s_fail && issued > 0;
    if (ok && warp < 4) {  // accumulator rows 32 w + lane -> y or this split's partial
        const int r = row0 + warp * 32 + lane;
        for (int c = 0; c < a.npad; c += 16) {
            float v[16];
            tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v);
            if (r < a.rows)
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    const int t = c + q;
                    if (t < a.nt) {
                        if (a.splits == 1) {
                            float *o = a.y + (size_t)t * a.ys + r;
                            *o = a.acc ? __fadd_rn(*o, v[q]) : v[q];
                        }
                        else a.part[((size_t)split * TC_NMAX + t) * a.rows + r] = v[q];
                    }
                }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TC_TMEM_COLS) : "memory");
    }
    if (!ok) {
        if (tid == 0 && s_fail) dev_fail(a.err, DEV_WAIT_TIMEOUT);
        return;
    }
    if (a.splits == 1) return;
    // split K: the tile's last CTA adds the partials in split order (release / acquire ticket)
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        uint32_t tk;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(tk) : "l"(a.tickets + tile) : "memory");
        s_last = tk == (uint32_t)a.splits - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // each thread's outputs (token t = it / 128, row it % 128; up to 8 of them): the splits added in order, one split's
    // loads of all its outputs in flight at once
    constexpr int PER = TC_NMAX * TC_M / TC_THREADS;
    float sum[PER];
#pragma unroll
    for (int m = 0; m < PER; ++m) sum[m] = 0.0f;
    for (int q = 0; q < a.splits; ++q) {
        float v[PER];
#pragma unroll
        for (int m = 0; m < PER; ++m) {
            const int it = tid + m * TC_THREADS, t = it / TC_M, r = row0 + (it % TC_M);
            v[m] = t < a.nt && r < a.rows ? __ldcg(a.part + ((size_t)q * TC_NMAX + t) * a.rows + r) : 0.0f;
        }
#pragma unroll
        for (int m = 0; m < PER; ++m) sum[m] += v[m];
    }
#pragma unroll
    for (int m = 0; m < PER; ++m) {
        const int it = tid + m * TC_THREADS, t = it / TC_M, r = row0 + (it % TC_M);
        if (t < a.nt && r < a.rows) {
            float *o = a.y + (size_t)t * a.ys + r;
            *o = a.acc ? __fadd_rn(*o, sum[m]) : sum[m];
        }
    }
    if (tid == 0) a.tickets[tile] = 0u;
}

// ---- resident weights for the tensor-core path: GGUF rows at a 16-byte stride, plus the split-K scratch --------------

struct TcH {
    CUtensorMap tmap;
    uint32_t type = 0;
    int rows = 0, cols = 0, dev = 0, splits = 1, chunks_per_split = 1;
    uint32_t raw_stride = 0;
    size_t smem = 0;
    uint64_t rb = 0;
    uint32_t ldw = 0;
    DevBuf W, part, tickets;
};
static std::vector<TcH *> g_tc;
static std::mutex g_tc_mu;

static TcH *tc_get(int h) {
    std::lock_guard<std::mutex> l(g_tc_mu);
    return h >= 1 && h <= (int)g_tc.size() ? g_tc[h - 1] : nullptr;
}

static int tc_plan(TcH &w) {
    const int tiles = (w.rows + TC_M - 1) / TC_M, nchunks = w.cols / TC_KC;
    int qk = 0, tb = 0;
    type_info(w.type, qk, tb);
    uint32_t mx = 0;
    for (int c = 0; c < nchunks; ++c) {
        uint32_t st, en;
        tc_chunk_bytes(c, qk, tb, st, en);
        mx = std::max(mx, en - st);
    }
    // the TMA box is one raw chunk of every row: an odd number of 16-byte units keeps a warp's 16-byte reads of its 32
    // rows free of bank conflicts where that fits; a box row is at most 256 bytes
    w.raw_stride = mx + ((mx / 16) % 2 == 0 && mx + 16 <= 256 && (size_t)TC_RAW + 2ull * TC_M * (mx + 16) <= TC_SMEM_MAX
                             ? 16 : 0);
    w.smem = (size_t)TC_RAW + 2ull * TC_M * w.raw_stride;
    if (w.smem > TC_SMEM_MAX || w.raw_stride > 256) return fail("tc: rows too wide for the raw chunk slots");
    const int target = std::max(1, std::min(8, num_sms() / tiles));  // one CTA per SM; at most 8 partials per row
    w.splits = std::max(1, std::min(nchunks, target));
    w.chunks_per_split = (nchunks + w.splits - 1) / w.splits;
    w.splits = (nchunks + w.chunks_per_split - 1) / w.chunks_per_split;  // no empty split
    return 0;
}

int launch_tc_gemv(const TcH &w, const float *x, int xs, float *y, int ys, int nt, cudaStream_t s, bool acc = false) {
    if (nt < 1 || nt > TC_NMAX) return fail("tc gemv: nt out of range (1..32)");
    if (((uintptr_t)x & 15) || (xs & 3)) return fail("tc gemv: x must be 16-byte aligned, xs % 4 == 0");
    TcArgs a;
    a.tmap = w.tmap;
    a.W = w.W.as<uint8_t>();
    a.ldw = w.ldw;
    a.rows = w.rows;
    a.cols = w.cols;
    a.x = x;
    a.xs = xs;
    a.y = y;
    a.ys = ys;
    a.nt = nt;
    a.npad = nt <= 16 ? 16 : 32;
    a.acc = acc ? 1 : 0;
    a.chunks_per_split = w.chunks_per_split;
    a.splits = w.splits;
    a.part = w.part.as<float>();
    a.tickets = w.tickets.as<uint32_t>();
    a.raw_stride = w.raw_stride;
    a.err = dev_error_ptr();
    const dim3 grid((w.rows + TC_M - 1) / TC_M, w.splits);
    cudaError_t e = cudaSuccess;
    const bool known = dispatch_type(w.type, [&]<uint32_t TY>() {
        e = allow_max_dynamic_smem(k_tc_gemv<TY>);
        if (e == cudaSuccess) e = launch_k(k_tc_gemv<TY>, grid, dim3(TC_THREADS), w.smem, s, a);
    });
    if (!known) return fail("tc gemv: unsupported type");
    if (e != cudaSuccess) return fail(std::string("tc gemv launch: ") + cudaGetErrorString(e));
    return 0;
}

// the driver's tensor-map encoder, looked up through the runtime (the library links no driver symbol, so it loads on a
// machine without a GPU driver)
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiled encode_tiled() {
    static EncodeTiled f = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (EncodeTiled) nullptr;
        return (EncodeTiled)p;
    }();
    return f;
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
    w->ldw = (uint32_t)tc_align(rb, 16);
    cudaGetDevice(&w->dev);
    if (tc_plan(*w)) {
        delete w;
        return nullptr;
    }
    const int tiles = (rows + TC_M - 1) / TC_M;
    if (cudaMalloc(&w->W.p, (size_t)w->ldw * rows) != cudaSuccess ||
        cudaMemcpy2D(w->W.p, w->ldw, Wh, rb, rb, rows, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMalloc(&w->part.p, (size_t)w->splits * TC_NMAX * rows * 4) != cudaSuccess ||
        cudaMalloc(&w->tickets.p, (size_t)tiles * 4) != cudaSuccess ||
        cudaMemset(w->tickets.p, 0, (size_t)tiles * 4) != cudaSuccess) {
        delete w;
        fail("tc: device allocation / copy failed");
        return nullptr;
    }
    // W as a 2-D byte tensor: dims {ldw, rows}, row stride ldw (a 16-byte multiple, base 256-byte aligned)
    const cuuint64_t dims[2] = {w->ldw, (cuuint64_t)rows}, strides[1] = {w->ldw};
    const cuuint32_t box[2] = {w->raw_stride, (cuuint32_t)TC_M}, es[2] = {1, 1};
    const EncodeTiled enc = encode_tiled();
    const CUresult cr = enc ? enc(&w->tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->W.p, dims, strides, box, es,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE)
                            : CUDA_ERROR_NOT_FOUND;
    if (cr != CUDA_SUCCESS) {
        delete w;
        fail("tc: tensor map encoding failed (" + std::to_string((int)cr) + ")");
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
