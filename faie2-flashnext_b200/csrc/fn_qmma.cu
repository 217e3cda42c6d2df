// Quantised GEMV on the tensor cores as exact integer products (tcgen05.mma kind::i8), for 1..4 tokens.
//
// y[t][r] = sum_g s_{r,g} . sum_{k in g} q_{r,k} x_t[k] (+ the format's offset term): every weight of a K-quant group is
// a small unsigned integer q (Q4_K 0..15, Q6_K 0..63) times its group's scale. The CUDA-core GEMV turns each q into a
// float and multiplies it by x (about 3 instructions per weight, the limit of the decode's small GEMVs and of the
// lm_head). Here the q bytes go to the tensor cores as they are (A, u8), and x goes in as exact integers: per token,
// X_k = round(x_k 2^s) with s chosen so |X| < 2^30 (x in fixed point, 2^-31 of max |x|), split into four balanced
// base-256 digits (B, s8), X = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3. One MMA per 32-value group and 128 rows computes
// sum q d_i for every digit (and token) at once in int32 (no rounding), in its own tensor-memory columns; the epilogue
// recombines the digits in double (exact: below 2^53), applies the group's scale and offset in double, and adds the
// groups of a row in a fixed order. Per weight the CUDA cores only unpack its bits into a byte (no conversion, no FMA);
// the result is the exact dot product of the fp32 weights with the fixed-point x, rounded once to fp32.
//
// Q6_K's scales change every 16 values: the B operand then carries each half-group's digits in its own N columns (the
// other half's K positions zero), so the MMA still covers the 32-value group in one instruction.
//
// Per CTA: a contiguous row range (as the CUDA-core plan), walked in 128-row tiles; per tile the K axis in chunks of
// QM_C groups. The quant planes of a chunk (plane layout, the same device weights as k_gemv) arrive by 2-D bulk tensor
// copies into a ring; 512 threads unpack them into the MMA's K-major A tiles (8-row x 16-byte core matrices); one thread
// issues the chunk's MMAs and commits them to a barrier; the warps then read back the previous chunk's accumulators
// (tcgen05.ld) while the tensor cores work. Group order of a row's sum: the four warps of a lane quarter take the groups
// g = j mod 4 (j = 0..3) in ascending order, then ((p0 + p1) + (p2 + p3)): fixed by the format and row length, so a
// token's result does not depend on the batch or the launch shape. Every wait is bounded (DEV_WAIT_TIMEOUT).
#include <cuda.h>

#include <mutex>

#include "fn_engine.h"
#include "fn_gemv_impl.cuh"

namespace fn {

constexpr int QM_M = 128;       // rows per tile (the MMA's M)
constexpr int QM_C = 8;         // groups of 32 columns per chunk
constexpr int QM_THREADS = 512;
constexpr int QM_N = 16;        // the MMA's N: 4 digits x halves x tokens, padded
constexpr int QM_KMAX = 2048;   // columns (the B operand of every column stays in shared memory)
constexpr int QM_NBUF = 4;      // tensor-memory chunk buffers in flight between the MMA warp and the read-back warps

// per-format layout of the plane rows (fn_fastdot.cuh PlaneSpec / encode_block) as this kernel reads them
template <uint32_t TY> struct Qm;
template <> struct Qm<T_Q4_K> {
    static constexpr int H = 1;            // scale groups per 32 values
    static constexpr int RS = 4;           // raw ring stages
    static constexpr int QB = 16;          // quant bytes per group (plane 0 at 0)
    static constexpr int HB = 0;           // high-bit bytes per group (none)
    static int scale_off(int nb) { return 128 * nb; }  // [12 nb scale bytes][4 nb d, dmin]
    static int scale_bytes(int nb) { return 16 * nb; }
};
template <> struct Qm<T_Q6_K> {
    static constexpr int H = 2;
    static constexpr int RS = 3;
    static constexpr int QB = 16;          // low nibbles, plane 0 at 0
    static constexpr int HB = 8;           // 2-bit highs, plane 1 at 128 nb
    static int scale_off(int nb) { return 192 * nb; }  // [16 nb int8 scales][2 nb d]
    static int scale_bytes(int nb) { return 18 * nb; }
};

struct QmArgs {
    CUtensorMap tq;  // quant plane chunk: box QRS bytes x 128 rows
    CUtensorMap th;  // Q6_K high-bit plane chunk: box HRS bytes x 128 rows
    CUtensorMap ts;  // scale planes of a tile: box SRS bytes x 128 rows
    int rows, cols, nb, G, nt;
    const float *x;
    int xs;
    float *y;
    int ys, acc, early;
    const float *nw;  // RMSNorm folded in (nullable)
    float eps;
    uint32_t qrs, hrs, srs;         // bytes per row of a staged quant / high-bit / scale box
    uint32_t hoff;                  // byte offset of the high-bit plane in a row (Q6_K)
    uint32_t soff;                  // byte offset of the scale planes in a row
    uint32_t a_off, raw_off, b_off, s_off, sx_off, bar_off;  // shared-memory layout
    uint32_t raw_stage;             // bytes of one raw ring stage
    GemvArgs g;                     // the fused argmax fields (amx, row0, aidx, akey, kacc, ticket, xr, nt) and err
};

// sm_100 shared-memory matrix descriptor: start, leading / stride byte offsets (>> 4), version 1, no swizzle
__device__ __forceinline__ uint64_t qm_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
           (1ull << 46);
}
// instruction descriptor of kind::i8: s32 accumulator (dtype 2), A u8 (0), B s8 (1), both K-major, N >> 3, M >> 4
__host__ __device__ constexpr uint32_t qm_idesc(int m, int n) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void qm_mma(uint32_t dtmem, uint64_t a, uint64_t b, uint32_t idesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(dtmem),
        "l"(a), "l"(b), "r"(idesc), "r"(0)
        : "memory");
}
__device__ __forceinline__ void qm_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void qm_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void qm_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void qm_proxy_fence() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
// 16 consecutive 32-bit columns of this warp's 32 tensor-memory lanes
__device__ __forceinline__ void qm_ld16(uint32_t taddr, int (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = (int)r[i];
}
__device__ __forceinline__ void qm_tma2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// the 32 quant bytes of group gc of staged row r (A's two 16-byte core-matrix rows: values 0..15, 16..31)
template <uint32_t TY>
__device__ __forceinline__ void qm_unpack(const uint8_t *rq, const uint8_t *rh, int gc, uint4 &lo, uint4 &hi) {
    const uint4 w = *(const uint4 *)(rq + 16 * gc);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    uint32_t l[4], h[4];
    if constexpr (TY == T_Q4_K) {  // byte i = q[i] | q[16 + i] << 4
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            l[k] = ws[k] & 0x0F0F0F0Fu;
            h[k] = (ws[k] >> 4) & 0x0F0F0F0Fu;
        }
    } else {  // Q6_K: low nibbles as Q4_K, the 2-bit highs of values 4k + i in bits 2k of byte i of word A (B: 16..)
        const uint2 hb = *(const uint2 *)(rh + 8 * gc);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t ta = (k < 2 ? (hb.x << (4 - 2 * k)) : (hb.x >> (2 * k - 4))) & 0x30303030u;
            const uint32_t tb = (k < 2 ? (hb.y << (4 - 2 * k)) : (hb.y >> (2 * k - 4))) & 0x30303030u;
            l[k] = (ws[k] & 0x0F0F0F0Fu) | ta;
            h[k] = ((ws[k] >> 4) & 0x0F0F0F0Fu) | tb;
        }
    }
    lo = make_uint4(l[0], l[1], l[2], l[3]);
    hi = make_uint4(h[0], h[1], h[2], h[3]);
}

// the balanced base-256 digits of X (|X| < 2^30) and their bytes packed four values to a word
__device__ __forceinline__ void qm_digits(int X, int (&d)[4]) {
    d[0] = (int)(int8_t)(X & 255);
    int r = (X - d[0]) >> 8;
    d[1] = (int)(int8_t)(r & 255);
    r = (r - d[1]) >> 8;
    d[2] = (int)(int8_t)(r & 255);
    d[3] = (r - d[2]) >> 8;
}

__device__ __forceinline__ void qm_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void qm_named_sync(int id, int n) { asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory"); }

// warp roles: 0 issues the bulk tensor copies, 1 the MMAs (one lane each), 2..7 unpack the quant bytes into A,
// 8..15 read the accumulators back (two warps per tensor-memory lane quarter); they meet only at mbarriers
constexpr int QM_NPREP = 6, QM_NREAD = 8;

template <uint32_t TY>
__global__ void __launch_bounds__(QM_THREADS, 1) k_qmma(const __grid_constant__ QmArgs a) {
    using T = Qm<TY>;
    constexpr int H = T::H, NB8 = QM_N / 8, RS = T::RS;
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_fail;
    __shared__ int s_mx[4], s_shift[4];
    __shared__ float s_ns[4];
    uint8_t *A = sm + a.a_off, *raw = sm + a.raw_off, *B = sm + a.b_off, *S = sm + a.s_off;
    double *SX = (double *)(sm + a.sx_off);     // [nt][G][H]: sum of X over each scale group (nt H <= 4, G <= 64)
    double *part = SX + 256;                    // [2][QM_M]: a tile's row partials by group class m
    uint64_t *rfull = (uint64_t *)(sm + a.bar_off), *rempty = rfull + RS, *aready = rempty + RS, *afree = aready + 2,
             *mdone = afree + 2, *tfree = mdone + QM_NBUF, *sfull = tfree + QM_NBUF, *sfree = sfull + 2;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r0 = (int)((long long)blockIdx.x * a.rows / gridDim.x);
    const int nrow = (int)((long long)(blockIdx.x + 1) * a.rows / gridDim.x) - r0;
    const int ntile = (nrow + QM_M - 1) / QM_M, nch = a.G / QM_C, total = ntile * nch, nt = a.nt;
    const uint32_t idesc = qm_idesc(QM_M, QM_N);
    // a bounded wait that gives up at once when another role already failed
    auto wt = [&](uint64_t *bar, uint32_t par) {
        if (s_fail) return false;
        if (mbar_wait(bar, par)) return true;
        s_fail = 1;
        return false;
    };

    if (tid == 0) {
        for (int i = 0; i < RS; ++i) {
            mbar_init(&rfull[i], 1);
            mbar_init(&rempty[i], QM_NPREP);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&aready[i], QM_NPREP);
            mbar_init(&afree[i], 1);
            mbar_init(&sfull[i], 1);
            mbar_init(&sfree[i], QM_NREAD);
        }
        for (int i = 0; i < QM_NBUF; ++i) {
            mbar_init(&mdone[i], 1);
            mbar_init(&tfree[i], QM_NREAD);
        }
        mbar_fence_init();
        s_fail = 0;
    }
    if (tid < 4) s_mx[tid] = 0;
    if (warp == 1) {  // tensor memory: QM_NBUF chunk buffers of QM_C groups x QM_N columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&s_tmem)),
                     "r"(QM_NBUF * QM_C * QM_N)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    for (int i = tid; i < a.cols; i += QM_THREADS) *(uint4 *)(B + 16 * (size_t)i) = make_uint4(0, 0, 0, 0);  // B
    qm_fence_before();
    __syncthreads();
    qm_fence_after();
    const uint32_t tmem = s_tmem;
    int n_raw = 0, n_scl = 0, n_mma = 0;  // copies / tile scales / chunk MMAs issued (the issuing lanes)
    unsigned long long best[4] = {0ull, 0ull, 0ull, 0ull};  // fused argmax: per token, the best key of this thread's rows
    if (warp == 0) {
        // ---- bulk tensor copies: a tile's scale planes before its first chunk, each chunk's quant planes once its
        // ring slot is empty; the weights are read-only, so the first RS chunks go before the wait
        if (lane == 0) {
            for (int i = 0; i < total && !s_fail; ++i) {
                const int tile = i / nch, c = i % nch, sl = i % RS;
                if (c == 0) {
                    if (tile >= 2 && !wt(&sfree[tile & 1], (uint32_t)((tile >> 1) - 1) & 1u)) break;
                    mbar_arrive_tx(&sfull[tile & 1], (uint32_t)QM_M * a.srs);
                    qm_tma2d(S + (size_t)(tile & 1) * QM_M * a.srs, &a.ts, (int)a.soff, r0 + tile * QM_M, &sfull[tile & 1]);
                    n_scl = tile + 1;
                }
                if (i >= RS && !wt(&rempty[sl], (uint32_t)((i / RS) - 1) & 1u)) break;
                uint8_t *dst = raw + (size_t)sl * a.raw_stage;
                mbar_arrive_tx(&rfull[sl], (uint32_t)QM_M * (a.qrs + a.hrs));
                qm_tma2d(dst, &a.tq, T::QB * QM_C * c, r0 + tile * QM_M, &rfull[sl]);
                if constexpr (T::HB > 0)
                    qm_tma2d(dst + QM_M * a.qrs, &a.th, (int)a.hoff + T::HB * QM_C * c, r0 + tile * QM_M, &rfull[sl]);
                n_raw = i + 1;
                if (i == min(total, RS) - 1 && !a.early) {  // the first copies fly; then the programmatic chain
                    pdl_wait();
                    pdl_trigger();
                }
            }
            if (total == 0 && !a.early) {
                pdl_wait();
                pdl_trigger();
            }
        }
    } else {
        if (a.early) pdl_trigger();
        else {
            pdl_wait();
            pdl_trigger();
        }
        // ---- x -> B (warps 1..15): thread (t, g) takes token t's group g (32 values): x * nw, its max |.|, its sum of
        // squares; then X = round(v 2^s), |X| < 2^30, whose four digits go to B's rows n = 4 (H t + h) + d
        constexpr int NX = QM_THREADS - 32;
        const float *x = after_wait(a.x);
        const int xi = tid - 32, xt = xi / a.G, xg = xi % a.G;
        const bool xl = xt < nt;
        float v[32];
        float gss = 0.0f, mx = 0.0f;
        if (xl) {
            const float4 *src = (const float4 *)(x + (size_t)xt * a.xs + 32 * xg);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 f = src[i];
                v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
            }
            if (a.nw) {
                const float4 *wv = (const float4 *)(a.nw + 32 * xg);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 w = wv[i];
                    const float wq[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        gss = __fmaf_rn(v[4 * i + u], v[4 * i + u], gss);
                        v[4 * i + u] = __fmul_rn(v[4 * i + u], wq[u]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fabsf(v[i]));
            atomicMax(&s_mx[xt], __float_as_int(mx));  // non-negative floats order like their bits
            part[xt * 64 + xg] = (double)gss;          // the group's sum of squares (for the norm), through part
        }
        qm_named_sync(1, NX);
        if (warp - 1 < nt) {  // token warp: the fixed-point shift and the folded norm's scale (norm_scale's order)
            const int t = warp - 1;
            const int e = ((s_mx[t] >> 23) & 255) - 127;  // max |v| in [2^e, 2^(e+1))
            float ss = 0.0f;
            if (a.nw) {
                for (int g = lane; g < a.G; g += 32) ss = __fadd_rn(ss, (float)part[t * 64 + g]);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
            }
            if (lane == 0) {
                s_shift[t] = s_mx[t] == 0 ? 0 : 29 - e;
                s_ns[t] = a.nw ? rsqrtf(ss / (float)a.cols + a.eps) : 1.0f;
            }
        }
        qm_named_sync(1, NX);
        if (xl) {
            const double sc = ldexp(1.0, s_shift[xt]);
            long long sx[2] = {0, 0};
#pragma unroll
            for (int kc = 0; kc < 2; ++kc) {  // values 16 kc .. 16 kc + 15: core-matrix column 2 xg + kc
                uint32_t w[4][4];
#pragma unroll
                for (int u = 0; u < 4; ++u) w[0][u] = w[1][u] = w[2][u] = w[3][u] = 0;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int X = (int)__double2ll_rn((double)v[16 * kc + i] * sc);
                    sx[H == 2 ? kc : 0] += X;
                    int d[4];
                    qm_digits(X, d);
#pragma unroll
                    for (int dd = 0; dd < 4; ++dd) w[dd][i >> 2] |= ((uint32_t)d[dd] & 255u) << (8 * (i & 3));
                }
                const int h = H == 2 ? kc : 0;
                uint8_t *col = B + (size_t)(2 * xg + kc) * NB8 * 128;
#pragma unroll
                for (int dd = 0; dd < 4; ++dd) {
                    const int n = 4 * (H * xt + h) + dd;
                    *(uint4 *)(col + (n >> 3) * 128 + (n & 7) * 16) = make_uint4(w[dd][0], w[dd][1], w[dd][2], w[dd][3]);
                }
            }
#pragma unroll
            for (int h = 0; h < H; ++h) SX[(xt * a.G + xg) * H + h] = (double)sx[h];
        }
        qm_proxy_fence();  // B's generic-proxy stores before the tensor cores read it
        qm_named_sync(1, NX);
        if (warp == 1) {
            // ---- MMAs: chunk i's groups from A[i & 1] into tensor buffer i % QM_NBUF, one commit per buffer and A
            if (lane == 0) {
                const uint32_t bbase = smem_u32(B);
                for (int i = 0; i < total; ++i) {
                    const int c = i % nch, ab = i & 1, tb = i % QM_NBUF;
                    if (!wt(&aready[ab], (uint32_t)(i >> 1) & 1u)) break;
                    if (i >= QM_NBUF && !wt(&tfree[tb], (uint32_t)((i / QM_NBUF) - 1) & 1u)) break;
                    qm_fence_after();
                    const uint32_t abase = smem_u32(A + (size_t)ab * QM_C * 4096);
#pragma unroll
                    for (int gc = 0; gc < QM_C; ++gc) {
                        const int g = c * QM_C + gc;
                        const uint64_t ad = qm_desc(abase + gc * 4096, 2048u, 128u);
                        const uint64_t bd = qm_desc(bbase + (uint32_t)(2 * g) * NB8 * 128, NB8 * 128u, 128u);
                        qm_mma(tmem + (uint32_t)(tb * QM_C + gc) * QM_N, ad, bd, idesc);
                    }
                    qm_commit(&mdone[tb]);
                    qm_commit(&afree[ab]);
                    n_mma = i + 1;
                }
            }
        } else if (warp < 2 + QM_NPREP) {
            // ---- unpack: chunk i's quant planes (ring slot i % RS) into A[i & 1]; a warp takes 32 consecutive rows
            // of a group at a time, so its 16-byte stores fill whole core matrices
            const int pt = tid - 64;
            for (int i = 0; i < total; ++i) {
                const int tile = i / nch, ab = i & 1, sl = i % RS;
                bool ok = wt(&rfull[sl], (uint32_t)(i / RS) & 1u);
                if (ok && i >= 2) ok = wt(&afree[ab], (uint32_t)((i >> 1) - 1) & 1u);
                if (ok) {
                    const uint8_t *rq = raw + (size_t)sl * a.raw_stage, *rh = rq + QM_M * a.qrs;
                    uint8_t *Ab = A + (size_t)ab * QM_C * 4096;
                    for (int it = pt; it < QM_M * QM_C; it += 32 * QM_NPREP) {
                        const int r = it & (QM_M - 1), gc = it >> 7;
                        if (tile * QM_M + r >= nrow) continue;  // rows past the range: accumulator lanes never read
                        uint4 lo, hi;
                        qm_unpack<TY>(rq + (size_t)r * a.qrs, rh + (size_t)r * a.hrs, gc, lo, hi);
                        uint8_t *dst = Ab + gc * 4096 + (r >> 3) * 128 + (r & 7) * 16;
                        *(uint4 *)dst = lo;
                        *(uint4 *)(dst + 2048) = hi;
                    }
                }
                qm_proxy_fence();
                __syncwarp();
                if (lane == 0) {
                    qm_arrive(&aready[ab]);
                    qm_arrive(&rempty[sl]);
                }
            }
        } else {
            // ---- read-back: warp (m, q) takes lanes 32 q .. 32 q + 31 (the tile's rows) and the groups with
            // gc = m mod 2 of each chunk; a row's sum: each class in ascending group order, then p0 + p1
            const int q = warp & 3, m = (warp - 2 - QM_NPREP) >> 2;
            const int row = 32 * q + lane;
            double acc[4] = {0.0, 0.0, 0.0, 0.0};
            for (int p = 0; p < total; ++p) {
                const int tile = p / nch, c = p % nch, tb = p % QM_NBUF;
                bool ok = true;
                if (c == 0) ok = wt(&sfull[tile & 1], (uint32_t)(tile >> 1) & 1u);
                ok = ok && wt(&mdone[tb], (uint32_t)(p / QM_NBUF) & 1u);
                ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective: all lanes or none
                qm_fence_after();
                const bool valid = ok && tile * QM_M + row < nrow;
                const uint8_t *srow = S + (size_t)(tile & 1) * QM_M * a.srs + (size_t)row * a.srs;
#pragma unroll
                for (int k = 0; k < QM_C / 2; ++k) {
                    const int gc = m + 2 * k, g = c * QM_C + gc;
                    int vv[16];
                    if (ok) qm_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(tb * QM_C + gc) * QM_N, vv);
                    if (!valid) continue;
                    const int b = g >> 3;
                    if constexpr (TY == T_Q4_K) {
                        uint32_t sc, mn;
                        kq_scale_min(g & 7, srow + 12 * b, sc, mn);
                        const uint32_t dm = u32_at(srow + 12 * a.nb + 4 * b);
                        const double dl = (double)__fmul_rn(f16_of(dm, 0), (float)sc);
                        const double ml = (double)__fmul_rn(f16_of(dm, 1), (float)mn);
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            if (t >= nt) break;
                            const double sv = (double)vv[4 * t] + 256.0 * vv[4 * t + 1] + 65536.0 * vv[4 * t + 2] +
                                              16777216.0 * vv[4 * t + 3];
                            acc[t] += dl * sv - ml * SX[t * a.G + g];
                        }
                    } else {
                        const uint32_t s2 = u16_at(srow + 16 * b + 2 * (g & 7));
                        const float d = f16_at(srow + 16 * a.nb + 2 * b);
                        const double ds0 = (double)__fmul_rn(d, (float)(int8_t)(s2 & 255u));
                        const double ds1 = (double)__fmul_rn(d, (float)(int8_t)(s2 >> 8));
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            if (t >= nt) break;
                            const int *w0 = vv + 8 * t;
                            const double s0 = (double)w0[0] + 256.0 * w0[1] + 65536.0 * w0[2] + 16777216.0 * w0[3];
                            const double s1 = (double)w0[4] + 256.0 * w0[5] + 65536.0 * w0[6] + 16777216.0 * w0[7];
                            acc[t] += ds0 * (s0 - 32.0 * SX[(t * a.G + g) * 2]) +
                                      ds1 * (s1 - 32.0 * SX[(t * a.G + g) * 2 + 1]);
                        }
                    }
                }
                qm_fence_before();
                __syncwarp();
                if (lane == 0) qm_arrive(&tfree[tb]);
                if (c != nch - 1) continue;
                // the tile's rows are complete: the two classes, 2^-s, the norm scale, y and the argmax key
                for (int t = 0; t < nt; ++t) {
                    part[m * QM_M + row] = acc[t];
                    acc[t] = 0.0;
                    qm_named_sync(2, 32 * QM_NREAD);
                    if (m == 0 && valid && !s_fail) {
                        const double tot = part[row] + part[QM_M + row];
                        float yv = (float)ldexp(tot, -s_shift[t]);
                        if (a.nw) yv = __fmul_rn(yv, s_ns[t]);
                        const int r = r0 + tile * QM_M + row;
                        if (a.y) {
                            float *o = a.y + (size_t)t * a.ys + r;
                            *o = a.acc ? __fadd_rn(*o, yv) : yv;
                        }
                        if (a.g.amx) best[t] = kmax(best[t], amax_key(yv, a.g.row0 + r));
                    }
                    qm_named_sync(2, 32 * QM_NREAD);
                }
                __syncwarp();
                if (lane == 0) qm_arrive(&sfree[tile & 1]);
            }
        }
    }
    // ---- wind down: the copies and MMAs this CTA issued complete before its shared and tensor memory are released
    if (s_fail) {
        if (tid == 0) {
            dev_fail(a.g.err, DEV_WAIT_TIMEOUT);
            for (int k = max(0, n_raw - RS); k < n_raw; ++k) mbar_wait(&rfull[k % RS], (uint32_t)(k / RS) & 1u, 1u << 16);
            for (int k = max(0, n_scl - 2); k < n_scl; ++k) mbar_wait(&sfull[k & 1], (uint32_t)(k >> 1) & 1u, 1u << 16);
        }
        if (tid == 32)
            for (int k = max(0, n_mma - QM_NBUF); k < n_mma; ++k)
                mbar_wait(&mdone[k % QM_NBUF], (uint32_t)(k / QM_NBUF) & 1u, 1u << 16);
    }
    qm_fence_before();
    __syncthreads();
    if (warp == 1) {
        qm_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(QM_NBUF * QM_C * QM_N)
                     : "memory");
    }
    if (a.early) pdl_wait();
    if (a.g.amx && !s_fail) {  // the read-back warps hold the written rows: their maxima per token, then the grid's
        __shared__ unsigned long long s_best[16][4][4];
        for (int i = tid; i < 16 * 4 * 4; i += QM_THREADS) (&s_best[0][0][0])[i] = 0ull;
        __syncthreads();
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const unsigned long long k = warp_kmax(best[t]);
            if (lane == 0) s_best[warp][0][t] = k;
        }
        gemv_argmax_epilogue<4>(0ull, s_best, a.g);  // begins with a barrier
    }
}

// ---- host: plan, tensor maps, launch ---------------------------------------------------------------------------

using EncodeTiledQ = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledQ qm_encoder() {
    static EncodeTiledQ f = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (EncodeTiledQ) nullptr;
        return (EncodeTiledQ)p;
    }();
    return f;
}

// tokens per call the integer tensor-core path takes for a format (0: not this path)
int qmma_cap(uint32_t type, int cols) {
    if (cols < 256 || cols % 256 || cols > QM_KMAX) return 0;
    return type == T_Q4_K ? 4 : type == T_Q6_K ? 2 : 0;
}

static uint32_t qm_box_bytes(uint32_t need) {  // a 16-byte multiple, an odd number of 16-byte units where it fits
    uint32_t b = (need + 15u) & ~15u;
    if ((b / 16) % 2 == 0 && b + 16 <= 256) b += 16;
    return b;
}

template <uint32_t TY>
static int qmma_launch_t(const GemvPlan &p, const uint8_t *W, const float *x, int xs, float *y, int ys, int nt,
                         bool acc, bool early, cudaStream_t s, const GemvArgmax *am) {
    using T = Qm<TY>;
    QmArgs a{};
    const int nb = p.cols / 256;
    a.rows = p.rows;
    a.cols = p.cols;
    a.nb = nb;
    a.G = p.cols / 32;
    a.nt = nt;
    a.x = x;
    a.xs = xs;
    a.y = y;
    a.ys = ys;
    a.acc = acc ? 1 : 0;
    a.early = early && settings().early && settings().pdl ? 1 : 0;
    a.nw = p.nw;
    a.eps = p.eps;
    a.qrs = qm_box_bytes(T::QB * QM_C);
    a.hrs = T::HB ? qm_box_bytes(T::HB * QM_C) : 0;
    a.srs = qm_box_bytes((uint32_t)T::scale_bytes(nb));
    a.hoff = 128u * nb;
    a.soff = (uint32_t)T::scale_off(nb);
    if (a.qrs > 256 || a.hrs > 256 || a.srs > 256) return fail("qmma: rows too wide for the staging boxes");
    auto al = [](size_t v, size_t q) { return (v + q - 1) / q * q; };
    a.a_off = 0;
    a.raw_off = 2u * QM_C * 4096;
    a.raw_stage = (uint32_t)al((size_t)QM_M * (a.qrs + a.hrs), 128);
    a.b_off = a.raw_off + T::RS * a.raw_stage;
    a.s_off = (uint32_t)al(a.b_off + (size_t)p.cols * 16, 128);
    a.sx_off = (uint32_t)al(a.s_off + 2ull * QM_M * a.srs, 128);
    a.bar_off = a.sx_off + 4096;  // SX [256] + part [2][128] doubles
    const size_t smem = a.bar_off + (2 * T::RS + 2 * QM_NBUF + 8) * 8;
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, k_qmma<TY>) != cudaSuccess || smem + fa.sharedSizeBytes > 227 * 1024)
        return fail("qmma: shared memory plan too large");
    const EncodeTiledQ enc = qm_encoder();
    if (!enc) return fail("qmma: no tensor-map encoder");
    const cuuint64_t dims[2] = {p.ldw, (cuuint64_t)p.rows}, strides[1] = {p.ldw};
    const cuuint32_t es[2] = {1, 1};
    auto encode = [&](CUtensorMap *m, uint32_t box) {
        const cuuint32_t bx[2] = {box, (cuuint32_t)QM_M};
        return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)W, dims, strides, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    };
    if (encode(&a.tq, a.qrs) != CUDA_SUCCESS || (T::HB && encode(&a.th, a.hrs) != CUDA_SUCCESS) ||
        encode(&a.ts, a.srs) != CUDA_SUCCESS)
        return fail("qmma: tensor map encoding failed");
    a.g.err = dev_error_ptr();
    a.g.nt = nt;
    a.g.amx = 0;
    if (am) {
        if (!am->kacc || !am->ticket || (!am->index && !am->key && !am->xr)) return fail("qmma argmax: missing scratch");
        a.g.amx = 1;
        a.g.row0 = am->row0;
        a.g.aidx = am->index;
        a.g.akey = am->key;
        a.g.kacc = am->kacc;
        a.g.ticket = am->ticket;
        if (am->xr) a.g.xr = *am->xr;
    } else if (!y) {
        return fail("qmma: y is null");
    }
    const int ctas = std::max(1, std::min(num_sms(), p.rows));
    cudaError_t e = allow_max_dynamic_smem(k_qmma<TY>);
    if (e == cudaSuccess) e = launch_k(k_qmma<TY>, dim3(ctas), dim3(QM_THREADS), smem, s, a);
    if (e != cudaSuccess) return fail(std::string("qmma launch: ") + cudaGetErrorString(e));
    return 0;
}

int launch_qmma(const GemvPlan &p, const uint8_t *W, const float *x, int xs, float *y, int ys, int nt, bool acc,
                bool early, cudaStream_t s, const GemvArgmax *am) {
    if (nt < 1 || nt > qmma_cap(p.type, p.cols)) return fail("qmma: unsupported type, width or token count");
    if (((uintptr_t)W & 15) || ((uintptr_t)x & 15) || (xs & 3)) return fail("qmma: W and x must be 16-byte aligned");
    if (p.type == T_Q4_K) return qmma_launch_t<T_Q4_K>(p, W, x, xs, y, ys, nt, acc, early, s, am);
    return qmma_launch_t<T_Q6_K>(p, W, x, xs, y, ys, nt, acc, early, s, am);
}

}  // namespace fn
