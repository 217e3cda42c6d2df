// Routed-expert kernel templates (gate/up, down + combine), the fused top-k routing, and their per-format launchers
// (instantiated in fn_moe_i*.cu, one group of formats per translation unit). See fn_moe.cu for the design.
#pragma once

#include <unordered_set>

#include "fn_engine.h"
#include "fn_moe.h"
#include "fn_rowdot.cuh"

namespace fn {

// ---------------------------------------------------------------------------------------------------------------
// top-k routing

// order-preserving 64-bit key: larger logit first, then lower index first. -0 and +0 are the same probability
// (a tie, won by the lower index), so -0 is keyed as +0.
__device__ __forceinline__ unsigned long long route_key(float l, int idx) {
    uint32_t u = __float_as_uint(l == 0.0f ? 0.0f : l);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ int key_index(unsigned long long k) { return (int)(0xFFFFFFFFu - (uint32_t)k); }

// Descending bitonic sort of 32 * E keys held by one warp, element i = lane * E + e.
template <int E> __device__ __forceinline__ void warp_sort_desc(unsigned long long (&v)[E], int lane) {
#pragma unroll
    for (int size = 2; size <= 32 * E; size <<= 1) {
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
            if (j >= E) {
                const int lm = j / E;
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const int i = lane * E + e;
                    const unsigned long long o = __shfl_xor_sync(0xffffffffu, v[e], lm);
                    const bool desc = (i & size) == 0, lower = (lane & lm) == 0;
                    const bool keep_max = desc == lower;
                    v[e] = keep_max ? (v[e] > o ? v[e] : o) : (v[e] < o ? v[e] : o);
                }
            } else {
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const int p = e ^ j;
                    if (p > e) {
                        const int i = lane * E + e;
                        const bool desc = (i & size) == 0;
                        const unsigned long long a = v[e], b = v[p];
                        const bool sw = desc ? a < b : a > b;
                        v[e] = sw ? b : a;
                        v[p] = sw ? a : b;
                    }
                }
            }
        }
    }
}

template <int E>
__device__ __forceinline__ void warp_topk_keys(const float *logits, int lo, int hi, int k, unsigned long long *out,
                                               int lane) {
    unsigned long long v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int idx = lo + lane * E + e;
        v[e] = idx < hi ? route_key(logits[idx], idx) : 0ull;
    }
    warp_sort_desc<E>(v, lane);
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int i = lane * E + e;
        if (i < k) out[i] = v[e];
    }
}

// Route one token: the k best of logits[0, ne) into sel[k], w[k] (shared memory). Every thread of the block calls it;
// needs 256 threads (8 warps), ne <= 1024, k <= 16, and keys[] of 8 * 16 entries in shared memory.
__device__ __forceinline__ void route_token(const float *logits, int ne, int k, int *sel, float *w, unsigned long long *keys) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per = (ne + 7) / 8, lo = warp * per, hi = min(ne, lo + per);
    if (per <= 32) warp_topk_keys<1>(logits, lo, hi, k, keys + warp * 16, lane);
    else if (per <= 64) warp_topk_keys<2>(logits, lo, hi, k, keys + warp * 16, lane);
    else warp_topk_keys<4>(logits, lo, hi, k, keys + warp * 16, lane);
    __syncthreads();
    if (warp == 0) {
        unsigned long long v[4];  // 8 warps x k <= 16 candidates = 128 = 32 x 4
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int i = lane * 4 + e, wi = i / 16, j = i % 16;
            v[e] = j < k ? keys[wi * 16 + j] : 0ull;
        }
        warp_sort_desc<4>(v, lane);
        // lanes 0..3 hold ranks 0..15; rank r = lane * 4 + e
        const float lmax = logits[key_index(__shfl_sync(0xffffffffu, v[0], 0))];
        float ev[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = lane * 4 + e;
            ev[e] = r < k ? expf(logits[key_index(v[e])] - lmax) : 0.0f;
        }
        // s = sum over ranks 0..k-1 in rank order (lane 0 gathers, sequential like the reference)
        float s = 0.0f;
        for (int r = 0; r < k; ++r) s += __shfl_sync(0xffffffffu, ev[r & 3], r >> 2);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = lane * 4 + e;
            if (r < k) {
                sel[r] = key_index(v[e]);
                w[r] = ev[e] / s;
            }
        }
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------------------------------------------
// gate / up

struct MoeGuArgs {
    const uint8_t *Wg, *Wu, *Wsg, *Wsu;  // routed (ne * ffe rows) and shared (ffe rows), stride ldw
    uint32_t ldw;
    int nb;  // blocks per row
    int ne, k, ffe, d, nt;
    const float *logits;
    int ls;  // logits token stride (>= ne + 1: column ne is the shared-gate logit)
    const float *x;  // [nt][d]
    float *act;      // [nt][k + 1][ffe]
    int *sel_out;    // [nt][k] or null (written by CTA 0)
    float *w_out;
    int rps, slots;
    uint32_t stage_bytes, ring_off, x_off, grid_off, misc_off;
    uint32_t *err;
};

template <uint32_t TY, int LPR, int GPL, bool XREG, bool SOA>
__global__ void __launch_bounds__(256, 1) k_moe_gu(const MoeGuArgs a) {
    constexpr int RR = LPR == 32 ? 2 : 1;
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t *full = (uint64_t *)sm;
    uint8_t *ring = sm + a.ring_off;
    float *xsm = (float *)(sm + a.x_off);
    uint32_t *grid = (uint32_t *)(sm + a.grid_off);
    int *sel = (int *)(sm + a.misc_off);                          // [nt][16]
    float *wsel = (float *)(sel + 8 * 16);                          // [nt][16]
    unsigned long long *keys = (unsigned long long *)(wsel + 8 * 16);  // [128]
    float *res = (float *)(keys + 128);                              // [2 * rps]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const int G = a.d / 32, ks = a.k + 1;
    const long long U = (long long)a.nt * ks * a.ffe;
    const long long u0 = (long long)blockIdx.x * U / gridDim.x, u1 = (long long)(blockIdx.x + 1) * U / gridDim.x;
    // stages: runs of <= rps consecutive units inside one (t, slot) segment
    auto stage_span = [&](long long from, long long &to) {
        const long long seg_end = (from / a.ffe + 1) * a.ffe;
        to = min(min(from + a.rps, seg_end), u1);
    };
    int nst = 0;
    for (long long u = u0, v; u < u1; u = v, ++nst) stage_span(u, v);

    if (tid == 0) {
        for (int s = 0; s < a.slots; ++s) mbar_init(&full[s], 1);
        mbar_fence_init();
    }
    stage_grid<TY>(grid);
    pdl_wait();
    const float *logits = after_wait(a.logits);
    const float *x = after_wait(a.x);
    for (int t = 0; t < a.nt; ++t) route_token(logits + (size_t)t * a.ls, a.ne, a.k, sel + t * 16, wsel + t * 16, keys);
    if (blockIdx.x == 0 && a.sel_out && tid < a.nt * a.k) {
        const int t = tid / a.k, i = tid % a.k;
        a.sel_out[t * a.k + i] = sel[t * 16 + i];
        a.w_out[t * a.k + i] = wsel[t * 16 + i];
    }
    stage_x(xsm, x, a.d, a.nt, G, ScaleX<TY, SOA>::v);
    pdl_trigger();

    auto rows_ptr = [&](long long u, const uint8_t *&g, const uint8_t *&up) {
        const int t = (int)(u / ((long long)ks * a.ffe)), rem = (int)(u % ((long long)ks * a.ffe));
        const int s = rem / a.ffe, r = rem % a.ffe;
        if (s < a.k) {
            const int e = sel[t * 16 + s];
            const size_t off = ((size_t)e * a.ffe + r) * a.ldw;
            g = a.Wg + off;
            up = a.Wu + off;
        } else {
            g = a.Wsg + (size_t)r * a.ldw;
            up = a.Wsu + (size_t)r * a.ldw;
        }
    };
    long long next_u = u0;
    int issued = 0;
    auto issue_next = [&]() {  // thread 0
        long long to;
        stage_span(next_u, to);
        const int slot = issued % a.slots, n = (int)(to - next_u);
        const uint32_t half = (uint32_t)n * a.ldw;
        const uint8_t *g, *up;
        rows_ptr(next_u, g, up);
        uint8_t *dst = ring + (size_t)slot * a.stage_bytes;
        mbar_arrive_tx(&full[slot], 2 * half);
        bulk_g2s(dst, g, half, &full[slot]);
        bulk_g2s(dst + (size_t)a.rps * a.ldw, up, half, &full[slot]);
        next_u = to;
        ++issued;
    };
    if (tid == 0)
        while (issued < min(nst, a.slots)) issue_next();

    constexpr int RPW = 32 / LPR;
    const int lr = lane % LPR, sub = lane / LPR;
    XReg<LPR, (GPL > 0 ? GPL : 1)> xr;
    if constexpr (XREG) xr.load(xsm, lr);  // one token (nt == 1)

    long long u = u0;
    int st = 0;
    for (; st < nst; ++st) {
        long long to;
        stage_span(u, to);
        const int n = (int)(to - u), slot = st % a.slots;
        const int t = (int)(u / ((long long)ks * a.ffe));
        const bool ok = warp_wait(&full[slot], (uint32_t)(st / a.slots) & 1u);
        if (ok) {
            const uint8_t *sbuf = ring + (size_t)slot * a.stage_bytes;
            for (int base = warp * RPW * RR; base < 2 * n; base += nw * RPW * RR) {  // rows 0..n-1 gate, n..2n-1 up
                const uint8_t *rp[RR];
                bool valid[RR];
                int row[RR];
#pragma unroll
                for (int q = 0; q < RR; ++q) {
                    row[q] = base + q * RPW + sub;
                    valid[q] = row[q] < 2 * n;
                    const int srow = !valid[q] ? 0 : row[q] < n ? row[q] : a.rps + (row[q] - n);
                    rp[q] = sbuf + (size_t)srow * a.ldw;
                }
                double acc[RR][1];
                rows_dot<TY, SOA, 1, LPR, GPL, XREG, RR>(rp, valid, a.nb, grid, xr, xsm + (size_t)t * G * XPAD, G, lr, 1,
                                                        acc);
                const bool hi = RR == 2 && (lane & 16);  // selects keep valid / row / acc in registers
                if ((hi ? valid[RR - 1] : valid[0]) && (RR == 2 ? (lane & 15) == 0 : lr == 0))
                    res[hi ? row[RR - 1] : row[0]] = __double2float_rn(acc[0][0]);
            }
        }
        if (__syncthreads_or(!ok)) {
            if (tid == 0) dev_fail(a.err, DEV_WAIT_TIMEOUT);
            break;
        }
        for (int i = tid; i < n; i += blockDim.x) a.act[u + i] = silu(res[i]) * res[n + i];  // act = silu(g) * u
        __syncthreads();
        if (tid == 0 && issued < nst) issue_next();
        u = to;
    }
    if (st < nst && tid == 0)
        for (int s2 = st; s2 < min(nst, st + a.slots); ++s2) mbar_wait(&full[s2 % a.slots], (uint32_t)(s2 / a.slots) & 1u, 1u << 16);
}

// ---------------------------------------------------------------------------------------------------------------
// down + shared expert + combine

struct MoeDownArgs {
    const uint8_t *Wd, *Wsd;  // routed (ne * d rows) and shared (d rows), ffe columns, stride ldw
    uint32_t ldw;
    int nb;
    int ne, k, ffe, d, nt;
    const float *logits;
    int ls;
    const float *act;  // [nt][k + 1][ffe]
    float *y;          // [nt][d]
    int acc;
    int chunks;  // row chunks per token (gridDim.x)
    int rps, slots;
    uint32_t stage_bytes, ring_off, x_off, grid_off, misc_off;
    uint32_t *err;
};

template <uint32_t TY, int LPR, bool SOA>
__global__ void __launch_bounds__(256, 1) k_moe_down(const MoeDownArgs a) {
    constexpr int RR = LPR == 32 ? 2 : 1;
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t *full = (uint64_t *)sm;
    uint8_t *ring = sm + a.ring_off;
    float *xsm = (float *)(sm + a.x_off);
    uint32_t *grid = (uint32_t *)(sm + a.grid_off);
    int *sel = (int *)(sm + a.misc_off);  // [16]
    float *wsel = (float *)(sel + 16);
    unsigned long long *keys = (unsigned long long *)(wsel + 16);
    float *res = (float *)(keys + 128);  // [(k + 1) * rps]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const int t = blockIdx.y, G = a.ffe / 32, ks = a.k + 1;
    const int r0 = (int)((long long)blockIdx.x * a.d / gridDim.x), r1 = (int)((long long)(blockIdx.x + 1) * a.d / gridDim.x);
    const int nchunk = (r1 - r0 + a.rps - 1) / a.rps, nst = nchunk * ks;

    if (tid == 0) {
        for (int s = 0; s < a.slots; ++s) mbar_init(&full[s], 1);
        mbar_fence_init();
    }
    __syncthreads();
    // routing: the logits were written before the previous kernel (k_moe_gu) passed its own wait, so they are
    // complete here without waiting; the expert rows to stream follow from them
    route_token(a.logits + (size_t)t * a.ls, a.ne, a.k, sel, wsel, keys);
    auto issue = [&](int st) {  // thread 0: stage st = (chunk c, slot s)
        const int c = st / ks, s = st % ks, rr = r0 + c * a.rps, n = min(a.rps, r1 - rr), slot = st % a.slots;
        const uint8_t *src = s < a.k ? a.Wd + ((size_t)sel[s] * a.d + rr) * a.ldw : a.Wsd + (size_t)rr * a.ldw;
        const uint32_t bytes = (uint32_t)n * a.ldw;
        mbar_arrive_tx(&full[slot], bytes);
        bulk_g2s(ring + (size_t)slot * a.stage_bytes, src, bytes, &full[slot]);
    };
    if (tid == 0)
        for (int st = 0; st < min(nst, a.slots); ++st) issue(st);
    stage_grid<TY>(grid);
    pdl_wait();
    const float *act = after_wait(a.act);
    stage_x(xsm, act + (size_t)t * ks * a.ffe, a.ffe, ks, G, ScaleX<TY, SOA>::v);
    pdl_trigger();

    constexpr int RPW = 32 / LPR;
    const int lr = lane % LPR, sub = lane / LPR;
    const float sg = sigm(a.logits[(size_t)t * a.ls + a.ne]);
    XReg<LPR, 1> xr;
    int st = 0;
    for (; st < nst; ++st) {
        const int c = st / ks, s = st % ks, rr = r0 + c * a.rps, n = min(a.rps, r1 - rr), slot = st % a.slots;
        const bool ok = warp_wait(&full[slot], (uint32_t)(st / a.slots) & 1u);
        if (ok) {
            const uint8_t *sbuf = ring + (size_t)slot * a.stage_bytes;
            for (int base = warp * RPW * RR; base < n; base += nw * RPW * RR) {
                const uint8_t *rp[RR];
                bool valid[RR];
                int row[RR];
#pragma unroll
                for (int q = 0; q < RR; ++q) {
                    row[q] = base + q * RPW + sub;
                    valid[q] = row[q] < n;
                    rp[q] = sbuf + (size_t)(valid[q] ? row[q] : 0) * a.ldw;
                }
                double acc[RR][1];
                rows_dot<TY, SOA, 1, LPR, 0, false, RR>(rp, valid, a.nb, grid, xr, xsm + (size_t)s * G * XPAD, G, lr, 1,
                                                       acc);
                const bool hi = RR == 2 && (lane & 16);
                if ((hi ? valid[RR - 1] : valid[0]) && (RR == 2 ? (lane & 15) == 0 : lr == 0))
                    res[s * a.rps + (hi ? row[RR - 1] : row[0])] = __double2float_rn(acc[0][0]);
            }
        }
        if (__syncthreads_or(!ok)) {
            if (tid == 0) dev_fail(a.err, DEV_WAIT_TIMEOUT);
            break;
        }
        if (s == a.k) {  // chunk complete: combine in slot order, then the gated shared expert
            for (int i = tid; i < n; i += blockDim.x) {
                float m = 0.0f;
                for (int q = 0; q < a.k; ++q) m = __fmaf_rn(wsel[q], res[q * a.rps + i], m);
                const float v = __fmaf_rn(sg, res[a.k * a.rps + i], m);
                float *o = a.y + (size_t)t * a.d + rr + i;
                *o = a.acc ? *o + v : v;
            }
            __syncthreads();
        }
        if (tid == 0 && st + a.slots < nst) issue(st + a.slots);
    }
    if (st < nst && tid == 0)
        for (int s2 = st; s2 < min(nst, st + a.slots); ++s2) mbar_wait(&full[s2 % a.slots], (uint32_t)(s2 / a.slots) & 1u, 1u << 16);
}


template <uint32_t TY>
cudaError_t moe_gu_launch_t(const MoeGuArgs &a, bool planes, int nt, int G, int ctas, size_t smem, cudaStream_t s) {
    void (*k)(const MoeGuArgs) = nullptr;
    if (planes) k = nt == 1 && G == 64 ? k_moe_gu<TY, 32, 2, true, true> : k_moe_gu<TY, 32, 0, false, true>;
    else k = nt == 1 && G == 64 ? k_moe_gu<TY, 32, 2, true, false> : k_moe_gu<TY, 32, 0, false, false>;
    const cudaError_t e = allow_max_dynamic_smem(k);
    if (e != cudaSuccess) return e;
    return launch_k(k, dim3(ctas), dim3(256), smem, s, a);
}

template <uint32_t TY>
cudaError_t moe_down_launch_t(const MoeDownArgs &a, bool planes, int lpr, dim3 grid, size_t smem, cudaStream_t s) {
    void (*k)(const MoeDownArgs) = nullptr;
    if (planes) k = lpr == 16 ? k_moe_down<TY, 16, true> : k_moe_down<TY, 32, true>;
    else k = lpr == 16 ? k_moe_down<TY, 16, false> : k_moe_down<TY, 32, false>;
    const cudaError_t e = allow_max_dynamic_smem(k);
    if (e != cudaSuccess) return e;
    return launch_k(k, grid, dim3(256), smem, s, a);
}

#define FN_MOE_SIG(TY)                                                                                       \
    cudaError_t moe_gu_launch_t<TY>(const MoeGuArgs &, bool, int, int, int, size_t, cudaStream_t);            \
    template cudaError_t moe_down_launch_t<TY>(const MoeDownArgs &, bool, int, dim3, size_t, cudaStream_t);
#define FN_MOE_DECL(TY)                                                                                            \
    extern template cudaError_t moe_gu_launch_t<TY>(const MoeGuArgs &, bool, int, int, int, size_t, cudaStream_t); \
    extern template cudaError_t moe_down_launch_t<TY>(const MoeDownArgs &, bool, int, dim3, size_t, cudaStream_t);
#define FN_MOE_INST(TY) template FN_MOE_SIG(TY)

}  // namespace fn
