// Dense GEMV kernel template and its per-format launcher (instantiated in fn_gemv_i*.cu, one group of formats per
// translation unit so the build compiles them in parallel). See fn_gemv.cu for the design.
#pragma once

#include <unordered_set>

#include "fn_engine.h"
#include "fn_argmax.cuh"
#include "fn_rowdot.cuh"

namespace fn {

struct GemvArgs {
    const uint8_t *W;  // plane rows (GGUF rows for formats without a plane layout)
    uint32_t ldw;
    int rows, G, nb;
    const float *x;
    int xs;
    float *y;
    int ys, nt;
    int rps, slots;
    uint32_t stage_bytes, x_off, ring_off, grid_off;
    int acc, early;
    const uint8_t *pf;  // L2 prefetch hint (GemvPlan::pf), null: none
    uint64_t pf_bytes;
    const float *nw;  // RMSNorm folded in (GemvPlan::nw), null: none
    float eps;
    uint32_t *err;
    // fused argmax (GemvArgmax); amx == 0: none
    int amx, row0;
    int *aidx;
    unsigned long long *akey, *kacc;
    unsigned int *ticket;
    KeyExchange xr;  // xr.n == 0: no exchange
};

// Fused argmax, end of the CTA. The CTA's best key per token (a register per storing lane for one token, else
// s_best[warp][writer][t]) goes by one relaxed atomic max into kacc[t]; then a release-acquire ticket: the CTA that
// takes the last ticket sees every CTA's max, publishes the winner and clears kacc and the ticket for the next launch.
// Every thread calls this.
template <int NT>
__device__ __forceinline__ void gemv_argmax_epilogue(unsigned long long best1, const unsigned long long (*s_best)[4][NT],
                                                     const GemvArgs &a) {
    __shared__ unsigned long long s_w[16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if constexpr (NT == 1) {
        best1 = warp_kmax(best1);
        if (lane == 0) s_w[warp] = best1;
    }
    __syncthreads();
    if (warp != 0) return;
    for (int t = 0; t < a.nt; ++t) {  // warp 0: lane w takes warp w's keys
        unsigned long long k = 0;
        if (lane < nw) {
            if constexpr (NT == 1) {
                k = s_w[lane];
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) k = kmax(k, s_best[lane][i][t]);
            }
        }
        k = warp_kmax(k);
        if (lane == 0 && k) asm volatile("red.relaxed.gpu.global.max.u64 [%0], %1;" ::"l"(a.kacc + t), "l"(k) : "memory");
    }
    if (lane != 0) return;
    uint32_t tk;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(tk) : "l"(a.ticket) : "memory");
    if (tk != gridDim.x - 1) return;
    unsigned long long kt[8];
    for (int t = 0; t < a.nt; ++t) {
        asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(kt[t]) : "l"(a.kacc + t) : "memory");
        if (a.aidx) a.aidx[t] = amax_index(kt[t]);
        if (a.akey) a.akey[t] = kt[t];
        a.kacc[t] = 0ull;
    }
    *a.ticket = 0u;
    if (a.xr.n > 0) {  // row-split lm_head: keys to every rank, then one release-add on each rank's counter
        const uint32_t c = *a.xr.calls;
        *a.xr.calls = c + 1;
        const int slot = ((int)(c & 1u) * MAX_RANKS + a.xr.rank) * 8;
        for (int p = 0; p < a.xr.n; ++p)
            for (int t = 0; t < a.nt; ++t) a.xr.keys[p][slot + t] = kt[t];
        for (int p = 0; p < a.xr.n; ++p) red_release_sys_add(a.xr.counters[p] + a.xr.rank, 1u);
    }
}

template <uint32_t TY, int NT, int LPR, int GPL, bool XREG>
__global__ void __launch_bounds__(512, 1) k_gemv(const GemvArgs a) {
    constexpr int RR = LPR == 32 ? 2 : 1;  // rows per lane group per stage
    constexpr int RPW = 32 / LPR;          // lane groups per warp
    constexpr int RU = RR * RPW;           // rows per warp stage
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    uint64_t *full = (uint64_t *)sm + warp * a.slots;  // this warp's stage barriers
    uint8_t *ring = sm + a.ring_off + (size_t)warp * a.slots * a.stage_bytes;
    float *xsm = (float *)(sm + a.x_off);
    uint32_t *grid = (uint32_t *)(sm + a.grid_off);
    // the CTA's rows, split into one contiguous range per warp
    const int r0 = (int)((long long)blockIdx.x * a.rows / gridDim.x);
    const int r1 = (int)((long long)(blockIdx.x + 1) * a.rows / gridDim.x);
    const int w0 = r0 + (int)((long long)(r1 - r0) * warp / nw), w1 = r0 + (int)((long long)(r1 - r0) * (warp + 1) / nw);
    const int nst = (w1 - w0 + RU - 1) / RU;

    auto issue = [&](int st, int slot) {  // lane 0: stage st of this warp's rows into ring slot `slot`
        const int rr = w0 + st * RU, n = min(RU, w1 - rr);
        const uint32_t bytes = (uint32_t)n * a.ldw;
        mbar_arrive_tx(&full[slot], bytes);
        bulk_g2s(ring + (size_t)slot * a.stage_bytes, a.W + (size_t)rr * a.ldw, bytes, &full[slot]);
    };
    if (lane == 0) {
        for (int s = 0; s < a.slots; ++s) mbar_init(&full[s], 1);
        mbar_fence_init();
        for (int st = 0; st < min(nst, a.slots); ++st) issue(st, st);
    }
    __syncwarp();
    l2_prefetch_share(a.pf, a.pf_bytes);  // the next weights of a chain: read-only, so before any wait
    // The next kernel may launch (its CTAs stage their own weights beside this one where they fit; its
    // griddepcontrol.wait still waits for this whole grid; a dependent grid starts about 2 us after the trigger):
    // an early GEMV triggers at once, as the reference's does (engine/faie2fn.cu:920-922); any other kernel only after
    // its own wait, so that everything before it is complete when the kernel after it starts.
    if (a.early) pdl_trigger();
    stage_grid<TY>(grid);

    // fused argmax: best key per storing lane (one token: a register; else per (warp, writer, token) in shared
    // memory, cleared before stage_x's barriers)
    __shared__ unsigned long long s_best[NT == 1 ? 1 : 16][4][NT];
    float bv = -INFINITY;  // one token: the lane's best value and its row (rows rise along a lane's stages, so a
    int br = -1;           // strict > keeps the lowest row of equal values; NaN and -inf never enter)
    if (NT > 1 && a.amx)
        for (int i = tid; i < 16 * 4 * NT; i += blockDim.x) (&s_best[0][0][0])[i] = 0ull;

    if (!a.early) {
        pdl_wait();
        pdl_trigger();
    }
    const float *x = after_wait(a.x);
    const int nt = a.nt;
    stage_x(xsm, x, a.xs, nt, a.G, ScaleX<TY, true>::v, a.nw);
    // RMSNorm folded in: y = s_t (W . (x_t * nw)), s_t applied to the row result
    float ns[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) ns[t] = a.nw && (NT == 1 || t < nt) ? norm_scale(xsm, a.G, t, 32 * a.G, a.eps) : 1.0f;

    const int lr = lane % LPR, sub = lane / LPR;
    XReg<LPR, (GPL > 0 ? GPL : 1)> xr;
    if constexpr (XREG) xr.load(xsm, lr);

    // the ring position of stage st: slot = st mod slots and its phase parity, kept incrementally (no division)
    int st = 0, slot = 0;
    uint32_t phase = 0;
    for (; st < nst; ++st) {
        if (!warp_wait(&full[slot], phase)) {
            if (lane == 0) dev_fail(a.err, DEV_WAIT_TIMEOUT);
            break;
        }
        const uint8_t *sbuf = ring + (size_t)slot * a.stage_bytes;
        const int rr0 = w0 + st * RU;
        const uint8_t *rp[RR];
        bool valid[RR];
        int row[RR];
#pragma unroll
        for (int q = 0; q < RR; ++q) {
            row[q] = q * RPW + sub;
            valid[q] = rr0 + row[q] < w1;
            rp[q] = sbuf + (size_t)(valid[q] ? row[q] : 0) * a.ldw;
        }
        double acc[RR][NT];
        rows_dot<TY, true, NT, LPR, GPL, XREG, RR>(rp, valid, a.nb, grid, xr, xsm, a.G, lr, nt, acc);
        // the lane that stores a row: lane 0 / 16 of the two halves (RR == 2), else lane 0 of each lane group; after
        // the butterfly acc[0] holds that lane's row total (selects, not a dynamic register index, keep it in registers)
        const bool hi = RR == 2 && (lane & 16);
        const bool vq = hi ? valid[RR - 1] : valid[0];
        if (vq && (RR == 2 ? (lane & 15) == 0 : lr == 0)) {
            const int r = rr0 + (hi ? row[RR - 1] : row[0]);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (NT > 1 && t >= nt) break;
                float v = __double2float_rn(acc[0][t]);
                if (a.nw) v = __fmul_rn(v, ns[t]);
                if (a.y) {
                    float *o = a.y + (size_t)t * a.ys + r;
                    *o = a.acc ? __fadd_rn(*o, v) : v;
                }
                if (a.amx) {
                    if constexpr (NT == 1) {
                        if (v > bv) {
                            bv = v;
                            br = r;
                        }
                    } else {
                        unsigned long long &b = s_best[warp][lane / (LPR == 32 ? 16 : LPR)][t];
                        b = kmax(b, amax_key(v, a.row0 + r));
                    }
                }
            }
        }
        __syncwarp();  // every lane is done reading the slot
        if (lane == 0 && st + a.slots < nst) issue(st + a.slots, slot);
        if (++slot == a.slots) {
            slot = 0;
            phase ^= 1u;
        }
    }
    if (st < nst && lane == 0)  // wound down early: let the copies already issued land (bounded) before exiting
        for (int s2 = st; s2 < min(nst, st + a.slots); ++s2) mbar_wait(&full[s2 % a.slots], (uint32_t)(s2 / a.slots) & 1u, 1u << 16);
    if (a.early) pdl_wait();
    if (a.amx) gemv_argmax_epilogue<NT>(br < 0 ? 0ull : amax_key(bv, a.row0 + br), s_best, a);
}

template <uint32_t TY> cudaError_t gemv_launch_t(const GemvPlan &p, const GemvArgs &a, size_t smem, cudaStream_t s) {
    void (*k)(const GemvArgs) = nullptr;
    if (p.ntcap == 1) {
        if (p.xreg) {
            if (p.lpr == 8) k = k_gemv<TY, 1, 8, 1, true>;
            else if (p.lpr == 16) k = k_gemv<TY, 1, 16, 1, true>;
            else if (p.gpl == 1) k = k_gemv<TY, 1, 32, 1, true>;
            else k = k_gemv<TY, 1, 32, 2, true>;
        } else {
            k = k_gemv<TY, 1, 32, 0, false>;
        }
    } else {
        if (p.lpr == 8) k = k_gemv<TY, 8, 8, 0, false>;
        else if (p.lpr == 16) k = k_gemv<TY, 8, 16, 0, false>;
        else k = k_gemv<TY, 8, 32, 0, false>;
    }
    const cudaError_t e = allow_max_dynamic_smem(k);
    if (e != cudaSuccess) return e;
    return launch_k(k, dim3(p.ctas), dim3(p.threads), smem, s, a);
}


#define FN_GEMV_DECL(TY) extern template cudaError_t gemv_launch_t<TY>(const GemvPlan &, const GemvArgs &, size_t, cudaStream_t);
#define FN_GEMV_INST(TY) template cudaError_t gemv_launch_t<TY>(const GemvPlan &, const GemvArgs &, size_t, cudaStream_t);

}  // namespace fn
