// One MoE layer of one token on one GPU as a single persistent kernel: the routed experts' gate/up rows, then their
// down rows and the slot-order combine, with the hand-off between the two through per-slot counters in global memory
// instead of a kernel boundary. This is the reference's stated next lever (a per-pair counter so that the down
// projection of pair p starts once pair p's gate/up blocks are done; its kernels engine/faie2fn.cu:1082-1184).
//
// Grid: one CTA per SM, 16 warps. CTA b owns (a) an even share of the (k + 1) * ffe gate/up units (slot, row), one
// contiguous run per warp, as k_moe_gu, and (b) output rows [b d / grid, (b + 1) d / grid) of the down projection for
// all k + 1 slots, as k_moe_down. After the routing is read (k_moe_route, the kernel before), every CTA issues the
// bulk copies of ALL its weights at once: its gate/up rows (one region per warp, at most two runs) and its down rows
// (one copy per slot), so the down weights stream while the gate/up rows are computed, where the two-kernel form
// cannot start them until the gate/up kernel's CTAs leave the SMs. A warp's finished units are published by a
// release add of their count on their slot's counter (lane 0 wrote them); the down phase waits (acquire, bounded)
// until every slot counts ffe rows, stages the activations through L2 and computes exactly as k_moe_down does, so the
// layer's output is bit-identical to the two-kernel form. All CTAs of the grid are resident at once (one per SM, no
// CTA waits on a CTA that started after it), so the waits end; they are bounded all the same (about a second, then
// an error word). The CTA that takes the last ticket zeroes the counters for the layer's next launch.
#pragma once

#include "fn_moe_impl.cuh"

namespace fn {

struct MoeFusedArgs {
    const uint8_t *Wg, *Wu, *Wsg, *Wsu;  // gate / up: routed (ne * ffe rows) and shared (ffe rows), stride ldw_g
    uint32_t ldw_g;
    int nb_g;
    const uint8_t *Wd, *Wsd;  // down: routed (ne * d rows) and shared (d rows), stride ldw_d
    uint32_t ldw_d;
    int nb_d;
    int ne, k, ffe, d;
    const float *logits;  // [ls]: column ne is the shared-gate logit
    int ls;
    const float *x;  // [d]
    float *act;      // [k + 1][ffe], global scratch
    float *y;
    int acc;
    const int *rsel;  // routing (k_moe_route, the kernel before this one)
    const float *rw;
    uint32_t *cnt;  // [0, 16): rows published per slot; [16]: ticket. Zero between launches.
    int x_early;
    const float *nw;  // RMSNorm folded in (MoePlan::nw), null: none
    float eps;
    int upw;   // gate/up units per warp at most (<= ffe)
    int rows;  // down rows per CTA at most
    uint32_t gu_off, dw_off, res_off, grid_off, xs_off, as_off;
    uint32_t *err;
    const uint8_t *pf;  // L2 prefetch hint, null: none
    uint64_t pf_bytes;
};

// Bounded wait until the 32-bit counter at p (this GPU's memory) reaches target, with acquire loads at GPU scope.
__device__ __forceinline__ bool wait_counter_gpu(const uint32_t *p, uint32_t target, uint32_t limit = 1u << 22) {
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if (v >= target) return true;
        __nanosleep(64);
    }
    return false;
}
__device__ __forceinline__ void red_release_gpu_add(uint32_t *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

constexpr int FUSED_WARPS = MOE_THREADS / 32;

template <uint32_t TG, uint32_t TD, int XG, int LPR>
__global__ void __launch_bounds__(MOE_THREADS, 1) k_moe_fused(const MoeFusedArgs a) {
    static_assert(Gguf<TD>::gridw == 0, "the fused layer stages one codebook, the gate/up format's");
    constexpr int RR = LPR == 32 ? 2 : 1, RPW = 32 / LPR, RU = RR * RPW;
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    uint64_t *gbar = (uint64_t *)sm;             // [warp][2]: a warp's gate/up runs have landed
    uint64_t *dbar = gbar + 2 * FUSED_WARPS;      // [slot]: the slot's down rows have landed
    uint8_t *gu = sm + a.gu_off + (size_t)warp * a.upw * 2 * a.ldw_g;
    uint8_t *dw = sm + a.dw_off;
    float *res = (float *)(sm + a.res_off);  // [k + 1][rows]
    uint32_t *grid = (uint32_t *)(sm + a.grid_off);
    float *xsm = (float *)(sm + a.xs_off);   // x staged (XG == 0)
    float *asg = (float *)(sm + a.as_off);   // the activations staged for the down rows
    __shared__ int sel[16];
    __shared__ float wsel[16];
    __shared__ int s_fail;
    const int ks = a.k + 1, G = a.d / 32, Gd = a.ffe / 32;
    const int r0 = (int)((long long)blockIdx.x * a.d / gridDim.x), r1 = (int)((long long)(blockIdx.x + 1) * a.d / gridDim.x);
    const int n = r1 - r0;

    if (tid == 0) {
        for (int i = 0; i < 2 * FUSED_WARPS + ks; ++i) mbar_init(&gbar[i], 1);
        mbar_fence_init();
        s_fail = 0;
    }
    stage_grid<TG>(grid);
    l2_prefetch_share(a.pf, a.pf_bytes);  // the next weights of a chain: read-only, so before the wait
    XReg<32, (XG > 0 ? XG : 1)> xr;
    float xscale = 1.0f;
    if constexpr (XG > 0)
        if (a.x_early) xscale = xr.load_global(a.x, lane, ScaleX<TG, true>::v, a.nw, a.eps);  // beside the routing kernel
    pdl_wait();
    pdl_trigger();
    if (tid < a.k) {
        sel[tid] = after_wait(a.rsel)[tid];
        wsel[tid] = after_wait(a.rw)[tid];
    }
    __syncthreads();  // the routing and the barriers' initialisation, before any copy

    // this warp's gate/up units [w0, w1): at most two runs (contiguous rows of one slot), run 0 [w0, e0)
    const int U = ks * a.ffe;
    const int u0 = (int)((long long)blockIdx.x * U / gridDim.x), u1 = (int)((long long)(blockIdx.x + 1) * U / gridDim.x);
    const int w0 = u0 + (u1 - u0) * warp / nw, w1 = u0 + (u1 - u0) * (warp + 1) / nw;
    const int e0 = min(w1, (w0 / a.ffe + 1) * a.ffe);
    const int nrun[2] = {e0 - w0, w1 - e0};
    const size_t wslot = (size_t)a.rows * a.ldw_d;
    if (lane == 0) {
        // gate/up first (needed first): run j's gate rows, then its up rows, at 2 * (units before it) rows
        for (int j = 0, st = w0, off = 0; j < 2; ++j) {
            const int m = nrun[j];
            if (m > 0) {
                const int q = st / a.ffe, r = st - q * a.ffe;
                const size_t src = q < a.k ? ((size_t)sel[q] * a.ffe + r) * a.ldw_g : (size_t)r * a.ldw_g;
                const uint32_t bytes = (uint32_t)m * a.ldw_g;
                mbar_arrive_tx(&gbar[2 * warp + j], 2 * bytes);
                bulk_g2s(gu + (size_t)off * a.ldw_g, (q < a.k ? a.Wg : a.Wsg) + src, bytes, &gbar[2 * warp + j]);
                bulk_g2s(gu + (size_t)(off + m) * a.ldw_g, (q < a.k ? a.Wu : a.Wsu) + src, bytes, &gbar[2 * warp + j]);
            }
            st += m;
            off += 2 * m;
        }
        // then the down rows [r0, r1) of the slots this warp issues (slot q by warp q mod nw)
        for (int q = warp; q < ks; q += nw) {
            const uint8_t *src = q < a.k ? a.Wd + ((size_t)sel[q] * a.d + r0) * a.ldw_d : a.Wsd + (size_t)r0 * a.ldw_d;
            mbar_arrive_tx(&dbar[q], (uint32_t)(n * a.ldw_d));
            bulk_g2s(dw + q * wslot, src, (uint32_t)(n * a.ldw_d), &dbar[q]);
        }
    }
    const float *x = after_wait(a.x);
    if constexpr (XG > 0) {
        if (!a.x_early) xscale = xr.load_global(x, lane, ScaleX<TG, true>::v, a.nw, a.eps);
        __syncwarp();
    } else {
        stage_x(xsm, x, a.d, 1, G, ScaleX<TG, true>::v, a.nw);  // ends with a __syncthreads
        if (a.nw) xscale = norm_scale(xsm, G, 0, a.d, a.eps);
    }

    // ---- gate / up: k_moe_gu's arithmetic for each unit; lane 0 stores act and publishes each run's count
    bool ok = true;
    for (int j = 0, st = w0, off = 0; j < 2; ++j) {
        const int m = nrun[j];
        if (m > 0 && ok) {
            if (!warp_wait(&gbar[2 * warp + j], 0u)) {
                ok = false;
            } else {
                const int q = st / a.ffe;
                for (int i = 0; i < m; ++i) {
                    const int r = st + i - q * a.ffe;
                    const uint8_t *gp = gu + (size_t)(off + i) * a.ldw_g, *up = gu + (size_t)(off + m + i) * a.ldw_g;
                    double accg = 0.0, accu = 0.0;
                    if constexpr (XG > 0) {
#pragma unroll
                        for (int ii = 0; ii < XG; ++ii) {
                            const int g = lane + 32 * ii;
                            const XRegA xa{xr.v[ii], xr.s[ii], xr.iv};
                            float rg[1], ru[1];
                            group_dot<TG, true, 1>(gp, a.nb_g, g, grid, xa, 1, rg);
                            group_dot<TG, true, 1>(up, a.nb_g, g, grid, xa, 1, ru);
                            accg += (double)rg[0];
                            accu += (double)ru[0];
                        }
                    } else {
#pragma unroll 1
                        for (int ii = 0; ii < (G + 31) / 32; ++ii) {
                            const int g = lane + 32 * ii;
                            if (g >= G) break;
                            XReg<32, 1> xg;
                            xg.load(xsm, g);
                            const XRegA xa{xg.v[0], xg.s[0], xg.iv};
                            float rg[1], ru[1];
                            group_dot<TG, true, 1>(gp, a.nb_g, g, grid, xa, 1, rg);
                            group_dot<TG, true, 1>(up, a.nb_g, g, grid, xa, 1, ru);
                            accg += (double)rg[0];
                            accu += (double)ru[0];
                        }
                    }
                    const bool uh = lane & 16;
                    double keep = uh ? accu : accg;
                    keep += __shfl_xor_sync(0xffffffffu, uh ? accg : accu, 16);
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
                    float v = __double2float_rn(keep);
                    if (a.nw) v = __fmul_rn(v, xscale);
                    const float u = __shfl_sync(0xffffffffu, v, 16);
                    if (lane == 0) a.act[(size_t)q * a.ffe + r] = silu(v) * u;
                }
                if (lane == 0) red_release_gpu_add(a.cnt + q, (uint32_t)m);  // after this lane's act stores of the run
            }
        }
        st += m;
        off += 2 * m;
    }
    if (!ok && lane == 0) s_fail = 1;

    // ---- down: every slot's ffe rows published (slot q polled by thread q), then k_moe_down's arithmetic
    if (tid < ks && !wait_counter_gpu(a.cnt + tid, (uint32_t)a.ffe)) s_fail = 1;
    __syncthreads();
    if (!s_fail) {
        stage_x(asg, a.act, a.ffe, ks, Gd, ScaleX<TD, true>::v, nullptr, true);  // through L2; ends with a barrier
        const int lr = lane % LPR, sub = lane / LPR;
        XReg<LPR, 1> xrd;
        const int npg = (n + RU - 1) / RU;
        for (int u = warp; u < ks * npg; u += nw) {
            const int q = u / npg, pg = u % npg;
            if (!warp_wait(&dbar[q], 0u)) {
                if (lane == 0) s_fail = 1;
                break;
            }
            const uint8_t *rp[RR];
            bool valid[RR];
            int row[RR];
#pragma unroll
            for (int h = 0; h < RR; ++h) {
                row[h] = pg * RU + h * RPW + sub;
                valid[h] = row[h] < n;
                rp[h] = dw + q * wslot + (size_t)(valid[h] ? row[h] : 0) * a.ldw_d;
            }
            double acc[RR][1];
            rows_dot<TD, true, 1, LPR, 0, false, RR>(rp, valid, a.nb_d, nullptr, xrd, asg + (size_t)q * Gd * XPAD, Gd, lr,
                                                     1, acc);
            const bool hi = RR == 2 && (lane & 16);
            if ((hi ? valid[RR - 1] : valid[0]) && (RR == 2 ? (lane & 15) == 0 : lr == 0))
                res[q * a.rows + (hi ? row[RR - 1] : row[0])] = __double2float_rn(acc[0][0]);
        }
    }
    __syncthreads();
    if (s_fail) {  // a copy never landed or a slot never completed: record it, let this CTA's copies land (bounded)
        if (tid == 0) {
            dev_fail(a.err, DEV_WAIT_TIMEOUT);
            for (int q = 0; q < ks; ++q) mbar_wait(&dbar[q], 0u, 1u << 16);
        }
        if (lane == 0)
            for (int j = 0; j < 2; ++j)
                if (nrun[j] > 0) mbar_wait(&gbar[2 * warp + j], 0u, 1u << 16);
    } else {  // combine in slot order, then the gated shared expert (k_moe_down's FMAs, in its order)
        const float sg = sigm(a.logits[a.ne]);
        for (int i = tid; i < n; i += blockDim.x) {
            float s = 0.0f;
            for (int q = 0; q < a.k; ++q) s = __fmaf_rn(wsel[q], res[q * a.rows + i], s);
            const float v = __fmaf_rn(sg, res[a.k * a.rows + i], s);
            float *o = a.y + r0 + i;
            *o = a.acc ? *o + v : v;
        }
    }
    // every CTA has finished polling once it takes a ticket: the last one zeroes the counters for the next launch
    __syncthreads();
    if (tid == 0) {
        uint32_t tk;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(tk) : "l"(a.cnt + 16) : "memory");
        if (tk == gridDim.x - 1) {
            for (int q = 0; q < 17; ++q) a.cnt[q] = 0u;
        }
    }
}

template <uint32_t TG, uint32_t TD>
cudaError_t moe_fused_launch_t(const MoeFusedArgs &a, int G, int lpr, int ctas, size_t smem, cudaStream_t s) {
    void (*k)(const MoeFusedArgs) = nullptr;
    if (G == 64) k = lpr == 4 ? k_moe_fused<TG, TD, 2, 4> : k_moe_fused<TG, TD, 2, 8>;
    else if (G == 32) k = lpr == 4 ? k_moe_fused<TG, TD, 1, 4> : k_moe_fused<TG, TD, 1, 8>;
    else k = lpr == 4 ? k_moe_fused<TG, TD, 0, 4> : k_moe_fused<TG, TD, 0, 8>;
    const cudaError_t e = allow_max_dynamic_smem(k);
    if (e != cudaSuccess) return e;
    return launch_k(k, dim3(ctas), dim3(MOE_THREADS), smem, s, a);
}

}  // namespace fn
