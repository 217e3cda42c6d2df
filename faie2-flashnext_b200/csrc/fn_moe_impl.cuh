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
//
// Order (the reference's k_route, engine/faie2fn.cu:1742-1800): m = the largest logit, v_i = expf(l_i - m) in fp32,
// larger v first, equal v to the lower expert index. Distinct logits can share one v (l - m rounds to the same float,
// or expf saturates at 0 or 1); the lower index then wins, as in the reference. The order is a 64-bit key: v's bits
// (v >= +0, so they order as unsigned integers) above the complemented index, so every key is distinct. 16 warps each
// sort their 32 E keys (a bitonic network in registers); a candidate's merged rank is the number of larger keys in
// the 16 sorted lists, and rank r < k is slot r.

__device__ __forceinline__ unsigned long long prob_key(float v, int idx) {
    return ((unsigned long long)__float_as_uint(v) << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ int key_index(unsigned long long k) { return (int)(0xFFFFFFFFu - (uint32_t)k); }
__device__ __forceinline__ float key_prob(unsigned long long k) { return __uint_as_float((uint32_t)(k >> 32)); }

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
                    v[e] = desc == lower ? (v[e] > o ? v[e] : o) : (v[e] < o ? v[e] : o);
                }
            } else {
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const int p = e ^ j;
                    if (p > e) {
                        const bool desc = ((lane * E + e) & size) == 0;
                        const unsigned long long x = v[e], y = v[p];
                        const bool sw = desc ? x < y : x > y;
                        v[e] = sw ? y : x;
                        v[p] = sw ? x : y;
                    }
                }
            }
        }
    }
}

constexpr int ROUTE_THREADS = 512;  // 16 warps

// Each warp's k best keys of logits[0, ne) (warp w holds experts [32 E w, 32 E (w + 1))), zero-padded to 16, into
// keys[w * 16 ..]. red: 16 floats for the block maximum.
template <int E>
__device__ __forceinline__ void route_warp_best(const float *logits, int ne, int k, unsigned long long *keys,
                                                float *red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float l[E];
    float m = -INFINITY;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int i = warp * 32 * E + lane * E + e;
        l[e] = i < ne ? logits[i] : -INFINITY;
        m = fmaxf(m, l[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int w2 = 1; w2 < 16; ++w2) m = fmaxf(m, red[w2]);
    unsigned long long v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int i = warp * 32 * E + lane * E + e;
        v[e] = i < ne ? prob_key(expf(l[e] - m), i) : 0ull;
    }
    warp_sort_desc<E>(v, lane);
#pragma unroll
    for (int e = 0; e < E; ++e)
        if (lane * E + e < 16) keys[warp * 16 + lane * E + e] = lane * E + e < k ? v[e] : 0ull;
}

// Route one token: the k best of logits[0, ne) into sel[k], w[k] (shared memory), with the reference's weights
// w_r = v_r / s, s = sum_r v_r in rank order (fp32, from 0). Every thread of a 512-thread block calls it; ne <= 1024,
// k <= 16. keys: 16 * 16 entries, vals: 16 floats of shared memory.
static __device__ __noinline__ void route_token(const float *logits, int ne, int k, int *sel, float *w,
                                                unsigned long long *keys, float *vals) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (ne <= 512) route_warp_best<1>(logits, ne, k, keys, vals);
    else route_warp_best<2>(logits, ne, k, keys, vals);
    __syncthreads();
    // candidate c = warp c / k's rank c % k: its merged rank = the number of larger keys in all 16 lists (the keys are
    // distinct); the k best go to sel in rank order, with their v
    const int c = threadIdx.x, wc = c / k;
    if (wc < 16) {
        const unsigned long long key = keys[wc * 16 + (c - wc * k)];
        int rank = 0;
#pragma unroll 4
        for (int w2 = 0; w2 < 16; ++w2) {
            const ulonglong2 *row = (const ulonglong2 *)(keys + w2 * 16);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const ulonglong2 q = row[j];
                rank += (q.x > key) + (q.y > key);
            }
        }
        if (rank < k && key != 0ull) {
            sel[rank] = key_index(key);
            vals[rank] = key_prob(key);
        }
    }
    __syncthreads();
    if (warp == 0) {
        const float ev = lane < k ? vals[lane] : 0.0f;
        float s = 0.0f;
        for (int r = 0; r < k; ++r) s += __shfl_sync(0xffffffffu, ev, r);
        if (lane < k) w[lane] = ev / s;
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------------------------------------------
// expert parallelism: which of a token's k + 1 slots this rank computes

// the rank holding expert e when ne experts are split over n ranks as [g ne / n, (g + 1) ne / n)
__device__ __forceinline__ int expert_owner(int e, int ne, int n) {
    int g = n - 1;
    while (g > 0 && (int)((long long)g * ne / n) > e) --g;
    return g;
}

// bit s set: this rank computes slot s of the token routed to sel[0..k) (slot k: the shared expert, computed by the
// rank holding the fewest of the routed slots, the lowest such rank). One GPU (ep.n == 0): every slot.
__device__ __forceinline__ uint32_t owned_slots(const int *sel, int k, int ne, const MoeEp &ep) {
    if (ep.n == 0) return (2u << k) - 1u;
    uint32_t m = 0;
    int cnt[MAX_RANKS];
    for (int g = 0; g < MAX_RANKS; ++g) cnt[g] = 0;
    for (int s = 0; s < k; ++s) {
        const int g = expert_owner(sel[s], ne, ep.n);
        ++cnt[g];
        if (g == ep.rank) m |= 1u << s;
    }
    int best = 0;
    for (int g = 1; g < ep.n; ++g)
        if (cnt[g] < cnt[best]) best = g;
    if (best == ep.rank) m |= 1u << k;
    return m;
}

// ---------------------------------------------------------------------------------------------------------------
// gate / up

constexpr int MOE_THREADS = 512;  // 16 warps per CTA, one CTA per SM

struct MoeGuArgs {
    const uint8_t *Wg, *Wu, *Wsg, *Wsu;  // routed (local experts * ffe rows) and shared (ffe rows), stride ldw
    uint32_t ldw;
    int nb;  // blocks per row
    int ne, k, ffe, d, nt;
    const float *logits;
    int ls;  // logits token stride (>= ne + 1: column ne is the shared-gate logit)
    const float *x;  // [nt][d]
    float *act;      // [nt][k + 1][ffe]
    const int *rsel;  // routing [nt][16] (k_moe_route, the kernel before this one), unless route_self
    int route_self;   // every CTA routes the tokens itself from the logits (no routing kernel before this one)
    int x_early;      // x was complete before the kernel before this one started: read it before the wait
    const float *nw;  // RMSNorm folded in (MoePlan::nw), null: none
    float eps;
    int slots;  // ring stages per warp
    int run;    // units per stage at most: `run` consecutive gate rows of one expert, then the matching up rows
    uint32_t stage_bytes, ring_off, x_off, grid_off, misc_off;
    uint32_t *err;
    MoeEp ep;
};

// Units are the (token, slot, row) triples this rank computes, in (pair, row) order; CTA b takes an even share and
// splits it into one contiguous run per warp. Each warp streams its units through its own ring of bulk copies (no
// block barrier after the staging). A lane takes groups lane, lane + 32, .. of both rows of a unit (gate and up) in
// one loop with a single decode body (the kernel runs once per layer: short code keeps instruction fetch off the
// critical path); the two rows meet in one transposed butterfly, lane 0 writes act = silu(g) * u.
// XG > 0: rows of G = 32 XG groups; each warp holds one token's x in registers (read from global memory by the warp,
// no staging barrier), reloading it when its units move to the next token; XG == 0: x staged in shared memory for
// any row length.
template <uint32_t TY, bool SOA, int XG>
__global__ void __launch_bounds__(MOE_THREADS, 1) k_moe_gu(const MoeGuArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    uint64_t *full = (uint64_t *)sm + warp * a.slots;
    uint8_t *ring = sm + a.ring_off + (size_t)warp * a.slots * a.stage_bytes;
    float *xsm = (float *)(sm + a.x_off);
    uint32_t *grid = (uint32_t *)(sm + a.grid_off);
    int *sel = (int *)(sm + a.misc_off);  // [nt][16]
    __shared__ int s_pair[MOE_MAXT * 17];  // the (token, slot) pairs this rank computes, t << 5 | s, in order
    __shared__ int s_np;
    const int G = a.d / 32, ks = a.k + 1;

    if (lane == 0) {
        for (int q = 0; q < a.slots; ++q) mbar_init(&full[q], 1);
        mbar_fence_init();
    }
    stage_grid<TY>(grid);
    XReg<32, (XG > 0 ? XG : 1)> xr;
    float xscale = 1.0f;  // RMSNorm scale of the token whose x the warp holds (1 without a folded norm)
    if constexpr (XG > 0)
        if (a.x_early) xscale = xr.load_global(a.x, lane, ScaleX<TY, SOA>::v, a.nw, a.eps);  // beside the kernel before
    pdl_wait();
    pdl_trigger();  // after the wait: the down kernel may rely on the router's logits being complete when it starts
    const float *x = after_wait(a.x);
    if (a.route_self) {
        // every CTA routes the tokens itself (no routing kernel, one launch fewer per layer); the scratch is the start
        // of the ring, which no copy has reached yet (the copies need the routing)
        unsigned long long *keys = (unsigned long long *)(sm + a.ring_off);
        float *vals = (float *)(keys + 256), *rw = vals + 16;
        int *rs = (int *)(rw + 16);
        const float *lg = after_wait(a.logits);
        for (int t = 0; t < a.nt; ++t) {
            route_token(lg + (size_t)t * a.ls, a.ne, a.k, rs, rw, keys, vals);
            if (tid < 16) sel[t * 16 + tid] = tid < a.k ? rs[tid] : 0;
        }
        __syncthreads();
    }
    if (warp == 0) {  // the routing and this rank's (token, slot) pairs, then one block barrier
        if (!a.route_self) {
            const int *rsel = after_wait(a.rsel);
            for (int i = lane; i < a.nt * 16; i += 32) sel[i] = rsel[i];
        }
        __syncwarp();
        if (lane == 0) {
            int np = 0;
            for (int t = 0; t < a.nt; ++t) {
                const uint32_t m = owned_slots(sel + t * 16, a.k, a.ne, a.ep);
                for (int q = 0; q < ks; ++q)
                    if (m >> q & 1u) s_pair[np++] = t << 5 | q;
            }
            s_np = np;
        }
    }
    __syncthreads();

    // (32-bit unit arithmetic: U <= 8 tokens * 17 slots * ffe)
    const int U = s_np * a.ffe;
    const int u0 = (int)((long long)blockIdx.x * U / gridDim.x), u1 = (int)((long long)(blockIdx.x + 1) * U / gridDim.x);
    const int w0 = u0 + (u1 - u0) * warp / nw, w1 = u0 + (u1 - u0) * (warp + 1) / nw;
    // stages: runs of at most `run` consecutive units of one pair (contiguous rows of one expert)
    auto run_end = [&](int u) { return min(min(u + a.run, w1), (u / a.ffe + 1) * a.ffe); };
    int nst = 0;
    for (int u = w0; u < w1; u = run_end(u)) ++nst;
    auto unit = [&](int u, int &t, int &q, int &r) {
        const int pi = u / a.ffe;
        const int pr = s_pair[pi];
        t = pr >> 5;
        q = pr & 31;
        r = u - pi * a.ffe;
    };
    const size_t up_off = (size_t)a.run * a.ldw;  // the up rows' place in a stage
    int u_issue = w0, n_issued = 0, issue_slot = 0;
    auto issue = [&]() {  // lane 0: the next run of this warp into its ring slot: n gate rows, then the n up rows
        const int e1 = run_end(u_issue), n = e1 - u_issue;
        int t, q, r;
        unit(u_issue, t, q, r);
        const uint8_t *g, *up;
        if (q < a.k) {
            const size_t off = ((size_t)(sel[t * 16 + q] - a.ep.e0) * a.ffe + r) * a.ldw;
            g = a.Wg + off;
            up = a.Wu + off;
        } else {
            g = a.Wsg + (size_t)r * a.ldw;
            up = a.Wsu + (size_t)r * a.ldw;
        }
        const int slot = issue_slot;
        issue_slot = issue_slot + 1 == a.slots ? 0 : issue_slot + 1;
        uint8_t *dst = ring + (size_t)slot * a.stage_bytes;
        mbar_arrive_tx(&full[slot], 2u * (uint32_t)n * a.ldw);
        bulk_g2s(dst, g, (uint32_t)n * a.ldw, &full[slot]);
        bulk_g2s(dst + up_off, up, (uint32_t)n * a.ldw, &full[slot]);
        u_issue = e1;
        ++n_issued;
    };
    if (lane == 0)  // the weight copies fly while x is staged
        while (n_issued < min(nst, a.slots)) issue();
    int x_tok = 0;  // the token whose x the warp holds in registers (XG > 0) or whose norm scale it holds (token 0)
    if constexpr (XG > 0) {
        if (!a.x_early) xscale = xr.load_global(x, lane, ScaleX<TY, SOA>::v, a.nw, a.eps);
        __syncwarp();
    } else {
        stage_x(xsm, x, a.d, a.nt, G, ScaleX<TY, SOA>::v, a.nw);  // ends with a __syncthreads
        if (a.nw) xscale = norm_scale(xsm, G, 0, a.d, a.eps);
    }

    const int ni = (G + 31) / 32;
    int st = 0, u_cons = w0, slot = 0;
    uint32_t phase = 0;  // ring position kept incrementally (no division per stage)
    for (; st < nst; ++st) {
        if (!warp_wait(&full[slot], phase)) {
            if (lane == 0) dev_fail(a.err, DEV_WAIT_TIMEOUT);
            break;
        }
        const int e1 = run_end(u_cons);
        for (int u = u_cons; u < e1; ++u) {
        int t, q, r;
        unit(u, t, q, r);
        const uint8_t *sbuf = ring + (size_t)slot * a.stage_bytes + (size_t)(u - u_cons) * a.ldw;
        const float *xt = xsm + (size_t)t * G * XPAD;
        double accg = 0.0, accu = 0.0;  // group sums of the gate and the up row, in group order
        if constexpr (XG > 0) {
            // several tokens: a warp's units run in (token, slot, row) order, so it reloads x at most once per token
            if (t != x_tok) {
                xscale = xr.load_global(x + (size_t)t * a.d, lane, ScaleX<TY, SOA>::v, a.nw, a.eps);
                x_tok = t;
            }
#pragma unroll
            for (int i = 0; i < XG; ++i) {
                const int g = lane + 32 * i;
                const XRegA xa{xr.v[i], xr.s[i], xr.iv};
                float rg[1], ru[1];
                group_dot<TY, SOA, 1>(sbuf, a.nb, g, grid, xa, 1, rg);
                group_dot<TY, SOA, 1>(sbuf + up_off, a.nb, g, grid, xa, 1, ru);
                accg += (double)rg[0];
                accu += (double)ru[0];
            }
        } else {
            if (a.nw && t != x_tok) {
                xscale = norm_scale(xsm, G, t, a.d, a.eps);
                x_tok = t;
            }
#pragma unroll 1
            for (int i = 0; i < ni; ++i) {
                const int g = lane + 32 * i;
                if (g >= G) break;
                XReg<32, 1> xg;  // group g of x in registers, shared by the two rows
                xg.load(xt, g);
                const XRegA xa{xg.v[0], xg.s[0], xg.iv};
                float rg[1], ru[1];
                group_dot<TY, SOA, 1>(sbuf, a.nb, g, grid, xa, 1, rg);
                group_dot<TY, SOA, 1>(sbuf + up_off, a.nb, g, grid, xa, 1, ru);
                accg += (double)rg[0];
                accu += (double)ru[0];
            }
        }
        // lanes 0-15 keep the gate row, 16-31 the up row (the halves' exchange adds the same pairs as a full butterfly)
        const bool uh = lane & 16;
        double keep = uh ? accu : accg;
        keep += __shfl_xor_sync(0xffffffffu, uh ? accg : accu, 16);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
        float v = __double2float_rn(keep);  // lanes 0-15: the gate row, 16-31: the up row
        if (a.nw) v = __fmul_rn(v, xscale);  // the folded RMSNorm's scale, on both rows
        const float up = __shfl_sync(0xffffffffu, v, 16);
        if (lane == 0) a.act[((size_t)t * ks + q) * a.ffe + r] = silu(v) * up;
        }
        u_cons = e1;
        __syncwarp();  // every lane is done reading the slot
        if (lane == 0 && n_issued < nst) issue();
        if (++slot == a.slots) {
            slot = 0;
            phase ^= 1u;
        }
    }
    if (st < nst && lane == 0)  // wound down early: let the copies already issued land (bounded) before exiting
        for (int s2 = st; s2 < n_issued; ++s2) mbar_wait(&full[s2 % a.slots], (uint32_t)(s2 / a.slots) & 1u, 1u << 16);
}

// ---------------------------------------------------------------------------------------------------------------
// down + shared expert + combine

struct MoeDownArgs {
    const uint8_t *Wd, *Wsd;  // routed (local experts * d rows) and shared (d rows), ffe columns, stride ldw
    uint32_t ldw;
    int nb;
    int ne, k, ffe, d, nt;
    const float *logits;
    int ls;
    const float *act;  // [nt][k + 1][ffe]
    float *y;          // [nt][d]
    int acc;
    const int *rsel;   // routing [nt][16] and its weights (k_moe_route, two kernels back), unless route_self
    const float *rw;
    int route_self;    // each CTA routes its token itself from the logits (before its wait)
    int *sel_out;      // route_self: the routing [nt][k] (nullable), written by the token's first CTA
    float *w_out;
    int rows;  // rows per CTA at most (gridDim.x chunks of d)
    uint32_t w_off, x_off, grid_off, res_off, misc_off;
    uint32_t *err;
    MoeEp ep;
    const uint8_t *pf;  // L2 prefetch hint (MoePlan::pf), null: none
    uint64_t pf_bytes;
};

// CTA (chunk, t) owns output rows [r0, r1) of token t. Before griddepcontrol.wait it routes token t and issues one
// bulk copy per computed slot (that slot's rows [r0, r1), all in shared memory at once, one mbarrier each), so its
// weight stream overlaps the gate/up kernel. After the wait the warps take (slot, row group) units independently;
// one barrier, then the slot-order combine (or, expert parallel, the stores of this rank's slot outputs).
template <uint32_t TY, int LPR, bool SOA>
__global__ void __launch_bounds__(MOE_THREADS, 1) k_moe_down(const MoeDownArgs a) {
    constexpr int RR = LPR == 32 ? 2 : 1, RPW = 32 / LPR, RU = RR * RPW;
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t *bars = (uint64_t *)sm;  // [17]
    uint8_t *wbuf = sm + a.w_off;
    float *xsm = (float *)(sm + a.x_off);
    uint32_t *grid = (uint32_t *)(sm + a.grid_off);
    float *res = (float *)(sm + a.res_off);  // [k + 1][rows]
    __shared__ int sel[16];
    __shared__ float wsel[16];
    __shared__ int s_fail;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const int t = blockIdx.y, G = a.ffe / 32, ks = a.k + 1;
    const int r0 = (int)((long long)blockIdx.x * a.d / gridDim.x), r1 = (int)((long long)(blockIdx.x + 1) * a.d / gridDim.x);
    const int n = r1 - r0;
    // the routing (k_moe_route's output, or the logits of the router GEMV) was complete before the previous kernel
    // (k_moe_gu) passed its own wait, so it is complete here without waiting; the expert rows to stream follow from it
    if (a.route_self) {  // route the token here (the same function and logits as the gate/up kernel: the same result)
        route_token(a.logits + (size_t)t * a.ls, a.ne, a.k, sel, wsel, (unsigned long long *)xsm, xsm + 512);
        if (blockIdx.x == 0 && a.sel_out && tid < a.k) {
            a.sel_out[t * a.k + tid] = sel[tid];
            a.w_out[t * a.k + tid] = wsel[tid];
        }
    } else {
        if (tid < a.k) {
            sel[tid] = a.rsel[t * 16 + tid];
            wsel[tid] = a.rw[t * 16 + tid];
        }
        __syncthreads();
    }
    const uint32_t own = owned_slots(sel, a.k, a.ne, a.ep);
    const int m = __popc(own);
    auto slot_at = [&](int j) {  // the j-th (from 0) set bit of own
        uint32_t mm = own;
        for (int i = 0; i < j; ++i) mm &= mm - 1u;
        return __ffs(mm) - 1;
    };
    const size_t wslot = (size_t)a.rows * a.ldw;  // bytes of one slot's rows
    if (tid == 0) s_fail = 0;
    for (int j = warp; j < m; j += nw)  // one copy per slot, issued by different warps at once
        if (lane == 0) {
            const int q = slot_at(j);
            const uint8_t *src = q < a.k ? a.Wd + ((size_t)(sel[q] - a.ep.e0) * a.d + r0) * a.ldw : a.Wsd + (size_t)r0 * a.ldw;
            mbar_init(&bars[j], 1);
            mbar_fence_init();
            mbar_arrive_tx(&bars[j], (uint32_t)(n * a.ldw));
            bulk_g2s(wbuf + j * wslot, src, (uint32_t)(n * a.ldw), &bars[j]);
        }
    stage_grid<TY>(grid);
    l2_prefetch_share(a.pf, a.pf_bytes);  // the next weights of a chain: read-only, so before the wait
    pdl_wait();
    pdl_trigger();
    const float *act = after_wait(a.act);
    const int par = a.ep.n ? (int)(*after_wait(a.ep.calls) & 1u) : 0;  // expert parallel: this call's output parity
    stage_x(xsm, act + (size_t)t * ks * a.ffe, a.ffe, ks, G, ScaleX<TY, SOA>::v);  // ends with a __syncthreads

    const int lr = lane % LPR, sub = lane / LPR;
    XReg<LPR, 1> xr;
    const int npg = (n + RU - 1) / RU;
    for (int u = warp; u < m * npg; u += nw) {
        const int j = u / npg, pg = u % npg, q = slot_at(j);
        if (!warp_wait(&bars[j], 0u)) {
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
            rp[h] = wbuf + j * wslot + (size_t)(valid[h] ? row[h] : 0) * a.ldw;
        }
        double acc[RR][1];
        rows_dot<TY, SOA, 1, LPR, 0, false, RR>(rp, valid, a.nb, grid, xr, xsm + (size_t)q * G * XPAD, G, lr, 1, acc);
        const bool hi = RR == 2 && (lane & 16);  // selects keep valid / row / acc in registers
        if ((hi ? valid[RR - 1] : valid[0]) && (RR == 2 ? (lane & 15) == 0 : lr == 0))
            res[q * a.rows + (hi ? row[RR - 1] : row[0])] = __double2float_rn(acc[0][0]);
    }
    __syncthreads();
    if (s_fail) {  // a copy never landed: record it, let the others land (bounded), publish nothing
        if (tid == 0) {
            dev_fail(a.err, DEV_WAIT_TIMEOUT);
            for (int j = 0; j < m; ++j) mbar_wait(&bars[j], 0u, 1u << 16);
        }
        return;
    }
    const float sg = sigm(a.logits[(size_t)t * a.ls + a.ne]);
    if (a.ep.n == 0) {  // one GPU: combine in slot order, then the gated shared expert
        for (int i = tid; i < n; i += blockDim.x) {
            float acc = 0.0f;
            for (int q = 0; q < a.k; ++q) acc = __fmaf_rn(wsel[q], res[q * a.rows + i], acc);
            const float v = __fmaf_rn(sg, res[a.k * a.rows + i], acc);
            float *o = a.y + (size_t)t * a.d + r0 + i;
            *o = a.acc ? *o + v : v;
        }
    } else {  // expert parallel: this rank's slot outputs to every rank's slot-output area, then count the arrival
        for (int i = tid; i < m * n; i += blockDim.x) {
            const int q = slot_at(i / n), r = i % n;
            const float v = res[q * a.rows + r];
            const size_t off = (((size_t)par * MOE_EP_MAXT + t) * ks + q) * a.d + r0 + r;
            for (int p = 0; p < a.ep.n; ++p) a.ep.dpart[p][off] = v;
        }
        __syncthreads();  // every thread's stores, then the release
        if (tid == 0)
            for (int p = 0; p < a.ep.n; ++p) red_release_sys_add(a.ep.counters[p] + a.ep.rank, 1u);
    }
}


template <uint32_t TY>
cudaError_t moe_gu_launch_t(const MoeGuArgs &a, bool planes, int nt, int G, int ctas, size_t smem, cudaStream_t s) {
    void (*k)(const MoeGuArgs) = nullptr;
    (void)nt;  // any token count: the warps hold one token's x in registers at a time
    if (G == 64) k = planes ? k_moe_gu<TY, true, 2> : k_moe_gu<TY, false, 2>;
    else if (G == 32) k = planes ? k_moe_gu<TY, true, 1> : k_moe_gu<TY, false, 1>;
    else k = planes ? k_moe_gu<TY, true, 0> : k_moe_gu<TY, false, 0>;
    const cudaError_t e = allow_max_dynamic_smem(k);
    if (e != cudaSuccess) return e;
    return launch_k(k, dim3(ctas), dim3(MOE_THREADS), smem, s, a);
}

template <uint32_t TY>
cudaError_t moe_down_launch_t(const MoeDownArgs &a, bool planes, int lpr, dim3 grid, size_t smem, cudaStream_t s) {
    void (*k)(const MoeDownArgs) = nullptr;
    if (planes) k = lpr == 4 ? k_moe_down<TY, 4, true> : lpr == 8 ? k_moe_down<TY, 8, true> : lpr == 16 ? k_moe_down<TY, 16, true> : k_moe_down<TY, 32, true>;
    else k = lpr == 4 ? k_moe_down<TY, 4, false> : lpr == 8 ? k_moe_down<TY, 8, false> : lpr == 16 ? k_moe_down<TY, 16, false> : k_moe_down<TY, 32, false>;
    const cudaError_t e = allow_max_dynamic_smem(k);
    if (e != cudaSuccess) return e;
    return launch_k(k, grid, dim3(MOE_THREADS), smem, s, a);
}

#define FN_MOE_SIG(TY)                                                                                       \
    cudaError_t moe_gu_launch_t<TY>(const MoeGuArgs &, bool, int, int, int, size_t, cudaStream_t);            \
    template cudaError_t moe_down_launch_t<TY>(const MoeDownArgs &, bool, int, dim3, size_t, cudaStream_t);
#define FN_MOE_DECL(TY)                                                                                            \
    extern template cudaError_t moe_gu_launch_t<TY>(const MoeGuArgs &, bool, int, int, int, size_t, cudaStream_t); \
    extern template cudaError_t moe_down_launch_t<TY>(const MoeDownArgs &, bool, int, dim3, size_t, cudaStream_t);
#define FN_MOE_INST(TY) template FN_MOE_SIG(TY)

}  // namespace fn
