// Routed-expert MoE layer for batch-1 decode on B200 (sm_100a): routing, expert gate/up, expert down, the shared
// expert and the slot-order combine (512 experts, top-10, expert width 512, hidden 2048).
//
// Reference behaviour: k_route (engine/faie2fn.cu:1742-1800: softmax over the router logits, top-k by probability
// descending with ties to the lower expert index, weights renormalised over the k), k_tmoe_gu8 (:1082-1156:
// act = silu(gate_e . x) * (up_e . x)), k_tmoe_down (:1158-1184: dpart = down_e . act), the shared expert
// (:2411-2416, swiglu in k_route :1758-1759) and the combine inside k_hc_add (:1299-1318:
// y = sum_k wsel[k] dpart[k] in slot order + sigmoid(shared-gate logit) * shared).
//
// B200 design: two kernels (one token on one GPU), or a routing kernel (k_moe_route, one CTA per token) and two.
//  k_moe_gu    routes the tokens itself for one token (a 64-bit-key bitonic top-k in shared memory, a few hundred
//              cycles, cheaper than a kernel boundary), then streams its share of the (token, slot, row) pairs of the k routed
//              experts plus the shared expert (slot k) through the TMA-bulk ring: a stage holds R gate rows and the R
//              matching up rows; act[t][slot][r] = silu(g) * u goes to a small scratch buffer.
//  k_moe_down  CTA (chunk, t) owns output rows [r0, r1) of token t for all k + 1 slots, so the slot-order combine
//              happens in the CTA (no per-slot partial buffer, no combine kernel). It routes from the logits (complete
//              two kernels back) and issues all of its down-weight stages BEFORE griddepcontrol.wait, so under
//              programmatic dependent launch its weight stream overlaps k_moe_gu; then it waits for act.
// Ranking (route_token): the reference's order, fp32 v = expf(l - max l) descending with equal v to the lower index,
// and its weights: s = sum of the k v's in rank order, w = v / s.
#include "fn_moe_impl.cuh"

namespace fn {

FN_MOE_DECL(T_Q4_0) FN_MOE_DECL(T_Q4_1) FN_MOE_DECL(T_Q5_0) FN_MOE_DECL(T_Q5_1) FN_MOE_DECL(T_Q8_0)
FN_MOE_DECL(T_Q2_K) FN_MOE_DECL(T_Q3_K) FN_MOE_DECL(T_Q4_K) FN_MOE_DECL(T_Q5_K) FN_MOE_DECL(T_Q6_K)
FN_MOE_DECL(T_IQ2_XXS) FN_MOE_DECL(T_IQ2_XS) FN_MOE_DECL(T_IQ2_S) FN_MOE_DECL(T_IQ3_XXS) FN_MOE_DECL(T_IQ3_S)
FN_MOE_DECL(T_IQ4_NL) FN_MOE_DECL(T_IQ4_XS) FN_MOE_DECL(T_BF16) FN_MOE_DECL(T_Q2_0)

// ---------------------------------------------------------------------------------------------------------------
// routing of a layer

// the routing of nt tokens, one CTA (>= 8 warps) per token: sel / w [nt][16] for the MoE kernels, and the caller's
// sel_out / w_out [nt][k] when given
__global__ void __launch_bounds__(ROUTE_THREADS) k_moe_route(const float *logits, int ls, int ne, int k, int *rsel,
                                                              float *rw, int *sel_out, float *w_out) {
    __shared__ int sel[16];
    __shared__ float w[16];
    __shared__ __align__(16) unsigned long long keys[16 * 16];
    __shared__ float vals[16];
    const int t = blockIdx.x;
    pdl_wait();
    pdl_trigger();  // the gate/up kernel may start its prologue (codebook, weight-independent staging) now
    const float *l = after_wait(logits) + (size_t)t * ls;
    route_token(l, ne, k, sel, w, keys, vals);
    if ((int)threadIdx.x < k) {
        rsel[t * 16 + threadIdx.x] = sel[threadIdx.x];
        rw[t * 16 + threadIdx.x] = w[threadIdx.x];
        if (sel_out) {
            sel_out[t * k + threadIdx.x] = sel[threadIdx.x];
            w_out[t * k + threadIdx.x] = w[threadIdx.x];
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// routing alone (fn_bench_route): logits = sum over ks split-K partials part[k][t][rsg] in split order, then route

__device__ __forceinline__ float sum_splits(const float *part, int ks, int kst, int ts, int t, int i) {
    const float *q = part + (size_t)t * ts + i;
    float s = q[0];
    for (int j = 1; j < ks; ++j) s += q[(size_t)j * kst];
    return s;
}

// variant 1: the engine's routing (route_token)
__global__ void __launch_bounds__(ROUTE_THREADS) k_route(const float *part, int ks, int kst, int ts, int ne, int k,
                                                         int *sel_out, float *w_out) {
    __shared__ float lg[1024];
    __shared__ int sel[16];
    __shared__ float w[16];
    __shared__ __align__(16) unsigned long long keys[16 * 16];
    __shared__ float vals[16];
    const int t = blockIdx.x;
    pdl_wait();
    for (int i = threadIdx.x; i < ne; i += blockDim.x) lg[i] = sum_splits(part, ks, kst, ts, t, i);
    __syncthreads();
    pdl_trigger();
    route_token(lg, ne, k, sel, w, keys, vals);
    if (threadIdx.x < k) {
        sel_out[t * k + threadIdx.x] = sel[threadIdx.x];
        w_out[t * k + threadIdx.x] = w[threadIdx.x];
    }
}

// variant 0: the reference's order counted out directly, the check for route_token. Expert i's rank is the number of
// experts ahead of it: larger v, or equal v and a lower index (v = expf(l - max l) in fp32); rank r < k is slot r,
// s = the k v's summed in rank order by one thread, w = v / s. ne comparisons per expert: a checker, not the
// engine's path.
__global__ void __launch_bounds__(ROUTE_THREADS) k_route_count(const float *part, int ks, int kst, int ts, int ne,
                                                               int k, int *sel_out, float *w_out) {
    __shared__ float lg[1024];
    __shared__ float pv[1024];
    __shared__ float wmax[ROUTE_THREADS / 32];
    __shared__ int sel[16];
    __shared__ float val[16];
    const int t = blockIdx.x, lane = threadIdx.x & 31;
    pdl_wait();
    float m = -INFINITY;
    for (int i = threadIdx.x; i < ne; i += blockDim.x) {
        lg[i] = sum_splits(part, ks, kst, ts, t, i);
        m = fmaxf(m, lg[i]);
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    m = wmax[0];
    for (int w2 = 1; w2 < (int)(blockDim.x >> 5); ++w2) m = fmaxf(m, wmax[w2]);
    for (int i = threadIdx.x; i < ne; i += blockDim.x) pv[i] = expf(lg[i] - m);
    __syncthreads();
    pdl_trigger();
    for (int i = threadIdx.x; i < ne; i += blockDim.x) {
        const float v = pv[i];
        int r = 0;
        for (int j = 0; j < ne; ++j) r += pv[j] > v || (pv[j] == v && j < i);
        if (r < k) {
            sel[r] = i;
            val[r] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int r = 0; r < k; ++r) s += val[r];
        for (int r = 0; r < k; ++r) {
            sel_out[t * k + r] = sel[r];
            w_out[t * k + r] = val[r] / s;
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// expert-parallel combine: CTA t waits (bounded) until every rank's down kernel has delivered its slot outputs of this
// call, then y[t] = sum_{s<k} w[s] dpart[s] in slot order + sigmoid(shared-gate logit) dpart[k], with the same fused
// multiply-adds in the same order as the one-GPU down kernel's combine, so the result is bit-identical to it. The CTA
// that takes the last ticket advances this rank's call count and expected arrivals.

struct MoeCombineArgs {
    const float *logits;
    const float *rw;  // routing weights [nt][16] (k_moe_route)
    int ls, ne, k, d, nt, n;
    const float *dpart;         // this rank's slot-output area
    const uint32_t *counters;   // this rank's arrival counters [n]
    uint32_t *calls;            // [call count, expected arrivals, ticket]
    uint32_t arrivals;          // arrivals per source rank of this call (its down kernel's CTAs)
    float *y;
    int acc;
    uint32_t *err;
};

__global__ void __launch_bounds__(256) k_moe_ep_combine(const MoeCombineArgs a) {
    __shared__ float wsel[16];
    __shared__ int s_ok;
    // CTA (chunk, t): rows [chunk d / gridDim.x, (chunk + 1) d / gridDim.x) of token t
    const int t = blockIdx.y, tid = threadIdx.x, ks = a.k + 1;
    const int i0 = (int)((long long)blockIdx.x * a.d / gridDim.x), i1 = (int)((long long)(blockIdx.x + 1) * a.d / gridDim.x);
    // the routing weights and logits were complete before the gate/up kernel two launches back passed its wait
    if (tid < a.k) wsel[tid] = a.rw[t * 16 + tid];
    pdl_wait();
    const uint32_t *calls = after_wait(a.calls);
    const uint32_t c = calls[0], expect = calls[1] + a.arrivals;
    if (tid == 0) {
        bool ok = true;
        for (int r = 0; r < a.n && ok; ++r) ok = wait_counter_sys(a.counters + r, expect);
        s_ok = ok;
    }
    __syncthreads();
    pdl_trigger();
    if (s_ok) {
        const float *dp = a.dpart + ((size_t)(c & 1u) * MOE_EP_MAXT + t) * ks * a.d;
        const float sg = sigm(a.logits[(size_t)t * a.ls + a.ne]);
        for (int i = i0 + tid; i < i1; i += blockDim.x) {
            float acc = 0.0f;
            for (int q = 0; q < a.k; ++q) acc = __fmaf_rn(wsel[q], dp[(size_t)q * a.d + i], acc);
            const float v = __fmaf_rn(sg, dp[(size_t)a.k * a.d + i], acc);
            float *o = a.y + (size_t)t * a.d + i;
            *o = a.acc ? *o + v : v;
        }
    } else if (tid == 0) {
        dev_fail(a.err, DEV_PEER_TIMEOUT);
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t tk;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(tk) : "l"(a.calls + 2) : "memory");
        if (tk == gridDim.x * gridDim.y - 1) {
            a.calls[0] = c + 1;
            a.calls[1] = expect;
            a.calls[2] = 0u;
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// host

static size_t al(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool plan_moe(MoePlan &p, uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d) {
    p = MoePlan{};
    p.gu_type = gu_type;
    p.down_type = down_type;
    p.ne = ne;
    p.k = k;
    p.ffe = ffe;
    p.d = d;
    const uint64_t rg = row_bytes(gu_type, d), rd = row_bytes(down_type, ffe);
    if (!rg || !rd || d % 32 || ffe % 32 || ne < 1 || ne > 1024 || k < 1 || k > 16 || k > ne || ffe > 65536 || d > 65536)
        return false;
    p.rb_gu = rg;
    p.rb_down = rd;
    p.ldw_gu = (uint32_t)al(rg, 16);
    p.ldw_down = (uint32_t)al(rd, 16);
    const int Gd = ffe / 32;
    // lanes per down row: about four groups per lane (fewer lanes per row, fewer butterfly levels per row)
    p.lpr_down = Gd >= 128 ? 32 : Gd >= 64 ? 16 : Gd >= 32 ? 8 : 4;
    return true;
}

static int sm_count() { return num_sms(); }

// dynamic shared memory of the MoE kernels: the SM's 227 KiB less 4 KiB for their static shared memory (routing pairs,
// x scale maxima)
constexpr size_t kMoeDynSmem = 227 * 1024 - 4 * 1024;


int launch_moe(const MoePlan &p, const MoeWeights &w, const float *logits, int ls, const float *x, float *act,
               uint32_t *route, float *y, int nt, bool acc, int *sel_out, float *w_out, bool planes, cudaStream_t s,
               const MoeEp *ep, bool x_early, uint32_t *sync) {
    if (nt < 1 || nt > (ep ? MOE_EP_MAXT : MOE_MAXT)) return fail("moe: nt out of range (1..32, 1..8 expert parallel)");
    if (!route) return fail("moe: no routing scratch");
    int *rsel = (int *)route;
    float *rw = (float *)(route + MOE_MAXT * 16);
    const MoeEp none{};
    const MoeEp &E = ep ? *ep : none;
    if (ep) {
        if (E.n < 1 || E.n > MAX_RANKS || E.rank < 0 || E.rank >= E.n || !E.calls ||
            E.e0 != (int)((long long)E.rank * p.ne / E.n))
            return fail("moe: bad expert-parallel group");
        for (int r = 0; r < E.n; ++r)
            if (!E.dpart[r] || !E.counters[r]) return fail("moe: expert parallel without peer memory");
    }
    if (ls < p.ne + 1) return fail("moe: logits stride must hold ne + 1 columns (router + shared gate)");
    if (((uintptr_t)x & 15) || ((uintptr_t)act & 15) || (p.d & 3) || (p.ffe & 3)) return fail("moe: x/act alignment");
    const int ks = p.k + 1;
    if (p.nw && ((uintptr_t)p.nw & 15)) return fail("moe: the norm weight must be 16-byte aligned");
    // ---- routing: one token on one GPU is routed inside the gate/up and down kernels (one launch fewer per layer);
    // otherwise once per layer by its own kernel (one CTA per token)
    const bool route_self = nt == 1 && !ep && settings().moe_var == 1;
    if (!route_self) {
        const cudaError_t e = launch_k(k_moe_route, dim3(nt), dim3(ROUTE_THREADS), 0, s, logits, ls, p.ne, p.k, rsel, rw,
                                       sel_out, w_out);
        if (e != cudaSuccess) return fail(std::string("moe route launch: ") + cudaGetErrorString(e));
    }
    // ---- the fused form: gate/up and down in one kernel (one token on one GPU)
    if (settings().moe_var == 2 && nt == 1 && !ep && planes && ls == p.ne + 1) {
        const int rc = launch_moe_fused(p, w, logits, x, act, rsel, rw, sync, y, acc, x_early, s);
        if (rc <= 0) return rc;  // launched, or an error; 1: no fused form, the two kernels below
    }
    // ---- gate / up
    {
        MoeGuArgs a;
        a.Wg = w.gate;
        a.Wu = w.up;
        a.Wsg = w.sh_gate;
        a.Wsu = w.sh_up;
        a.ldw = p.ldw_gu;
        {
            int qk, tb;
            type_info(p.gu_type, qk, tb);
            a.nb = p.d / qk;
        }
        a.ne = p.ne;
        a.k = p.k;
        a.ffe = p.ffe;
        a.d = p.d;
        a.nt = nt;
        a.logits = logits;
        a.ls = ls;
        a.x = x;
        a.act = act;
        a.rsel = rsel;
        a.route_self = route_self ? 1 : 0;
        a.x_early = x_early && settings().pdl ? 1 : 0;
        a.nw = p.nw;
        a.eps = p.eps;
        // one unit (a gate row and its up row) per ring stage; each warp has its own ring of `slots` stages
        constexpr int NW = MOE_THREADS / 32;
        const long long U = (long long)nt * ks * p.ffe;  // upper bound (every slot computed here)
        // with a routing kernel, one SM fewer than the GPU has: its CTA keeps an SM while the gate/up CTAs start beside
        // it (programmatic launch), and a gate/up CTA does not fit next to it
        const int ctas = (int)std::min<long long>(std::max(1, sm_count() - (route_self ? 0 : 1)), (U + 7) / 8);
        const long long per_warp0 = (U + (long long)ctas * NW - 1) / ((long long)ctas * NW);
        // rows of 32 or 64 groups: the warps read x into registers themselves, nothing is staged in shared memory
        const bool xreg = p.d == 1024 || p.d == 2048;
        const size_t xb = xreg ? 0 : (size_t)nt * (p.d / 32) * XPAD * 4, misc = (size_t)nt * 16 * 4,
                     gw = (size_t)grid_words(p.gu_type) * 4;
        const size_t fixed = 1024 + gw + 128 + misc + 128 + xb + 128;
        // a warp's few units in one stage (one more stage where its run crosses an expert boundary); else two units
        // per stage (several tokens: many units per warp); shorter runs where rows are wide
        a.run = per_warp0 <= 4 ? (int)per_warp0 : 2;
        while (a.run > 1 && fixed + (size_t)NW * al((size_t)2 * a.run * p.ldw_gu, 128) > kMoeDynSmem / 2) --a.run;
        a.stage_bytes = (uint32_t)al((size_t)2 * a.run * p.ldw_gu, 128);
        if (fixed + (size_t)NW * a.stage_bytes > kMoeDynSmem) return fail("moe: gate/up rows too wide for shared memory");
        const long long per_warp = (per_warp0 + a.run - 1) / a.run + 1;  // stages per warp at most
        const long long fit = (long long)(std::min<size_t>(192 * 1024, kMoeDynSmem - fixed) / ((size_t)NW * a.stage_bytes));
        a.slots = (int)std::max<long long>(1, std::min<long long>(std::min<long long>(8, per_warp), fit));
        a.slots = std::min(a.slots, 1024 / (8 * NW));  // barriers: 1 KiB
        a.ring_off = 1024;
        a.grid_off = (uint32_t)al(a.ring_off + (size_t)NW * a.slots * a.stage_bytes, 128);
        a.misc_off = (uint32_t)al(a.grid_off + gw, 128);
        a.x_off = (uint32_t)al(a.misc_off + misc, 128);
        const size_t smem = al(a.x_off + xb, 128);
        if (smem > kMoeDynSmem) return fail("moe: gate/up shared memory too large");
        if (route_self && (size_t)NW * a.slots * a.stage_bytes < 2304) return fail("moe: ring too small for the routing scratch");
        a.err = dev_error_ptr();
        a.ep = E;
        const int G = p.d / 32;
        cudaError_t e = cudaSuccess;
        const bool known = dispatch_type(p.gu_type, [&]<uint32_t TY>() { e = moe_gu_launch_t<TY>(a, planes, nt, G, ctas, smem, s); });
        if (!known) return fail("moe: unsupported gate/up type");
        if (e != cudaSuccess) return fail(std::string("moe gate/up launch: ") + cudaGetErrorString(e));
    }
    // ---- down + combine
    {
        MoeDownArgs a;
        a.Wd = w.down;
        a.Wsd = w.sh_down;
        a.ldw = p.ldw_down;
        {
            int qk, tb;
            type_info(p.down_type, qk, tb);
            a.nb = p.ffe / qk;
        }
        a.ne = p.ne;
        a.k = p.k;
        a.ffe = p.ffe;
        a.d = p.d;
        a.nt = nt;
        a.logits = logits;
        a.ls = ls;
        a.act = act;
        a.y = y;
        a.acc = acc ? 1 : 0;
        a.rsel = rsel;
        a.rw = rw;
        a.route_self = route_self ? 1 : 0;
        a.sel_out = sel_out;
        a.w_out = w_out;
        a.pf = p.pf;
        a.pf_bytes = p.pf_bytes;
        // CTA (chunk, t): rows [r0, r1) of token t, every computed slot's rows in shared memory at once
        const size_t xb = (size_t)ks * (p.ffe / 32) * XPAD * 4, misc = 0,
                     gw = (size_t)grid_words(p.down_type) * 4;
        const size_t fixed = 256 + 128 + gw + 128 + misc + 128 + xb + 128;
        if (fixed + (size_t)ks * (p.ldw_down + 4) > kMoeDynSmem) return fail("moe: down rows too wide for shared memory");
        const int max_rows = (int)((kMoeDynSmem - fixed) / ((size_t)ks * (p.ldw_down + 4)));
        int chunks = std::max(1, std::min((p.d + 7) / 8, sm_count() / nt));
        int rows = (p.d + chunks - 1) / chunks;
        if (rows > max_rows) {  // more CTAs than SMs: as many chunks as fill whole waves of one CTA per SM
            rows = max_rows;
            chunks = (p.d + rows - 1) / rows;
            const int waves = (chunks * nt + sm_count() - 1) / sm_count();
            chunks = std::min(p.d, std::max(chunks, waves * sm_count() / nt));
        }
        rows = (p.d + chunks - 1) / chunks;  // the largest chunk of the even split
        a.rows = rows;
        a.w_off = 256;
        a.res_off = (uint32_t)al(a.w_off + (size_t)ks * rows * p.ldw_down, 128);
        a.grid_off = (uint32_t)al(a.res_off + (size_t)ks * rows * 4, 128);
        a.misc_off = (uint32_t)al(a.grid_off + gw, 128);
        a.x_off = (uint32_t)al(a.misc_off + misc, 128);
        const size_t smem = al(a.x_off + xb, 128);
        if (smem > kMoeDynSmem) return fail("moe: down shared memory too large");
        if (route_self && xb < 2304) return fail("moe: activation staging too small for the routing scratch");
        a.err = dev_error_ptr();
        a.ep = E;
        cudaError_t e = cudaSuccess;
        const bool known = dispatch_type(p.down_type, [&]<uint32_t TY>() {
            e = moe_down_launch_t<TY>(a, planes, p.lpr_down, dim3(chunks, nt), smem, s);
        });
        if (!known) return fail("moe: unsupported down type");
        if (e != cudaSuccess) return fail(std::string("moe down launch: ") + cudaGetErrorString(e));
        if (ep) {  // ---- expert parallel: combine the ranks' slot outputs on every rank
            MoeCombineArgs c{logits, rw, ls, p.ne, p.k, p.d, nt, E.n, E.dpart[E.rank], E.counters[E.rank], E.calls,
                             (uint32_t)(chunks * nt), y, acc ? 1 : 0, dev_error_ptr()};
            e = launch_k(k_moe_ep_combine, dim3(std::max(1, std::min(16, p.d / 128)), nt), dim3(256), 0, s, c);
            if (e != cudaSuccess) return fail(std::string("moe combine launch: ") + cudaGetErrorString(e));
        }
    }
    return 0;
}

int launch_route(int variant, const float *part, int ks, size_t kst, int ts, int ne, int k, int nt, int *sel, float *w,
                 cudaStream_t s) {
    if (ne < 1 || ne > 1024 || k < 1 || k > 16 || k > ne || nt < 1) return fail("route: unsupported ne/k/nt");
    if (variant != 0 && variant != 1) return fail("route: variant must be 0 or 1");
    cudaError_t e = launch_k(variant == 0 ? k_route_count : k_route, dim3(nt), dim3(ROUTE_THREADS), 0, s, part, ks,
                             (int)kst, ts, ne, k, sel, w);
    if (e != cudaSuccess) return fail(std::string("route launch: ") + cudaGetErrorString(e));
    return 0;
}

}  // namespace fn
