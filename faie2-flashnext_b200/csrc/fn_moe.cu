// Routed-expert MoE layer for batch-1 decode on B200 (sm_100a): routing, expert gate/up, expert down, the shared
// expert and the slot-order combine (512 experts, top-10, expert width 512, hidden 2048).
//
// Reference behaviour: k_route (engine/faie2fn.cu:1742-1800: softmax over the router logits, top-k by probability
// descending with ties to the lower expert index, weights renormalised over the k), k_tmoe_gu8 (:1082-1156:
// act = silu(gate_e . x) * (up_e . x)), k_tmoe_down (:1158-1184: dpart = down_e . act), the shared expert
// (:2411-2416, swiglu in k_route :1758-1759) and the combine inside k_hc_add (:1299-1318:
// y = sum_k wsel[k] dpart[k] in slot order + sigmoid(shared-gate logit) * shared).
//
// B200 design: two kernels.
//  k_moe_gu    every CTA routes all tokens itself (a 64-bit-key bitonic top-k in shared memory, a few hundred cycles,
//              cheaper than a kernel boundary), then streams its share of the (token, slot, row) pairs of the k routed
//              experts plus the shared expert (slot k) through the TMA-bulk ring: a stage holds R gate rows and the R
//              matching up rows; act[t][slot][r] = silu(g) * u goes to a small scratch buffer.
//  k_moe_down  CTA (chunk, t) owns output rows [r0, r1) of token t for all k + 1 slots, so the slot-order combine
//              happens in the CTA (no per-slot partial buffer, no combine kernel). It routes from the logits (complete
//              two kernels back) and issues all of its down-weight stages BEFORE griddepcontrol.wait, so under
//              programmatic dependent launch its weight stream overlaps k_moe_gu; then it waits for act.
// Ranking: by logit descending, ties to the lower index. exp is monotone, so this is the probability order of the
// reference; it differs from ranking the rounded fp32 exp values only where two different logits round to the same
// probability (the reference then prefers the lower index). The weights are the reference's arithmetic on the chosen
// logits: v_i = expf(l_i - l_max), s = sum_i v_i in rank order, w_i = v_i / s.
#include "fn_moe_impl.cuh"

namespace fn {

FN_MOE_DECL(T_Q4_0) FN_MOE_DECL(T_Q4_1) FN_MOE_DECL(T_Q5_0) FN_MOE_DECL(T_Q5_1) FN_MOE_DECL(T_Q8_0)
FN_MOE_DECL(T_Q2_K) FN_MOE_DECL(T_Q3_K) FN_MOE_DECL(T_Q4_K) FN_MOE_DECL(T_Q5_K) FN_MOE_DECL(T_Q6_K)
FN_MOE_DECL(T_IQ2_XXS) FN_MOE_DECL(T_IQ2_XS) FN_MOE_DECL(T_IQ2_S) FN_MOE_DECL(T_IQ3_XXS) FN_MOE_DECL(T_IQ3_S)
FN_MOE_DECL(T_IQ4_NL) FN_MOE_DECL(T_IQ4_XS) FN_MOE_DECL(T_BF16) FN_MOE_DECL(T_Q2_0)

// ---------------------------------------------------------------------------------------------------------------
// routing alone (fn_bench_route): logits = sum over ks split-K partials part[k][t][rsg] in split order, then route

__global__ void __launch_bounds__(256) k_route(const float *part, int ks, int kst, int ts, int ne, int k, int *sel_out,
                                               float *w_out) {
    __shared__ float lg[1024];
    __shared__ int sel[16];
    __shared__ float w[16];
    __shared__ unsigned long long keys[128];
    const int t = blockIdx.x;
    pdl_wait();
    for (int i = threadIdx.x; i < ne; i += blockDim.x) {
        const float *q = part + (size_t)t * ts + i;
        float s = q[0];
        for (int j = 1; j < ks; ++j) s += q[(size_t)j * kst];
        lg[i] = s;
    }
    __syncthreads();
    pdl_trigger();
    route_token(lg, ne, k, sel, w, keys);
    if (threadIdx.x < k) {
        sel_out[t * k + threadIdx.x] = sel[threadIdx.x];
        w_out[t * k + threadIdx.x] = w[threadIdx.x];
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
    if (!rg || !rd || d % 32 || ffe % 32 || ne < 1 || ne > 1024 || k < 1 || k > 16 || k > ne) return false;
    p.rb_gu = rg;
    p.rb_down = rd;
    p.ldw_gu = (uint32_t)al(rg, 16);
    p.ldw_down = (uint32_t)al(rd, 16);
    const int Gd = ffe / 32;
    p.lpr_down = Gd == 16 ? 16 : 32;
    return true;
}

static int sm_count() { return num_sms(); }


int launch_moe(const MoePlan &p, const MoeWeights &w, const float *logits, int ls, const float *x, float *act, float *y,
               int nt, bool acc, int *sel_out, float *w_out, bool planes, cudaStream_t s) {
    if (nt < 1 || nt > 8) return fail("moe: nt out of range (1..8)");
    if (ls < p.ne + 1) return fail("moe: logits stride must hold ne + 1 columns (router + shared gate)");
    if (((uintptr_t)x & 15) || ((uintptr_t)act & 15) || (p.d & 3) || (p.ffe & 3)) return fail("moe: x/act alignment");
    const int ks = p.k + 1;
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
        a.sel_out = sel_out;
        a.w_out = w_out;
        const long long U = (long long)nt * ks * p.ffe;
        const int ctas = (int)std::min<long long>(sm_count(), (U + 7) / 8);
        const int per_cta = (int)((U + ctas - 1) / ctas);
        a.rps = std::max(1, std::min(per_cta, std::max(8, (int)(12 * 1024 / (2 * p.ldw_gu)) / 8 * 8)));
        a.stage_bytes = (uint32_t)al((size_t)2 * a.rps * p.ldw_gu, 128);
        a.slots = std::max(2, std::min(16, (int)(96 * 1024 / a.stage_bytes)));
        a.ring_off = 128;
        a.grid_off = (uint32_t)al(a.ring_off + (size_t)a.slots * a.stage_bytes, 128);
        a.misc_off = (uint32_t)al(a.grid_off + (size_t)grid_words(p.gu_type) * 4, 128);
        a.x_off = (uint32_t)al(a.misc_off + 8 * 16 * 8 + 128 * 8 + 2 * a.rps * 4, 128);
        const size_t smem = al(a.x_off + (size_t)nt * (p.d / 32) * XPAD * 4, 128);
        if (smem > 227 * 1024) return fail("moe: gate/up shared memory too large");
        a.err = dev_error_ptr();
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
        const int chunks = std::max(1, std::min((p.d + 7) / 8, sm_count() / nt));
        a.chunks = chunks;
        const int rows_per = (p.d + chunks - 1) / chunks;
        a.rps = std::max(1, std::min(rows_per, std::max(1, (int)(8 * 1024 / p.ldw_down))));
        a.stage_bytes = (uint32_t)al((size_t)a.rps * p.ldw_down, 128);
        a.slots = std::max(2, std::min(16, (int)(96 * 1024 / a.stage_bytes)));
        a.ring_off = 128;
        a.grid_off = (uint32_t)al(a.ring_off + (size_t)a.slots * a.stage_bytes, 128);
        a.misc_off = (uint32_t)al(a.grid_off + (size_t)grid_words(p.down_type) * 4, 128);
        a.x_off = (uint32_t)al(a.misc_off + 16 * 8 + 128 * 8 + (size_t)ks * a.rps * 4, 128);
        const size_t smem = al(a.x_off + (size_t)ks * (p.ffe / 32) * XPAD * 4, 128);
        if (smem > 227 * 1024) return fail("moe: down shared memory too large");
        a.err = dev_error_ptr();
        cudaError_t e = cudaSuccess;
        const bool known = dispatch_type(p.down_type, [&]<uint32_t TY>() {
            e = moe_down_launch_t<TY>(a, planes, p.lpr_down, dim3(chunks, nt), smem, s);
        });
        if (!known) return fail("moe: unsupported down type");
        if (e != cudaSuccess) return fail(std::string("moe down launch: ") + cudaGetErrorString(e));
    }
    return 0;
}

int launch_route(const float *part, int ks, size_t kst, int ts, int ne, int k, int nt, int *sel, float *w,
                 cudaStream_t s) {
    if (ne < 1 || ne > 1024 || k < 1 || k > 16 || k > ne || nt < 1) return fail("route: unsupported ne/k/nt");
    cudaError_t e = launch_k(k_route, dim3(nt), dim3(256), 0, s, part, ks, (int)kst, ts, ne, k, sel, w);
    if (e != cudaSuccess) return fail(std::string("route launch: ") + cudaGetErrorString(e));
    return 0;
}

}  // namespace fn
