// Host interface of the routed-expert MoE layer (fn_moe.cu).
#pragma once

#include "fn_engine.h"

namespace fn {

struct MoePlan {
    uint32_t gu_type = 0, down_type = 0;  // gate/up format (routed and shared), down format (routed and shared)
    int ne = 0, k = 0, ffe = 0, d = 0;     // experts, experts per token, expert width, hidden size
    uint64_t rb_gu = 0, rb_down = 0;       // GGUF row bytes
    uint32_t ldw_gu = 0, ldw_down = 0;     // device row strides (16-byte multiples)
    int lpr_down = 32;
    const uint8_t *pf = nullptr;  // L2 prefetch hint of the down kernel (GemvPlan::pf)
    uint64_t pf_bytes = 0;
    const float *nw = nullptr;    // RMSNorm folded in (GemvPlan::nw): the layer's input is rmsnorm(x) * nw
    float eps = 0.0f;
};

// device weights, rows at the plan's strides: gate/up ne * ffe rows of d columns (expert e at rows e * ffe ..),
// down ne * d rows of ffe columns (expert e at rows e * d ..); the shared expert: ffe (gate/up) and d (down) rows
struct MoeWeights {
    const uint8_t *gate = nullptr, *up = nullptr, *down = nullptr;
    const uint8_t *sh_gate = nullptr, *sh_up = nullptr, *sh_down = nullptr;
};

bool plan_moe(MoePlan &p, uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d);

// Expert parallelism over n ranks (one GPU each; n == 0: one GPU holds every expert). Rank g holds the routed experts
// [g ne / n, (g + 1) ne / n) (local weights start at expert e0) and a copy of the shared expert. Every rank routes
// every token (the router logits are replicated); a routed slot is computed by the rank that holds its expert, the
// shared slot by the rank holding the fewest of the token's routed slots (the lowest such rank). The down kernel
// stores each computed slot's output rows into every rank's slot-output area (peer memory over NVLink) and counts
// the CTA's arrival at every rank; the combine kernel then adds the k + 1 slot outputs in slot order on every rank,
// exactly as the one-GPU down kernel does.
constexpr int MOE_EP_MAXT = 8;   // tokens per call of an expert-parallel layer
constexpr int MOE_MAXT = 32;     // tokens per call of a one-GPU layer (batched decode)
struct MoeEp {
    int n = 0, rank = 0, e0 = 0;
    float *dpart[MAX_RANKS] = {};        // each rank's slot-output area [2][MOE_EP_MAXT][k + 1][d]
    uint32_t *counters[MAX_RANKS] = {};  // each rank's MoE arrival counters [MAX_RANKS]
    uint32_t *calls = nullptr;           // this rank's [call count, expected arrivals per source rank, ticket]
};

// y[t] (+)= sum_{s<k} w[t][s] down_{sel[t][s]} . act[t][s] + sigmoid(logits[t][ne]) shared(x[t]) for t < nt <= 32 (8 expert parallel), with
// act[t][s] = silu(gate_e . x[t]) * (up_e . x[t]) and (sel, w) the top-k routing of logits[t][0..ne). logits: token
// stride ls >= ne + 1. act: scratch of nt * (k + 1) * ffe floats; route: scratch of MOE_ROUTE_WORDS 32-bit words.
// sel_out / w_out (nullable): [nt][k]. planes: the weights are in the engine's plane layout (launch_plane_repack),
// else GGUF rows at the plan's strides. x_early: x was complete before the kernel before this layer started (the
// router GEMV's predecessor wrote it), so the gate/up kernel reads it beside the routing kernel.
constexpr int MOE_ROUTE_WORDS = 2 * MOE_MAXT * 16;  // sel [MOE_MAXT][16] ints, then w [MOE_MAXT][16] floats
// sync (nullable): MOE_SYNC_WORDS zeroed words of the layer's own, which allow the fused single-kernel form
// (fn_moe_var(2), one token on one GPU: launch_moe_fused).
constexpr int MOE_SYNC_WORDS = 32;
int launch_moe(const MoePlan &p, const MoeWeights &w, const float *logits, int ls, const float *x, float *act,
               uint32_t *route, float *y, int nt, bool acc, int *sel_out, float *w_out, bool planes, cudaStream_t s,
               const MoeEp *ep = nullptr, bool x_early = false, uint32_t *sync = nullptr);
// the fused form after the routing kernel: 0 launched, 1 no fused form for this layer, -1 error
int launch_moe_fused(const MoePlan &p, const MoeWeights &w, const float *logits, const float *x, float *act,
                     const int *rsel, const float *rw, uint32_t *cnt, float *y, bool acc, bool x_early, cudaStream_t s);

// routing alone on split-K partials: logits[t][i] = sum_{j<ks} part[j * kst + t * ts + i] (split order)
int launch_route(int variant, const float *part, int ks, size_t kst, int ts, int ne, int k, int nt, int *sel, float *w,
                 cudaStream_t s);

}  // namespace fn
