// Host interface of the routed-expert MoE layer (fn_moe.cu).
#pragma once

#include "fn_common.cuh"

namespace fn {

struct MoePlan {
    uint32_t gu_type = 0, down_type = 0;  // gate/up format (routed and shared), down format (routed and shared)
    int ne = 0, k = 0, ffe = 0, d = 0;     // experts, experts per token, expert width, hidden size
    uint64_t rb_gu = 0, rb_down = 0;       // GGUF row bytes
    uint32_t ldw_gu = 0, ldw_down = 0;     // device row strides (16-byte multiples)
    int lpr_down = 32;
};

// device weights, rows at the plan's strides: gate/up ne * ffe rows of d columns (expert e at rows e * ffe ..),
// down ne * d rows of ffe columns (expert e at rows e * d ..); the shared expert: ffe (gate/up) and d (down) rows
struct MoeWeights {
    const uint8_t *gate = nullptr, *up = nullptr, *down = nullptr;
    const uint8_t *sh_gate = nullptr, *sh_up = nullptr, *sh_down = nullptr;
};

bool plan_moe(MoePlan &p, uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d);

// y[t] (+)= sum_{s<k} w[t][s] down_{sel[t][s]} . act[t][s] + sigmoid(logits[t][ne]) shared(x[t]) for t < nt <= 8, with
// act[t][s] = silu(gate_e . x[t]) * (up_e . x[t]) and (sel, w) the top-k routing of logits[t][0..ne). logits: token
// stride ls >= ne + 1. act: scratch of nt * (k + 1) * ffe floats. sel_out / w_out (nullable): [nt][k]. planes: the
// weights are in the engine's plane layout (launch_plane_repack), else GGUF rows at the plan's strides.
int launch_moe(const MoePlan &p, const MoeWeights &w, const float *logits, int ls, const float *x, float *act, float *y,
               int nt, bool acc, int *sel_out, float *w_out, bool planes, cudaStream_t s);

// routing alone on split-K partials: logits[t][i] = sum_{j<ks} part[j * kst + t * ts + i] (split order)
int launch_route(const float *part, int ks, size_t kst, int ts, int ne, int k, int nt, int *sel, float *w,
                 cudaStream_t s);

}  // namespace fn
