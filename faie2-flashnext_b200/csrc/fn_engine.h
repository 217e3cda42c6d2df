// Host-side interfaces shared by the engine's translation units.
#pragma once

#include <unordered_set>

#include "fn_common.cuh"

namespace fn {

// ---------------------------------------------------------------------------------------------------------------
// dequant-GEMV launch plan. Depends on (format, rows, cols, token capacity) only, never on the tokens of a call, so
// a token's result is bit-identical in any batch up to the capacity.
struct GemvPlan {
    uint32_t type = 0;
    int rows = 0, cols = 0;
    uint64_t rb = 0;      // bytes of one GGUF row
    uint32_t ldw = 0;     // device row stride: rb rounded up to 16 bytes (the bulk-copy granule)
    int G = 0;            // 32-value groups per row
    int lpr = 32;         // lanes per row
    int gpl = 1;          // groups per lane (lane l of a row holds groups l, l + lpr, ...)
    int ntcap = 1;        // tokens per call the plan serves (1: x in registers where the row fits)
    int xreg = 0;         // 1: each lane keeps its x slice in registers
    int rps = 0;          // rows per pipeline stage
    int slots = 0;        // stages in the shared-memory ring
    int ctas = 0;         // grid size (contiguous row ranges)
    int threads = 256;
    uint32_t stage_bytes = 0;
    uint32_t x_off = 0, ring_off = 0, grid_off = 0;
    size_t smem = 0;
    const uint8_t *pf = nullptr;  // L2 prefetch hint: every launch also brings [pf, pf + pf_bytes) into L2 (the next
    uint64_t pf_bytes = 0;        // weights of a decode chain), spread over its CTAs
    const float *nw = nullptr;    // RMSNorm folded in: y[t] = rsqrt(mean x[t]^2 + eps) (W . (x[t] * nw)) (cols floats,
    float eps = 0.0f;             // device memory, 16-byte aligned); null: y = W . x
};

bool plan_gemv(GemvPlan &p, uint32_t type, int rows, int cols, int ntcap);
size_t plan_weight_bytes(const GemvPlan &p);  // device bytes of the padded weight

// Fused argmax epilogue of a GEMV (the lm_head): per token, the lowest global row index among the rows holding the
// largest value (NaN never wins, -0 ranks as +0, index 0 when no value exceeds -inf), as in k_argmax
// (engine/faie2fn.cu:1910-1935). Every CTA folds its best key into kacc[t] by an atomic max; the CTA that takes the
// last ticket publishes the winner and clears kacc and the ticket. The key orders (value, -index); row0 is the global
// index of the plan's row 0 (row split across GPUs: keys of the slices combine by max). One launch at a time may use
// a given kacc / ticket.
// Key exchange of a row-split lm_head: after the winner of this rank's slice is known, the publishing CTA stores its
// keys into slot [call parity][this rank][t] of every rank's key area (peer memory over NVLink) and adds 1 to this
// rank's counter in every rank's counter area with a system-scope release; the ranks' combine kernels wait for all
// counters (launch_keys_combine).
constexpr int MAX_RANKS = 8;
struct KeyExchange {
    int n = 0, rank = 0;
    unsigned long long *keys[MAX_RANKS] = {};  // each rank's key area [2][MAX_RANKS][8]
    uint32_t *counters[MAX_RANKS] = {};        // each rank's arrival counters [MAX_RANKS]
    uint32_t *calls = nullptr;                 // this rank's count of publishing launches (local)
};

struct GemvArgmax {
    int row0 = 0;
    int *index = nullptr;                // [nt] (nullable)
    unsigned long long *key = nullptr;   // [nt] (nullable; may be a peer GPU's memory)
    unsigned long long *kacc = nullptr;  // [8] scratch, zero between launches
    unsigned int *ticket = nullptr;      // zero between launches
    const KeyExchange *xr = nullptr;     // row-split lm_head: publish the keys to every rank
};

// y[t][r] (+)= W[r] . x[t] for t < nt <= p.ntcap. W: rows at stride p.ldw bytes (16-byte aligned); x, y: fp32 with
// token strides xs, ys (x 16-byte aligned, xs a multiple of 4). early: x was complete before the previous kernel
// started, so the GEMV does not wait for it before reading x (it waits before it exits). y may be null when am is
// given (no logits written).
// the same on the tensor cores as exact integer products (fn_qmma.cu): Q4_K / Q6_K rows of up to 2048 columns,
// qmma_cap(type, cols) tokens at most (0: not this path)
int qmma_cap(uint32_t type, int cols);
int launch_qmma(const GemvPlan &p, const uint8_t *W, const float *x, int xs, float *y, int ys, int nt, bool acc,
                bool early, cudaStream_t s, const GemvArgmax *am);
int launch_gemv(const GemvPlan &p, const uint8_t *W, const float *x, int xs, float *y, int ys, int nt, bool acc,
                bool early, cudaStream_t s, const GemvArgmax *am = nullptr);

// argmax of logits[t][0..n) for t < nt (token stride ls): same selection rule as the fused epilogue
int launch_argmax(const float *logits, int ls, int n, int nt, int *out, cudaStream_t s);
// out[t] = the index of the largest key keys[r][t] over r < nranks (per-rank keys of a row-split lm_head)
int launch_argmax_keys(const unsigned long long *keys, int nranks, int nt, int *out, cudaStream_t s);
// the consumer side of a KeyExchange on this rank: wait (bounded) until every rank's counter here reaches this rank's
// consumer call count + 1, then out[t] = the winner among the n ranks' keys of that call; counts the call
int launch_keys_combine(const unsigned long long *keys, const uint32_t *counters, uint32_t *calls, int n, int nt,
                        int *out, cudaStream_t s);

// GGUF rows (stride rb) -> the engine's row layout (planes for formats with a fast path, else unchanged) at stride
// ldw. src and dst must not overlap.
int launch_plane_repack(uint32_t type, const uint8_t *src, uint64_t rb, uint8_t *dst, uint32_t ldw, int rows, int cols,
                        cudaStream_t s);

// dequantise rows x cols of GGUF rows (row stride rb bytes) into out[r][c] fp32
int launch_dequant(uint32_t type, const uint8_t *W, uint64_t rb, int rows, int cols, float *out, cudaStream_t s);

// global launch settings (set through the C ABI)
struct Settings {
    bool pdl = true;         // programmatic dependent launch
    bool early = true;       // GEMVs marked early run beside their predecessor
    int warps_per_cta = 0;   // GEMV warps per CTA (0: by weight size)
    int ring_kb = 128;       // GEMV shared-memory rings per CTA (all warps)
    int stage_kb = 16;       // target bytes per pipeline stage
    int ctas_per_sm = 1;     // GEMV CTAs per SM
    int ov_rps = 0;          // overrides (0 = automatic)
    int bench_hot = 0;
    int moe_var = 0;         // MoE layer variant (fn_moe_var): 0 = a routing kernel before gate/up; 1 = one token
                             // on one GPU routed inside the gate/up and down kernels
    int qmma = 0;            // Q4_K / Q6_K GEMVs of 1..4 tokens as integer tensor-core products (fn_qmma)
};
Settings &settings();
int num_sms();
int hook_device();           // device of the synchronous test / bench hooks
cudaStream_t hook_stream();  // their stream (one non-blocking stream per device)

// device buffer freed when the scope ends
struct DevBuf {
    void *p = nullptr;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    template <typename T> T *as() const { return (T *)p; }
};

// allow a kernel the largest dynamic shared memory the SM grants next to its static shared memory, and ask for the
// SM's largest shared-memory carveout: an SM configured with a smaller carveout for one kernel cannot take a CTA of
// the next kernel that needs more until it drains, which would keep consecutive small kernels from overlapping under
// programmatic dependent launch (once per kernel)
template <typename K> cudaError_t allow_max_dynamic_smem(K *k) {
    static std::unordered_set<const void *> done;
    if (done.count((const void *)k)) return cudaSuccess;
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, k);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(227 * 1024 - fa.sharedSizeBytes));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e == cudaSuccess) done.insert((const void *)k);
    return e;
}

// launch with the programmatic-serialization attribute when enabled
template <typename... P, typename... A>
cudaError_t launch_k(void (*k)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = settings().pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, ((P)args)...);
}

// launch_k for a grid of thread-block clusters of `cluster` CTAs along x (gridDim.x a multiple of it)
template <typename... P, typename... A>
cudaError_t launch_kc(void (*k)(P...), dim3 grid, dim3 block, unsigned cluster, size_t smem, cudaStream_t s, A... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cluster;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = settings().pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, k, ((P)args)...);
}

}  // namespace fn
