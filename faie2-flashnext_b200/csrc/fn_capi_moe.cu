// C ABI of the MoE layer and the routing hook (declared in include/faie2fn.h).
#include <cuda.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "fn_engine.h"
#include "fn_moe.h"
#include "fn_peer.h"

namespace fn {

struct MoeH {
    MoePlan p;
    DevBuf gate, up, down, sg, su, sd, act, route, sync;
    MoeWeights w;
    int group = 0;  // expert parallel: the peer group (0: one GPU)
    int e0 = 0;
};
static std::vector<MoeH *> g_moe;
static std::mutex g_moe_mu;

static MoeH *moe_get(int h) {
    std::lock_guard<std::mutex> l(g_moe_mu);
    return h >= 1 && h <= (int)g_moe.size() ? g_moe[h - 1] : nullptr;
}

// upload GGUF rows (row bytes rb) to a device buffer in the engine's layout (planes, stride ldw)
static int upload_rows(DevBuf &b, uint32_t type, const uint8_t *src, uint64_t rb, uint32_t ldw, size_t rows, int cols,
                       cudaStream_t s) {
    DevBuf raw;
    FN_CK(cudaMalloc(&b.p, (size_t)ldw * rows));
    FN_CK(cudaMalloc(&raw.p, (size_t)rb * rows));
    FN_CK(cudaMemcpyAsync(raw.p, src, (size_t)rb * rows, cudaMemcpyHostToDevice, s));
    if (launch_plane_repack(type, raw.as<uint8_t>(), rb, b.as<uint8_t>(), ldw, (int)rows, cols, s)) return -1;
    FN_CK(cudaStreamSynchronize(s));
    return 0;
}

// ne_local: experts held here (all ne on one GPU; an expert-parallel rank's slice otherwise)
static MoeH *moe_build(uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d, const uint8_t *Wg,
                       const uint8_t *Wu, const uint8_t *Wd, const uint8_t *Wsg, const uint8_t *Wsu, const uint8_t *Wsd,
                       cudaStream_t s, int ne_local = -1) {
    if (ne_local < 0) ne_local = ne;
    MoeH *m = new MoeH();
    if (!plan_moe(m->p, gu_type, down_type, ne, k, ffe, d)) {
        delete m;
        fail("moe: unsupported types/shape");
        return nullptr;
    }
    const MoePlan &p = m->p;
    if (upload_rows(m->gate, gu_type, Wg, p.rb_gu, p.ldw_gu, (size_t)ne_local * ffe, d, s) ||
        upload_rows(m->up, gu_type, Wu, p.rb_gu, p.ldw_gu, (size_t)ne_local * ffe, d, s) ||
        upload_rows(m->down, down_type, Wd, p.rb_down, p.ldw_down, (size_t)ne_local * d, ffe, s) ||
        upload_rows(m->sg, gu_type, Wsg, p.rb_gu, p.ldw_gu, ffe, d, s) ||
        upload_rows(m->su, gu_type, Wsu, p.rb_gu, p.ldw_gu, ffe, d, s) ||
        upload_rows(m->sd, down_type, Wsd, p.rb_down, p.ldw_down, d, ffe, s) ||
        cudaMalloc(&m->act.p, (size_t)MOE_MAXT * (k + 1) * ffe * 4) != cudaSuccess ||
        cudaMemset(m->act.p, 0, (size_t)MOE_MAXT * (k + 1) * ffe * 4) != cudaSuccess ||
        cudaMalloc(&m->route.p, MOE_ROUTE_WORDS * 4) != cudaSuccess ||
        cudaMalloc(&m->sync.p, MOE_SYNC_WORDS * 4) != cudaSuccess ||
        cudaMemset(m->sync.p, 0, MOE_SYNC_WORDS * 4) != cudaSuccess) {
        delete m;
        if (err().empty()) fail("moe: device allocation failed");
        return nullptr;
    }
    m->w = MoeWeights{m->gate.as<uint8_t>(), m->up.as<uint8_t>(), m->down.as<uint8_t>(),
                      m->sg.as<uint8_t>(), m->su.as<uint8_t>(), m->sd.as<uint8_t>()};
    return m;
}

}  // namespace fn

using namespace fn;

// One MoE layer on host buffers: routed experts stacked by expert (gate/up ne * ffe GGUF rows of
// d columns, down ne * d rows of ffe columns), shared expert (ffe / d rows), logits [nt][ne + 1] (column ne: the
// shared-gate logit), x [nt][d] -> y [nt][d]; sel / wsel [nt][k] (nullable) receive the routing.
FN_API int fn_test_moe(uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d, int nt, const uint8_t *Wg,
                       const uint8_t *Wu, const uint8_t *Wd, const uint8_t *Wsg, const uint8_t *Wsu, const uint8_t *Wsd,
                       const float *logits, const float *x, float *y, int *sel, float *wsel) {
    if (nt < 1 || nt > MOE_MAXT) return fail("fn_test_moe: nt out of range (1..32)");
    FN_CK(cudaSetDevice(hook_device()));
    cudaStream_t s = hook_stream();
    MoeH *m = moe_build(gu_type, down_type, ne, k, ffe, d, Wg, Wu, Wd, Wsg, Wsu, Wsd, s);
    if (!m) return -1;
    DevBuf lg, xd, yd, sd, wd;
    int rc = 0;
    if (cudaMalloc(&lg.p, (size_t)nt * (ne + 1) * 4) != cudaSuccess || cudaMalloc(&xd.p, (size_t)nt * d * 4) != cudaSuccess ||
        cudaMalloc(&yd.p, (size_t)nt * d * 4) != cudaSuccess || cudaMalloc(&sd.p, (size_t)nt * k * 4) != cudaSuccess ||
        cudaMalloc(&wd.p, (size_t)nt * k * 4) != cudaSuccess)
        rc = fail("fn_test_moe: device allocation failed");
    if (!rc && (cudaMemcpyAsync(lg.p, logits, (size_t)nt * (ne + 1) * 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
                cudaMemcpyAsync(xd.p, x, (size_t)nt * d * 4, cudaMemcpyHostToDevice, s) != cudaSuccess))
        rc = fail("fn_test_moe: copy failed");
    if (!rc)
        rc = launch_moe(m->p, m->w, lg.as<float>(), ne + 1, xd.as<float>(), m->act.as<float>(), m->route.as<uint32_t>(),
                        yd.as<float>(), nt, false, sd.as<int>(), wd.as<float>(), true, s, nullptr, false,
                        m->sync.as<uint32_t>());
    if (!rc) {
        cudaMemcpyAsync(y, yd.p, (size_t)nt * d * 4, cudaMemcpyDeviceToHost, s);
        if (sel) cudaMemcpyAsync(sel, sd.p, (size_t)nt * k * 4, cudaMemcpyDeviceToHost, s);
        if (wsel) cudaMemcpyAsync(wsel, wd.p, (size_t)nt * k * 4, cudaMemcpyDeviceToHost, s);
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) rc = fail(std::string("fn_test_moe: ") + cudaGetErrorString(e));
    }
    cudaStreamSynchronize(s);
    delete m;
    if (rc) return rc;
    return check_dev_error("fn_test_moe");
}

// Resident MoE weights on the current device (same arguments as fn_test_moe); returns a handle >= 1 or -1.
FN_API int fn_moe_create(uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d, const uint8_t *Wg,
                         const uint8_t *Wu, const uint8_t *Wd, const uint8_t *Wsg, const uint8_t *Wsu, const uint8_t *Wsd) {
    MoeH *m = moe_build(gu_type, down_type, ne, k, ffe, d, Wg, Wu, Wd, Wsg, Wsu, Wsd, 0);
    if (!m) return -1;
    if (cudaDeviceSynchronize() != cudaSuccess) {
        delete m;
        return fail("fn_moe_create: upload failed");
    }
    std::lock_guard<std::mutex> l(g_moe_mu);
    g_moe.push_back(m);
    return (int)g_moe.size();
}

FN_API int fn_moe_free(int h) {
    MoeH *m = moe_get(h);
    if (!m) return fail("fn_moe_free: bad handle");
    delete m;
    std::lock_guard<std::mutex> l(g_moe_mu);
    g_moe[h - 1] = nullptr;
    return 0;
}

// L2 prefetch hint of a MoE layer: from now on its down kernel (the layer's last) also brings [ptr, ptr + bytes) into
// L2 before its wait (as fn_w_prefetch_after; typically the next layer's input projection).
FN_API int fn_moe_prefetch_after(int h, const void *ptr, uint64_t bytes) {
    MoeH *m = moe_get(h);
    if (!m) return fail("fn_moe_prefetch_after: bad handle");
    if ((uintptr_t)ptr & 15) return fail("fn_moe_prefetch_after: ptr must be 16-byte aligned");
    m->p.pf = (const uint8_t *)ptr;
    m->p.pf_bytes = ptr ? (bytes & ~15ull) : 0;
    return 0;
}

// RMSNorm folded into MoE layer h: from now on the layer's input is rmsnorm(x) * w (rsqrt(mean x^2 + eps)), computed
// by the gate/up kernel from the raw x it reads (no separate norm launch). w: d floats of device memory, 16-byte
// aligned, kept by reference; NULL turns it off.
FN_API int fn_moe_norm(int h, const float *w, float eps) {
    MoeH *m = moe_get(h);
    if (!m) return fail("fn_moe_norm: bad handle");
    if ((uintptr_t)w & 15) return fail("fn_moe_norm: w must be 16-byte aligned");
    m->p.nw = w;
    m->p.eps = eps;
    return 0;
}

// Launch one MoE layer on device pointers: logits [nt][ls] (ls >= ne + 1), x [nt][d] -> y [nt][d]. flags: bit 0 adds
// into y; bit 1 = x early: x was complete before the kernel before this call started (so the layer reads it without
// waiting for that kernel, as an early GEMV does; engine/faie2fn.cu:2247-2249).
FN_API int fn_moe_run(int h, const float *logits, int ls, const float *x, float *y, int nt, int acc, void *stream) {
    MoeH *m = moe_get(h);
    if (!m) return fail("fn_moe_run: bad handle");
    if (m->group) return fail("fn_moe_run: an expert-parallel handle runs with fn_moe_ep_run");
    return launch_moe(m->p, m->w, logits, ls, x, m->act.as<float>(), m->route.as<uint32_t>(), y, nt, (acc & 1) != 0,
                      nullptr, nullptr, true, (cudaStream_t)stream, nullptr, (acc & 2) != 0, m->sync.as<uint32_t>());
}

// Expert-parallel MoE layer on a peer group (one rank per GPU): this rank holds routed experts
// [rank ne / n, (rank + 1) ne / n) (Wg, Wu: those experts' ffe rows each; Wd: their d rows each, GGUF rows as in
// fn_moe_create) and the whole shared expert. Returns a handle >= 1 or -1.
FN_API int fn_moe_ep_create(uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d, int group,
                            const uint8_t *Wg, const uint8_t *Wu, const uint8_t *Wd, const uint8_t *Wsg,
                            const uint8_t *Wsu, const uint8_t *Wsd) {
    PeerGroup *g = peer_group(group);
    if (!g) return fail("fn_moe_ep_create: bad group");
    if ((size_t)PEER_MOE + (size_t)2 * MOE_EP_MAXT * (k + 1) * d * 4 > g->bytes)
        return fail("fn_moe_ep_create: the group's buffers are too small for the slot outputs");
    const int e0 = (int)((long long)g->rank * ne / g->n), e1 = (int)((long long)(g->rank + 1) * ne / g->n);
    MoeH *m = moe_build(gu_type, down_type, ne, k, ffe, d, Wg, Wu, Wd, Wsg, Wsu, Wsd, 0, e1 - e0);
    if (!m) return -1;
    if (cudaDeviceSynchronize() != cudaSuccess) {
        delete m;
        return fail("fn_moe_ep_create: upload failed");
    }
    m->group = group;
    m->e0 = e0;
    std::lock_guard<std::mutex> l(g_moe_mu);
    g_moe.push_back(m);
    return (int)g_moe.size();
}

// Launch one expert-parallel MoE layer (device pointers, replicated on every rank): logits [nt][ls], x [nt][d] ->
// y [nt][d] (+= if acc) on every rank. Every rank makes the same calls in the same order.
FN_API int fn_moe_ep_run(int h, const float *logits, int ls, const float *x, float *y, int nt, int acc, void *stream) {
    MoeH *m = moe_get(h);
    if (!m || !m->group) return fail("fn_moe_ep_run: bad handle");
    PeerGroup *g = peer_group(m->group);
    if (!g) return fail("fn_moe_ep_run: the group is gone");
    MoeEp ep;
    ep.n = g->n;
    ep.rank = g->rank;
    ep.e0 = m->e0;
    for (int r = 0; r < g->n; ++r) {
        ep.dpart[r] = (float *)(g->base[r] + PEER_MOE);
        ep.counters[r] = (uint32_t *)(g->base[r] + PEER_MOE_COUNTERS);
    }
    ep.calls = g->local_calls + 2;
    return launch_moe(m->p, m->w, logits, ls, x, m->act.as<float>(), m->route.as<uint32_t>(), y, nt, (acc & 1) != 0,
                      nullptr, nullptr, true, (cudaStream_t)stream, &ep, (acc & 2) != 0);
}

// Routing on router outputs given as split-K partials part[ks][8][528] (the reference's router + shared-gate GEMV
// output layout: 512 router rows, row stride 528): sel / wsel [nt][10] of nt <= 8 tokens and the time per call
// (iters calls replayed as one CUDA graph). variant 0: the reference's order counted out expert by expert (the
// role of k_route_ref, :1697-1740), 1: the engine's routing (k_route's role), bit-identical. Replaces fn_bench_route
// (engine/faie2fn.cu:2873-2912).
FN_API int fn_bench_route(int variant, int nt, int ks, const float *parth, int iters, int *selh, float *wselh, float *ms) {
    constexpr int NE = 512, NEU = 10, MAXT = 8, RSG = 528;
    if (variant < 0 || variant > 1 || nt < 1 || nt > MAXT || ks < 1 || iters < 1) return fail("fn_bench_route: bad arguments");
    FN_CK(cudaSetDevice(hook_device()));
    cudaStream_t st = hook_stream();
    DevBuf part, sel, w;
    const size_t np = (size_t)ks * MAXT * RSG;
    FN_CK(cudaMalloc(&part.p, np * 4));
    FN_CK(cudaMalloc(&sel.p, MAXT * NEU * 4));
    FN_CK(cudaMalloc(&w.p, MAXT * NEU * 4));
    FN_CK(cudaMemcpyAsync(part.p, parth, np * 4, cudaMemcpyHostToDevice, st));
    FN_CK(cudaStreamSynchronize(st));
    cudaGraph_t g;
    cudaGraphExec_t ge;
    FN_CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    int rc = 0;
    for (int i = 0; i < iters && !rc; ++i)
        rc = launch_route(variant, part.as<float>(), ks, (size_t)MAXT * RSG, RSG, NE, NEU, nt, sel.as<int>(), w.as<float>(), st);
    cudaError_t ce = cudaStreamEndCapture(st, &g);
    if (rc) return rc;
    FN_CK(ce);
    FN_CK(cudaGraphInstantiate(&ge, g, 0));
    FN_CK(cudaGraphLaunch(ge, st));
    cudaEvent_t a, b;
    FN_CK(cudaEventCreate(&a));
    FN_CK(cudaEventCreate(&b));
    FN_CK(cudaEventRecord(a, st));
    FN_CK(cudaGraphLaunch(ge, st));
    FN_CK(cudaEventRecord(b, st));
    FN_CK(cudaEventSynchronize(b));
    FN_CK(cudaEventElapsedTime(ms, a, b));
    *ms /= iters;
    FN_CK(cudaMemcpy(selh, sel.p, (size_t)nt * NEU * 4, cudaMemcpyDeviceToHost));
    FN_CK(cudaMemcpy(wselh, w.p, (size_t)nt * NEU * 4, cudaMemcpyDeviceToHost));
    cudaGraphExecDestroy(ge);
    cudaGraphDestroy(g);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return 0;
}

// ---- the MoE layer without any allocation --------------------------------------------------------------------------
//
// Some callers cannot call cudaMalloc: a host that owns all device memory through its own pool (an inference server,
// a framework allocator) and forbids raw allocations, or code that must not pay the implicit device-wide
// synchronisation cudaFree performs in the middle of a decode loop. fn_moe_layer_static takes every input and output
// as a device pointer the caller already owns and keeps its only scratch, the tokens' routing (written by the routing
// kernel, read by the others) and the activations passed from the gate/up kernel to the down kernel, in a fixed array
// of device memory that is part of the library image.
//
// Limits: 1 <= nt <= 32 tokens and nt * (k + 1) * ffe <= 65536 floats (256 KiB of activations); larger calls are
// rejected. Every GPU that loads the library holds the array until the process exits. All calls share it, so calls
// whose kernels overlap on the GPU (two streams, or two host threads) race on it: issue them in one stream. Nothing in
// it needs to start at zero (each kernel writes every element the next one reads). The first call on a device (and the
// first after that device's context was re-created, e.g. by cudaDeviceReset) resolves the array's device address in
// the current context (cudaGetSymbolAddress); make that first call outside stream capture.

namespace fn {
constexpr size_t kMoeStaticActFloats = 65536;
// activations, then the routing words
static __device__ __align__(256) float g_moe_static_act[kMoeStaticActFloats + MOE_ROUTE_WORDS];
// device address of g_moe_static_act per device, and the context it was resolved in
static float *g_moe_static_act_dev[64] = {};
static CUcontext g_moe_static_ctx[64] = {};
// the driver's cuCtxGetCurrent, looked up through the runtime (the library does not link the driver library itself)
static CUresult current_context(CUcontext *ctx) {
    using Fn = CUresult (*)(CUcontext *);
    static Fn f = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (Fn) nullptr;
        return (Fn)p;
    }();
    return f ? f(ctx) : CUDA_ERROR_NOT_FOUND;
}
}  // namespace fn

FN_API int fn_moe_layer_static(uint32_t gu_type, uint32_t down_type, int ne, int k, int ffe, int d, const uint8_t *Wg,
                               const uint8_t *Wu, const uint8_t *Wd, const uint8_t *Wsg, const uint8_t *Wsu,
                               const uint8_t *Wsd, const float *logits, int ls, const float *x, float *y, int nt,
                               void *stream) {
    MoePlan p;
    if (!plan_moe(p, gu_type, down_type, ne, k, ffe, d)) return fail("fn_moe_layer_static: unsupported types/shape");
    if (nt < 1 || nt > MOE_MAXT) return fail("fn_moe_layer_static: nt out of range (1..32)");
    const size_t need = (size_t)nt * (k + 1) * ffe;
    if (need > kMoeStaticActFloats)
        return fail("fn_moe_layer_static: nt * (k + 1) * ffe = " + std::to_string(need) +
                    " floats exceeds the static scratch of " + std::to_string(kMoeStaticActFloats) + " floats");
    const uint8_t *ws[6] = {Wg, Wu, Wd, Wsg, Wsu, Wsd};
    for (const uint8_t *w : ws)
        if (!w || ((uintptr_t)w & 15)) return fail("fn_moe_layer_static: weight pointers must be 16-byte aligned");
    int dev = 0;
    FN_CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail("fn_moe_layer_static: device index out of range");
    CUcontext ctx = nullptr;
    FN_CK(cudaFree(nullptr));  // makes the device's primary context current (allocates nothing)
    if (current_context(&ctx) != CUDA_SUCCESS || !ctx) return fail("fn_moe_layer_static: no current CUDA context");
    if (!g_moe_static_act_dev[dev] || g_moe_static_ctx[dev] != ctx) {
        void *ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_moe_static_act);
        if (e != cudaSuccess) return fail(std::string("fn_moe_layer_static: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        g_moe_static_act_dev[dev] = (float *)ptr;
        g_moe_static_ctx[dev] = ctx;
    }
    const MoeWeights w{Wg, Wu, Wd, Wsg, Wsu, Wsd};
    return launch_moe(p, w, logits, ls, x, g_moe_static_act_dev[dev],
                      (uint32_t *)(g_moe_static_act_dev[dev] + kMoeStaticActFloats), y, nt, false, nullptr, nullptr,
                      /*planes=*/false, (cudaStream_t)stream);
}
