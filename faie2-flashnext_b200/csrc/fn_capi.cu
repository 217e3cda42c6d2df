// C ABI of the engine (declared in include/faie2fn.h): errors, launch settings, the model-free test / bench hooks of
// the reference (engine/faie2fn.cu:2492-2935) and resident-weight handles for device-pointer callers.
// Conventions of the reference are kept: int return 0 = ok, -1 = error with the message in fn_error(); the caller
// owns every host buffer; every fn_test_* / fn_bench_* call is synchronous.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "fn_engine.h"
#include "fn_peer.h"

namespace fn {

std::string &err() {
    static std::string e;
    return e;
}
int fail(const std::string &msg) {
    err() = msg;
    return -1;
}

Settings &settings() {
    static Settings s = [] {
        Settings v;
        if (const char *e = getenv("FN_PDL")) v.pdl = atoi(e) != 0;  // FN_PDL=0: no programmatic launch (profiling)
        return v;
    }();
    return s;
}

int num_sms() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

// One error word per device, in a static __device__ variable (no allocation); kernels record the first failure.
__device__ uint32_t g_dev_err_word;
static uint32_t *g_err_ptr[64] = {};

uint32_t *dev_error_ptr() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!g_err_ptr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_dev_err_word) != cudaSuccess) return nullptr;
        g_err_ptr[dev] = (uint32_t *)p;
    }
    return g_err_ptr[dev];
}

int check_dev_error(const char *where) {
    uint32_t v = 0;
    FN_CK(cudaMemcpyFromSymbol(&v, g_dev_err_word, sizeof(v)));
    if (v == DEV_OK) return 0;
    const uint32_t z = 0;
    cudaMemcpyToSymbol(g_dev_err_word, &z, sizeof(z));
    return fail(std::string(where) + ": device " +
                (v == DEV_WAIT_TIMEOUT    ? "wait timed out (a pipeline barrier never completed)"
                 : v == DEV_PEER_TIMEOUT ? "wait for a peer GPU timed out (a rank did not arrive)"
                                         : "argument check failed") +
                " (code " + std::to_string(v) + ")");
}

static int g_device = -1;  // device the test / bench hooks use (FN_DEVICE, default 0)
int hook_device() {
    if (g_device < 0) {
        const char *e = getenv("FN_DEVICE");
        g_device = e ? atoi(e) : 0;
    }
    return g_device;
}

// a non-blocking stream per device for the synchronous hooks
cudaStream_t hook_stream() {
    static cudaStream_t st[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!st[dev]) cudaStreamCreateWithFlags(&st[dev], cudaStreamNonBlocking);
    return st[dev];
}


// ---- resident weights ------------------------------------------------------------------------------------------
struct WeightH {
    GemvPlan plan1, plan8;  // token capacity 1 and 8
    uint8_t *d = nullptr;   // rows at stride plan.ldw
    int dev = 0;
    float *xbuf = nullptr, *ybuf = nullptr;  // device staging for host-buffer calls
    unsigned long long *kacc = nullptr;      // fused-argmax key maxima [8] and ticket (zero between launches)
    unsigned int *ticket = nullptr;
    int *ibuf = nullptr;                     // device staging of host-buffer argmax calls [8]
};
static std::vector<WeightH *> g_w;
static std::mutex g_w_mu;

static WeightH *wget(int h) {
    std::lock_guard<std::mutex> l(g_w_mu);
    return h >= 1 && h <= (int)g_w.size() ? g_w[h - 1] : nullptr;
}

// a decode step's GEMVs on host buffers (fn_w_step_host)
struct StepPlan {
    DevBuf x, y;  // staging: the inputs back to back, then the outputs back to back (+ one int for the argmax)
    size_t xn = 0, yn = 0;
    cudaGraphExec_t exec = nullptr;
    ~StepPlan() {
        if (exec) cudaGraphExecDestroy(exec);
    }
};
static std::map<std::vector<int>, StepPlan *> g_steps;
static std::mutex g_steps_mu;

static int build_step(const std::vector<int> &key, int n, const int *handles, int head, StepPlan *sp) {
    size_t xn = 0, yn = 0;
    for (int i = 0; i < n; ++i) {
        WeightH *w = wget(handles[i]);
        if (!w) return fail("fn_w_step_host: bad handle " + std::to_string(handles[i]));
        xn += (size_t)w->plan1.cols;
        if (i != head) yn += (size_t)w->plan1.rows;
    }
    sp->xn = xn;
    sp->yn = yn;
    FN_CK(cudaMalloc(&sp->x.p, std::max<size_t>(xn, 1) * 4));
    FN_CK(cudaMalloc(&sp->y.p, (yn + 4) * 4));
    // The GEMVs are independent (inputs from the host copy, outputs to the host copy): they run as kStepBranches
    // concurrent chains of the graph (fork from the capture stream, join back), several resident on an SM at once.
    constexpr int kStepBranches = 8;
    cudaStream_t cap, side[kStepBranches];
    cudaEvent_t fork, join[kStepBranches];
    FN_CK(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
    for (int b = 0; b < kStepBranches; ++b) {
        FN_CK(cudaStreamCreateWithFlags(&side[b], cudaStreamNonBlocking));
        FN_CK(cudaEventCreateWithFlags(&join[b], cudaEventDisableTiming));
    }
    FN_CK(cudaEventCreateWithFlags(&fork, cudaEventDisableTiming));
    cudaGraph_t g = nullptr;
    int rc = 0;
    if (cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) rc = fail("fn_w_step_host: capture");
    if (!rc && cudaEventRecord(fork, cap) != cudaSuccess) rc = fail("fn_w_step_host: fork");
    for (int b = 0; b < kStepBranches && !rc; ++b)
        if (cudaStreamWaitEvent(side[b], fork, 0) != cudaSuccess) rc = fail("fn_w_step_host: fork");
    size_t xo = 0, yo = 0;
    for (int i = 0; i < n && !rc; ++i) {
        WeightH *w = wget(handles[i]);
        const GemvPlan &p = w->plan1;
        cudaStream_t s = side[i % kStepBranches];
        // inputs come from the copy before the graph: every GEMV may read its x before waiting
        if (i == head) {
            GemvArgmax am;
            am.index = (int *)(sp->y.as<float>() + yn);
            am.kacc = w->kacc;
            am.ticket = w->ticket;
            rc = launch_gemv(p, w->d, sp->x.as<float>() + xo, p.cols, nullptr, p.rows, 1, false, true, s, &am);
        } else {
            rc = launch_gemv(p, w->d, sp->x.as<float>() + xo, p.cols, sp->y.as<float>() + yo, p.rows, 1, false, true, s);
            yo += (size_t)p.rows;
        }
        xo += (size_t)p.cols;
    }
    for (int b = 0; b < kStepBranches && !rc; ++b)
        if (cudaEventRecord(join[b], side[b]) != cudaSuccess || cudaStreamWaitEvent(cap, join[b], 0) != cudaSuccess)
            rc = fail("fn_w_step_host: join");
    const cudaError_t ce = cudaStreamEndCapture(cap, &g);
    if (!rc && ce != cudaSuccess) rc = fail(std::string("fn_w_step_host: capture: ") + cudaGetErrorString(ce));
    if (!rc && cudaGraphInstantiate(&sp->exec, g, 0) != cudaSuccess) rc = fail("fn_w_step_host: graph instantiate");
    if (g) cudaGraphDestroy(g);
    for (int b = 0; b < kStepBranches; ++b) {
        cudaStreamDestroy(side[b]);
        cudaEventDestroy(join[b]);
    }
    cudaEventDestroy(fork);
    cudaStreamDestroy(cap);
    (void)key;
    return rc;
}

}  // namespace fn

using namespace fn;

FN_API const char *fn_error() { return err().c_str(); }

FN_API int fn_set_device(int dev) {
    int n = 0;
    FN_CK(cudaGetDeviceCount(&n));
    if (dev < 0 || dev >= n) return fail("fn_set_device: no device " + std::to_string(dev));
    g_device = dev;
    FN_CK(cudaSetDevice(dev));
    return 0;
}

// ---- launch settings (engine/faie2fn.cu:2786-2807) ---------------------------------------------------------------
FN_API void fn_pdl(int on) { settings().pdl = on != 0; }
FN_API void fn_early(int on) { settings().early = on != 0; }
FN_API void fn_bench_hot(int on) { settings().bench_hot = on; }
// GEMV plan settings for weights planned from now on: warps per CTA (0: automatic, < 0 keeps), ring KiB, stage KiB,
// CTAs per SM (0 = keep)
FN_API void fn_gemv_tune(int warps, int ring_kb, int stage_kb, int ctas_per_sm) {
    Settings &s = settings();
    if (warps >= 0) s.warps_per_cta = warps;  // 0: automatic
    if (ring_kb > 0) s.ring_kb = ring_kb;
    if (stage_kb > 0) s.stage_kb = stage_kb;
    if (ctas_per_sm > 0) s.ctas_per_sm = ctas_per_sm;
}
// The reference's plan override (engine/faie2fn.cu:2786-2791) with its argument meaning: tb = threads per CTA of the
// GEMVs planned from now on (0: automatic), warps_per_sm = the target warps per SM (the reference's default 16: one
// CTA of 16 warps per SM). wpt (weights per thread of a tile) and ks (split-K) have no counterpart in this plan, where
// a row never spans warps; they are accepted and ignored.
FN_API void fn_gemv_override(int wpt, int ks, int tb, int warps_per_sm) {
    (void)wpt;
    (void)ks;
    Settings &s = settings();
    const int warps = tb > 0 ? std::max(1, std::min(16, tb / 32)) : 0;
    s.warps_per_cta = warps;
    s.ctas_per_sm = warps > 0 && warps_per_sm > 0 ? std::max(1, warps_per_sm / warps) : 1;
}
// MoE layer variant (the reference's A/B switch, engine/faie2fn.cu:2799): 0 = a routing kernel before gate/up
// (default: measured faster on the config-5 decode step, 2.99 against 3.18 ms per token), 1 = one token on one GPU
// routed inside the gate/up and down kernels
FN_API void fn_moe_var(int v) { settings().moe_var = v; }
// Q4_K / Q6_K GEMVs of 1..4 tokens (rows up to 2048 columns) as exact integer products on the tensor cores (1) or on
// the CUDA cores (0, the default)
FN_API void fn_qmma(int on) { settings().qmma = on != 0; }
// The reference's routed-expert launch shapes (engine/faie2fn.cu:2801-2806). The B200 MoE kernels size their grids
// and rings from the layer's shape and the SM count, so there is nothing to override: accepted and ignored.
FN_API void fn_moe_override(int gu_wpt, int gu_tb, int dn_wpt, int dn_tb) {
    (void)gu_wpt;
    (void)gu_tb;
    (void)dn_wpt;
    (void)dn_tb;
}
FN_API void fn_gemv_waves(int ctas_per_sm) { settings().ctas_per_sm = ctas_per_sm > 0 ? ctas_per_sm : 1; }

// plan of a weight: out = {lpr, gpl, rows per stage, ring slots, CTAs, threads, row stride bytes}
FN_API int fn_gemv_plan(uint32_t type, int rows, int cols, int *out) {
    if (cudaSetDevice(hook_device()) != cudaSuccess) return fail("fn_gemv_plan: no CUDA device");
    GemvPlan p;
    if (!plan_gemv(p, type, rows, cols, 1)) return fail("unsupported type/shape");
    const int v[7] = {p.lpr, p.gpl, p.rps, p.slots, p.ctas, p.threads, (int)p.ldw};
    memcpy(out, v, sizeof(v));
    return 0;
}

// ---- model-free test hooks (engine/faie2fn.cu:2745-2782, 2914-2935) -----------------------------------------------

// out[r][c] = dequant of GGUF rows W (rows x row_bytes(type, cols))
FN_API int fn_test_dequant(uint32_t type, const uint8_t *Wh, int rows, int cols, float *outh) {
    const uint64_t rb = row_bytes(type, cols);
    if (!rb || cols % 32 || rows < 0) return fail("unsupported type/shape");
    if (rows == 0) return 0;
    FN_CK(cudaSetDevice(hook_device()));
    cudaStream_t s = hook_stream();
    DevBuf W, out;
    FN_CK(cudaMalloc(&W.p, rb * rows));
    FN_CK(cudaMalloc(&out.p, (size_t)rows * cols * 4));
    FN_CK(cudaMemcpyAsync(W.p, Wh, rb * rows, cudaMemcpyHostToDevice, s));
    if (launch_dequant(type, W.as<uint8_t>(), rb, rows, cols, out.as<float>(), s)) return -1;
    FN_CK(cudaMemcpyAsync(outh, out.p, (size_t)rows * cols * 4, cudaMemcpyDeviceToHost, s));
    FN_CK(cudaStreamSynchronize(s));
    return 0;
}

// y[t][r] = W[r] . x[t], t < nt <= 8, on GGUF rows W: uploaded to the engine's row layout, then the engine's GEMV
FN_API int fn_test_gemv(uint32_t type, const uint8_t *Wh, int rows, int cols, const float *xh, int nt, float *yh) {
    GemvPlan p;
    if (nt < 1 || nt > 8) return fail("nt out of range (1..8)");
    FN_CK(cudaSetDevice(hook_device()));
    if (!plan_gemv(p, type, rows, cols, nt == 1 ? 1 : 8)) return fail("unsupported type/shape");
    cudaStream_t s = hook_stream();
    DevBuf W, x, y;
    DevBuf raw;
    FN_CK(cudaMalloc(&W.p, plan_weight_bytes(p)));
    FN_CK(cudaMalloc(&raw.p, (size_t)p.rb * rows));
    FN_CK(cudaMalloc(&x.p, (size_t)nt * cols * 4));
    FN_CK(cudaMalloc(&y.p, (size_t)nt * rows * 4));
    FN_CK(cudaMemcpyAsync(raw.p, Wh, (size_t)p.rb * rows, cudaMemcpyHostToDevice, s));
    if (launch_plane_repack(type, raw.as<uint8_t>(), p.rb, W.as<uint8_t>(), p.ldw, rows, cols, s)) return -1;
    FN_CK(cudaMemcpyAsync(x.p, xh, (size_t)nt * cols * 4, cudaMemcpyHostToDevice, s));
    if (launch_gemv(p, W.as<uint8_t>(), x.as<float>(), cols, y.as<float>(), rows, nt, false, false, s)) return -1;
    FN_CK(cudaMemcpyAsync(yh, y.p, (size_t)nt * rows * 4, cudaMemcpyDeviceToHost, s));
    FN_CK(cudaStreamSynchronize(s));
    return check_dev_error("fn_test_gemv");
}

// GEMV timing on hash-random bytes of a format with the weights cold in L2 (as in a forward, where each weight is
// read once): `copies` rotating copies whose total exceeds twice the L2, `iters` calls captured in one CUDA graph,
// one warm-up replay, an L2 flush, then one timed replay. ms per call (engine/faie2fn.cu:2817-2866).
// Seeded GGUF rows of `type` as the benchmark's synthetic weights: uniform random bytes, the fp16
// scale fields of every block overwritten with finite |N(0,1)| 1e-3 values (here |u1 + u2 + u3 - 1.5| 2e-3 of three
// uniforms, a bell-shaped stand-in), BF16 rows as small normal values; x values likewise bell-shaped around 0. A
// 64-bit linear congruential generator makes the bytes.
namespace fn {
struct Lcg {
    uint64_t s;
    uint32_t next() {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        return (uint32_t)(s >> 33);
    }
    float uni() { return (float)(next() >> 8) * (1.0f / 16777216.0f); }
    float bell() { return uni() + uni() + uni() - 1.5f; }
};
static int scale_offsets(uint32_t t, int *off) {
    switch (t) {
        case T_Q4_1: case T_Q5_1: case T_Q4_K: case T_Q5_K: off[0] = 0; off[1] = 2; return 2;
        case T_Q2_K: off[0] = 80; off[1] = 82; return 2;
        case T_Q3_K: off[0] = 108; return 1;
        case T_Q6_K: off[0] = 208; return 1;
        case T_BF16: return 0;
        default: off[0] = 0; return 1;
    }
}
static std::vector<uint8_t> bench_rows(uint32_t type, int rows, int cols, uint64_t seed) {
    const uint64_t rb = row_bytes(type, cols);
    std::vector<uint8_t> h((size_t)rb * rows);
    Lcg g{seed};
    if (type == T_BF16) {
        for (size_t i = 0; i < h.size() / 2; ++i) {
            const float v = g.bell() * 0.1f;
            uint32_t u;
            std::memcpy(&u, &v, 4);
            const uint16_t b = (uint16_t)(u >> 16);
            std::memcpy(&h[2 * i], &b, 2);
        }
        return h;
    }
    for (auto &b : h) b = (uint8_t)g.next();
    int qk, tb, off[2];
    type_info(type, qk, tb);
    const int nf = scale_offsets(type, off);
    for (size_t blk = 0; blk < h.size() / tb; ++blk)
        for (int f = 0; f < nf; ++f) {
            const __half d = __float2half(fabsf(g.bell()) * 2e-3f);
            std::memcpy(&h[blk * tb + off[f]], &d, 2);
        }
    return h;
}
}  // namespace fn

FN_API int fn_bench_gemv(uint32_t type, int rows, int cols, int nt, int iters, float *ms) {
    GemvPlan p;
    if (nt < 1 || nt > 8 || iters < 1) return fail("nt/iters out of range");
    FN_CK(cudaSetDevice(hook_device()));
    if (!plan_gemv(p, type, rows, cols, nt == 1 ? 1 : 8)) return fail("unsupported type/shape");
    int dev = 0, l2 = 0;
    FN_CK(cudaGetDevice(&dev));
    FN_CK(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev));
    const size_t wb = plan_weight_bytes(p);
    const bool hot = settings().bench_hot != 0;
    int copies = hot ? 1 : (int)std::min<size_t>((size_t)iters, std::max<size_t>(2, (2 * (size_t)l2) / wb + 1));
    while (copies > 1 && wb * copies > (8ull << 30)) --copies;
    DevBuf W, x, y, flush;
    const size_t flush_n = 2 * (size_t)l2;
    FN_CK(cudaMalloc(&W.p, wb * copies));
    FN_CK(cudaMalloc(&x.p, (size_t)nt * cols * 4));
    FN_CK(cudaMalloc(&y.p, (size_t)nt * rows * 4));
    FN_CK(cudaMalloc(&flush.p, flush_n));
    {  // one copy of the weights in the engine's layout, then its duplicates; x bell-shaped around 0
        const std::vector<uint8_t> hb = bench_rows(type, rows, cols, 12345);
        DevBuf raw;
        FN_CK(cudaMalloc(&raw.p, hb.size()));
        FN_CK(cudaMemcpy(raw.p, hb.data(), hb.size(), cudaMemcpyHostToDevice));
        if (launch_plane_repack(type, raw.as<uint8_t>(), p.rb, W.as<uint8_t>(), p.ldw, rows, cols, 0)) return -1;
        FN_CK(cudaDeviceSynchronize());
        for (int c = 1; c < copies; ++c) FN_CK(cudaMemcpy(W.as<uint8_t>() + wb * c, W.p, wb, cudaMemcpyDeviceToDevice));
        std::vector<float> hx((size_t)nt * cols);
        Lcg g{777};
        for (float &v : hx) v = g.bell() * 2.0f;
        FN_CK(cudaMemcpy(x.p, hx.data(), hx.size() * 4, cudaMemcpyHostToDevice));
    }
    cudaStream_t st = hook_stream();
    cudaGraph_t g;
    cudaGraphExec_t ge;
    FN_CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    int rc = 0;
    for (int i = 0; i < iters && !rc; ++i)
        rc = launch_gemv(p, W.as<uint8_t>() + wb * (i % copies), x.as<float>(), cols, y.as<float>(), rows, nt, false, false, st);
    cudaError_t ce = cudaStreamEndCapture(st, &g);
    if (rc) return -1;
    FN_CK(ce);
    FN_CK(cudaGraphInstantiate(&ge, g, 0));
    cudaEvent_t a, b;
    FN_CK(cudaEventCreate(&a));
    FN_CK(cudaEventCreate(&b));
    FN_CK(cudaGraphLaunch(ge, st));
    if (!hot) FN_CK(cudaMemsetAsync(flush.p, 1, flush_n, st));
    FN_CK(cudaEventRecord(a, st));
    FN_CK(cudaGraphLaunch(ge, st));
    FN_CK(cudaEventRecord(b, st));
    FN_CK(cudaEventSynchronize(b));
    FN_CK(cudaEventElapsedTime(ms, a, b));
    *ms /= iters;
    cudaGraphExecDestroy(ge);
    cudaGraphDestroy(g);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return check_dev_error("fn_bench_gemv");
}

// ---- resident weights (device-pointer API for the bench and the engine's callers) --------------------------------

// Upload GGUF rows (rows x row_bytes(type, cols), host memory) to the current device in the engine's layout.
// Returns a handle >= 1, or -1.
FN_API int fn_w_create(uint32_t type, const uint8_t *Wh, int rows, int cols) {
    WeightH *w = new WeightH();
    if (!plan_gemv(w->plan1, type, rows, cols, 1) || !plan_gemv(w->plan8, type, rows, cols, 8)) {
        delete w;
        return fail("fn_w_create: unsupported type/shape");
    }
    cudaGetDevice(&w->dev);
    const GemvPlan &p = w->plan1;
    DevBuf raw;
    if (cudaMalloc(&w->d, plan_weight_bytes(p)) != cudaSuccess || cudaMalloc(&raw.p, (size_t)p.rb * rows) != cudaSuccess ||
        cudaMemcpy(raw.p, Wh, (size_t)p.rb * rows, cudaMemcpyHostToDevice) != cudaSuccess ||
        launch_plane_repack(type, raw.as<uint8_t>(), p.rb, w->d, p.ldw, rows, cols, 0) != 0 ||
        cudaDeviceSynchronize() != cudaSuccess ||
        cudaMalloc(&w->xbuf, (size_t)8 * cols * 4) != cudaSuccess || cudaMalloc(&w->ybuf, (size_t)8 * rows * 4) != cudaSuccess ||
        cudaMalloc(&w->kacc, 256) != cudaSuccess || cudaMemset(w->kacc, 0, 256) != cudaSuccess ||
        cudaMalloc(&w->ticket, 256) != cudaSuccess || cudaMemset(w->ticket, 0, 256) != cudaSuccess ||
        cudaMalloc(&w->ibuf, 8 * sizeof(int)) != cudaSuccess) {
        cudaFree(w->d);
        cudaFree(w->xbuf);
        cudaFree(w->ybuf);
        cudaFree(w->kacc);
        cudaFree(w->ticket);
        cudaFree(w->ibuf);
        delete w;
        return fail("fn_w_create: device allocation/copy failed");
    }
    std::lock_guard<std::mutex> l(g_w_mu);
    g_w.push_back(w);
    return (int)g_w.size();
}

FN_API int fn_w_free(int h) {
    WeightH *w = wget(h);
    if (!w) return fail("fn_w_free: bad handle");
    {
        std::lock_guard<std::mutex> l(g_steps_mu);
        for (auto it = g_steps.begin(); it != g_steps.end();) {
            bool uses = false;
            for (size_t i = 0; i + 1 < it->first.size(); ++i) uses = uses || it->first[i] == h;
            if (uses) {
                delete it->second;
                it = g_steps.erase(it);
            } else {
                ++it;
            }
        }
    }
    cudaFree(w->d);
    cudaFree(w->xbuf);
    cudaFree(w->ybuf);
    cudaFree(w->kacc);
    cudaFree(w->ticket);
    cudaFree(w->ibuf);
    delete w;
    std::lock_guard<std::mutex> l(g_w_mu);
    g_w[h - 1] = nullptr;
    return 0;
}

// bytes the GEMV must read per call: the GGUF weight bytes (rows x row_bytes), the padding excluded
FN_API double fn_w_bytes(int h) {
    WeightH *w = wget(h);
    return w ? (double)w->plan1.rb * w->plan1.rows : -1.0;
}

// Launch y[t][r] (+)= W[r] . x[t] for t < nt on `stream` with device pointers (no synchronisation). flags: bit 0 = add
// into y; bit 1 = early: x was complete before the previous kernel in the stream started, so the GEMV reads it without
// waiting and waits for the previous kernel only before it exits (engine/faie2fn.cu:2247-2249); y must not be read by
// the previous kernel.
FN_API int fn_w_gemv(int h, const float *x, int xs, float *y, int ys, int nt, int flags, void *stream) {
    WeightH *w = wget(h);
    if (!w) return fail("fn_w_gemv: bad handle");
    if (nt < 1 || nt > 8) return fail("fn_w_gemv: nt out of range (1..8)");
    return launch_gemv(nt == 1 ? w->plan1 : w->plan8, w->d, x, xs, y, ys, nt, (flags & 1) != 0, (flags & 2) != 0,
                       (cudaStream_t)stream);
}

// Device address and size of a resident weight (its rows at the handle's 16-byte stride), e.g. for a prefetch hint.
FN_API int fn_w_weights(int h, const void **ptr, uint64_t *bytes) {
    WeightH *w = wget(h);
    if (!w) return fail("fn_w_weights: bad handle");
    *ptr = w->d;
    *bytes = plan_weight_bytes(w->plan1);
    return 0;
}

// L2 prefetch hint: from now on every launch of GEMV handle h also brings [ptr, ptr + bytes) of device memory into L2,
// spread over its CTAs, before its wait for the previous kernel (read-only data that a later kernel of the chain
// reads, typically the next weight of a decode step). ptr must be 16-byte aligned; bytes is rounded down to 16;
// ptr = NULL clears the hint. No counterpart in the reference (its decode reads every weight cold).
FN_API int fn_w_prefetch_after(int h, const void *ptr, uint64_t bytes) {
    WeightH *w = wget(h);
    if (!w) return fail("fn_w_prefetch_after: bad handle");
    if ((uintptr_t)ptr & 15) return fail("fn_w_prefetch_after: ptr must be 16-byte aligned");
    w->plan1.pf = w->plan8.pf = (const uint8_t *)ptr;
    w->plan1.pf_bytes = w->plan8.pf_bytes = ptr ? (bytes & ~15ull) : 0;
    return 0;
}

// RMSNorm folded into GEMV handle h: from now on every launch computes y[t] = rsqrt(mean x[t]^2 + eps) (W . (x[t] * w))
// from the raw x (the reference's k_groupnorm before the GEMV, engine/faie2fn.cu:1222-1235, without its launch): the
// sum of squares is taken while x is staged and the scale is applied to each row's result. w: cols floats of device
// memory, 16-byte aligned, kept by reference; w = NULL turns it off.
FN_API int fn_w_norm(int h, const float *w, float eps) {
    WeightH *wh = wget(h);
    if (!wh) return fail("fn_w_norm: bad handle");
    if ((uintptr_t)w & 15) return fail("fn_w_norm: w must be 16-byte aligned");
    wh->plan1.nw = wh->plan8.nw = w;
    wh->plan1.eps = wh->plan8.eps = eps;
    return 0;
}

// The lm_head GEMV with the fused argmax (k_argmax, engine/faie2fn.cu:1910-1935, folded into the GEMV's last CTA):
// y (nullable: logits not written) as fn_w_gemv; index[t] (nullable) = the lowest global row index of the largest
// value for token t, global index = row0 + local row; keys[t] (nullable, may be a peer GPU's memory) = the 64-bit
// ordering key of that winner, for combining the keys of a row-split lm_head by max (fn_argmax_keys). One such call at
// a time per handle (the key maxima and the ticket belong to the handle).
FN_API int fn_w_gemv_argmax(int h, const float *x, int xs, float *y, int ys, int nt, int flags, int row0, int *index,
                            unsigned long long *keys, void *stream) {
    WeightH *w = wget(h);
    if (!w) return fail("fn_w_gemv_argmax: bad handle");
    if (nt < 1 || nt > 8) return fail("fn_w_gemv_argmax: nt out of range (1..8)");
    GemvArgmax am;
    am.row0 = row0;
    am.index = index;
    am.key = keys;
    am.kacc = w->kacc;
    am.ticket = w->ticket;
    return launch_gemv(nt == 1 ? w->plan1 : w->plan8, w->d, x, xs, y, ys, nt, (flags & 1) != 0, (flags & 2) != 0,
                       (cudaStream_t)stream, &am);
}

// The same with host buffers: x_host [nt][cols] in, y_host (nullable) [nt][rows] and index_host [nt] out, copies on
// `stream` (asynchronous; pinned buffers make the copies asynchronous to the host).
FN_API int fn_w_gemv_argmax_host(int h, const float *xh, int nt, float *yh, int *ih, void *stream) {
    WeightH *w = wget(h);
    if (!w) return fail("fn_w_gemv_argmax_host: bad handle");
    if (nt < 1 || nt > 8) return fail("fn_w_gemv_argmax_host: nt out of range (1..8)");
    cudaStream_t s = (cudaStream_t)stream;
    const GemvPlan &p = nt == 1 ? w->plan1 : w->plan8;
    GemvArgmax am;
    am.index = w->ibuf;
    am.kacc = w->kacc;
    am.ticket = w->ticket;
    FN_CK(cudaMemcpyAsync(w->xbuf, xh, (size_t)nt * p.cols * 4, cudaMemcpyHostToDevice, s));
    if (launch_gemv(p, w->d, w->xbuf, p.cols, yh ? w->ybuf : nullptr, p.rows, nt, false, false, s, &am)) return -1;
    if (yh) FN_CK(cudaMemcpyAsync(yh, w->ybuf, (size_t)nt * p.rows * 4, cudaMemcpyDeviceToHost, s));
    FN_CK(cudaMemcpyAsync(ih, w->ibuf, (size_t)nt * sizeof(int), cudaMemcpyDeviceToHost, s));
    return 0;
}

// Row-split lm_head on a peer group (one rank per GPU): this rank's handle holds rows [row0, row0 + rows) of the
// vocabulary. The GEMV's fused argmax publishes this slice's winning keys to every rank over NVLink; a one-warp
// kernel then waits (bounded) for every rank's keys of this call and writes index[t], the winner over the whole
// vocabulary, on every rank. y (nullable) receives this rank's logit slice. Every rank makes the same calls.
FN_API int fn_w_gemv_argmax_group(int h, int gid, const float *x, int xs, float *y, int ys, int nt, int flags, int row0,
                                  int *index, void *stream) {
    WeightH *w = wget(h);
    PeerGroup *g = peer_group(gid);
    if (!w || !g) return fail("fn_w_gemv_argmax_group: bad handle or group");
    if (nt < 1 || nt > 8 || !index) return fail("fn_w_gemv_argmax_group: nt out of range (1..8) or no index");
    const KeyExchange xr = key_exchange(*g);
    GemvArgmax am;
    am.row0 = row0;
    am.kacc = w->kacc;
    am.ticket = w->ticket;
    am.xr = &xr;
    if (launch_gemv(nt == 1 ? w->plan1 : w->plan8, w->d, x, xs, y, ys, nt, (flags & 1) != 0, (flags & 2) != 0,
                    (cudaStream_t)stream, &am))
        return -1;
    return launch_keys_combine(xr.keys[g->rank], xr.counters[g->rank], g->local_calls + 1, g->n, nt, index,
                               (cudaStream_t)stream);
}

// argmax of logits[t][0..n) (token stride ls, device pointers) into out[t], on `stream` (engine/faie2fn.cu:1910-1935)
FN_API int fn_argmax(const float *logits, int ls, int n, int nt, int *out, void *stream) {
    return launch_argmax(logits, ls, n, nt, out, (cudaStream_t)stream);
}

// out[t] = the winning index among the keys [nranks][nt] of a row-split lm_head (device pointers, on `stream`)
FN_API int fn_argmax_keys(const unsigned long long *keys, int nranks, int nt, int *out, void *stream) {
    return launch_argmax_keys(keys, nranks, nt, out, (cudaStream_t)stream);
}

// synchronous hook: argmax of host logits [nt][n] -> host out [nt]
FN_API int fn_test_argmax(const float *lh, int n, int nt, int *oh) {
    if (n < 1 || nt < 1 || nt > 65535) return fail("fn_test_argmax: bad shape");
    FN_CK(cudaSetDevice(hook_device()));
    cudaStream_t s = hook_stream();
    DevBuf l, o;
    FN_CK(cudaMalloc(&l.p, (size_t)nt * n * 4));
    FN_CK(cudaMalloc(&o.p, (size_t)nt * 4));
    FN_CK(cudaMemcpyAsync(l.p, lh, (size_t)nt * n * 4, cudaMemcpyHostToDevice, s));
    if (launch_argmax(l.as<float>(), n, n, nt, o.as<int>(), s)) return -1;
    FN_CK(cudaMemcpyAsync(oh, o.p, (size_t)nt * 4, cudaMemcpyDeviceToHost, s));
    FN_CK(cudaStreamSynchronize(s));
    return check_dev_error("fn_test_argmax");
}

// synchronous hook: the lm_head GEMV with fused argmax on GGUF rows (as fn_test_gemv), y_host nullable
FN_API int fn_test_gemv_argmax(uint32_t type, const uint8_t *Wh, int rows, int cols, const float *xh, int nt, float *yh,
                               int *ih) {
    GemvPlan p;
    if (nt < 1 || nt > 8) return fail("nt out of range (1..8)");
    FN_CK(cudaSetDevice(hook_device()));
    if (!plan_gemv(p, type, rows, cols, nt == 1 ? 1 : 8)) return fail("unsupported type/shape");
    cudaStream_t s = hook_stream();
    DevBuf W, raw, x, y, idx, kacc, ticket;
    FN_CK(cudaMalloc(&W.p, plan_weight_bytes(p)));
    FN_CK(cudaMalloc(&raw.p, (size_t)p.rb * rows));
    FN_CK(cudaMalloc(&x.p, (size_t)nt * cols * 4));
    FN_CK(cudaMalloc(&y.p, (size_t)nt * rows * 4));
    FN_CK(cudaMalloc(&idx.p, 8 * sizeof(int)));
    FN_CK(cudaMalloc(&kacc.p, 256));
    FN_CK(cudaMalloc(&ticket.p, 256));
    FN_CK(cudaMemsetAsync(kacc.p, 0, 256, s));
    FN_CK(cudaMemsetAsync(ticket.p, 0, 256, s));
    FN_CK(cudaMemcpyAsync(raw.p, Wh, (size_t)p.rb * rows, cudaMemcpyHostToDevice, s));
    if (launch_plane_repack(type, raw.as<uint8_t>(), p.rb, W.as<uint8_t>(), p.ldw, rows, cols, s)) return -1;
    FN_CK(cudaMemcpyAsync(x.p, xh, (size_t)nt * cols * 4, cudaMemcpyHostToDevice, s));
    GemvArgmax am;
    am.index = idx.as<int>();
    am.kacc = kacc.as<unsigned long long>();
    am.ticket = ticket.as<unsigned int>();
    // twice: the second launch finds the key maxima and the ticket the first one cleared
    for (int rep = 0; rep < 2; ++rep)
        if (launch_gemv(p, W.as<uint8_t>(), x.as<float>(), cols, yh ? y.as<float>() : nullptr, rows, nt, false, false, s,
                        &am))
            return -1;
    if (yh) FN_CK(cudaMemcpyAsync(yh, y.p, (size_t)nt * rows * 4, cudaMemcpyDeviceToHost, s));
    FN_CK(cudaMemcpyAsync(ih, idx.p, (size_t)nt * sizeof(int), cudaMemcpyDeviceToHost, s));
    FN_CK(cudaStreamSynchronize(s));
    return check_dev_error("fn_test_gemv_argmax");
}

// The same with host buffers: x (nt x cols) copied in, y (nt x rows) copied out, all on `stream` (x and y should be
// pinned for the copies to be asynchronous). Does not synchronise; see fn_sync.
FN_API int fn_w_gemv_host(int h, const float *xh, int nt, float *yh, void *stream) {
    WeightH *w = wget(h);
    if (!w) return fail("fn_w_gemv_host: bad handle");
    if (nt < 1 || nt > 8) return fail("fn_w_gemv_host: nt out of range (1..8)");
    cudaStream_t s = (cudaStream_t)stream;
    const GemvPlan &p = nt == 1 ? w->plan1 : w->plan8;
    FN_CK(cudaMemcpyAsync(w->xbuf, xh, (size_t)nt * p.cols * 4, cudaMemcpyHostToDevice, s));
    if (launch_gemv(p, w->d, w->xbuf, p.cols, w->ybuf, p.rows, nt, false, false, s)) return -1;
    FN_CK(cudaMemcpyAsync(yh, w->ybuf, (size_t)nt * p.rows * 4, cudaMemcpyDeviceToHost, s));
    return 0;
}

// ---- a decode step's GEMVs on host buffers ---------------------------------------------------------------------------
// One host->device copy of every input, the GEMVs as one CUDA graph (built on the first call for a list of handles and
// replayed after; the GEMVs are independent, so they run as concurrent chains), one device->host copy of every output:
// the per-call host overhead of a step is paid once.

// A decode step's GEMVs, one token each, on host buffers: x the inputs of handles[0..n) back to back (cols_i floats
// each), y the outputs back to back (rows_i floats each, the lm_head's left out); head (-1: none) is the index in
// handles of the lm_head, whose argmax goes to *index instead of its logits. One host->device copy, the GEMVs as one
// CUDA graph (built on the first call for this list of handles, then replayed), one device->host copy, on `stream`
// (pinned host buffers make the copies asynchronous); does not synchronise. New: the reference's fn_forward runs a
// whole step per call (engine/faie2fn.cu:2733); this is that call's shape for the GEMV path alone.
FN_API int fn_w_step_host(int n, const int *handles, const float *xh, float *yh, int head, int *index, void *stream) {
    if (n < 1 || head >= n || (head >= 0 && !index)) return fail("fn_w_step_host: bad arguments");
    std::vector<int> key(handles, handles + n);
    key.push_back(head);
    StepPlan *sp = nullptr;
    {
        std::lock_guard<std::mutex> l(g_steps_mu);
        auto it = g_steps.find(key);
        if (it != g_steps.end()) sp = it->second;
    }
    if (!sp) {
        sp = new StepPlan();
        if (build_step(key, n, handles, head, sp)) {
            delete sp;
            return -1;
        }
        std::lock_guard<std::mutex> l(g_steps_mu);
        g_steps[key] = sp;
    }
    cudaStream_t s = (cudaStream_t)stream;
    FN_CK(cudaMemcpyAsync(sp->x.p, xh, sp->xn * 4, cudaMemcpyHostToDevice, s));
    FN_CK(cudaGraphLaunch(sp->exec, s));
    if (sp->yn) FN_CK(cudaMemcpyAsync(yh, sp->y.p, sp->yn * 4, cudaMemcpyDeviceToHost, s));
    if (head >= 0) FN_CK(cudaMemcpyAsync(index, sp->y.as<float>() + sp->yn, 4, cudaMemcpyDeviceToHost, s));
    return 0;
}

FN_API int fn_sync(void *stream) {
    FN_CK(cudaStreamSynchronize((cudaStream_t)stream));
    FN_CK(cudaGetLastError());
    return check_dev_error("fn_sync");
}
