// C ABI of the gated-DeltaNet core (declared in include/faie2fn.h).
#include <cstring>
#include <mutex>
#include <vector>

#include "fn_engine.h"
#include "fn_gdn.h"

namespace fn {

struct GdnH {
    int batch = 1;  // independent sequences, each with its own state and conv histories
    GdnParams p;
    DevBuf conv_w, dt_bias, ssm_a, norm_w, S, conv_v, conv_qk;
    GdnState st;
};
static std::vector<GdnH *> g_gdn;
static std::mutex g_gdn_mu;

static GdnH *gdn_get(int h) {
    std::lock_guard<std::mutex> l(g_gdn_mu);
    return h >= 1 && h <= (int)g_gdn.size() ? g_gdn[h - 1] : nullptr;
}

// logical conv state [3][convch] (the reference's per-channel history, oldest first) <-> the engine's layout
static void conv_split(const float *logical, int nkh, int nvh, int ds, std::vector<float> &v, std::vector<float> &qk) {
    const int convch = 2 * nkh * ds + nvh * ds, nvd = nvh * ds;
    v.assign((size_t)3 * nvd, 0.f);
    qk.assign((size_t)nvh * 3 * 2 * ds, 0.f);
    for (int s = 0; s < 3; ++s) {
        for (int i = 0; i < nvd; ++i) v[(size_t)s * nvd + i] = logical[(size_t)s * convch + 2 * nkh * ds + i];
        for (int h = 0; h < nvh; ++h) {
            const int kh = h % nkh;
            for (int d = 0; d < ds; ++d) {
                qk[(((size_t)h * 3 + s) * 2 + 0) * ds + d] = logical[(size_t)s * convch + kh * ds + d];
                qk[(((size_t)h * 3 + s) * 2 + 1) * ds + d] = logical[(size_t)s * convch + nkh * ds + kh * ds + d];
            }
        }
    }
}
static void conv_join(float *logical, int nkh, int nvh, int ds, const std::vector<float> &v, const std::vector<float> &qk) {
    const int convch = 2 * nkh * ds + nvh * ds, nvd = nvh * ds;
    for (int s = 0; s < 3; ++s) {
        for (int i = 0; i < nvd; ++i) logical[(size_t)s * convch + 2 * nkh * ds + i] = v[(size_t)s * nvd + i];
        for (int kh = 0; kh < nkh; ++kh)  // value head kh holds a copy of key head kh's history
            for (int d = 0; d < ds; ++d) {
                logical[(size_t)s * convch + kh * ds + d] = qk[(((size_t)kh * 3 + s) * 2 + 0) * ds + d];
                logical[(size_t)s * convch + nkh * ds + kh * ds + d] = qk[(((size_t)kh * 3 + s) * 2 + 1) * ds + d];
            }
    }
}

static int up(DevBuf &b, const void *src, size_t bytes) {
    FN_CK(cudaMalloc(&b.p, bytes));
    FN_CK(cudaMemcpy(b.p, src, bytes, cudaMemcpyHostToDevice));
    return 0;
}

static GdnH *gdn_build(int nkh, int nvh, int ds, const float *conv_w, const float *dt_bias, const float *ssm_a,
                       const float *norm_w, const float *S0, const float *conv0) {
    if (ds != 128 || nkh < 1 || nvh < 1 || nvh % nkh) {
        fail("gdn: unsupported heads (head dim 128, value heads a multiple of key heads)");
        return nullptr;
    }
    GdnH *g = new GdnH();
    g->p.nkh = nkh;
    g->p.nvh = nvh;
    g->p.ds = ds;
    const size_t convch = (size_t)2 * nkh * ds + (size_t)nvh * ds;
    std::vector<float> cv, cqk;
    conv_split(conv0, nkh, nvh, ds, cv, cqk);
    if (up(g->conv_w, conv_w, convch * 16) || up(g->dt_bias, dt_bias, nvh * 4) || up(g->ssm_a, ssm_a, nvh * 4) ||
        up(g->norm_w, norm_w, ds * 4) || up(g->S, S0, (size_t)nvh * ds * ds * 4) ||
        up(g->conv_v, cv.data(), cv.size() * 4) || up(g->conv_qk, cqk.data(), cqk.size() * 4)) {
        delete g;
        return nullptr;
    }
    g->p.conv_w = g->conv_w.as<float>();
    g->p.dt_bias = g->dt_bias.as<float>();
    g->p.ssm_a = g->ssm_a.as<float>();
    g->p.norm_w = g->norm_w.as<float>();
    g->st = GdnState{g->S.as<float>(), g->conv_v.as<float>(), g->conv_qk.as<float>()};
    return g;
}

static int gdn_read_state(GdnH *g, float *S, float *conv) {
    const GdnParams &p = g->p;
    std::vector<float> cv((size_t)3 * p.nvh * p.ds), cqk((size_t)p.nvh * 3 * 2 * p.ds);
    if (S) FN_CK(cudaMemcpy(S, g->S.p, (size_t)p.nvh * p.ds * p.ds * 4, cudaMemcpyDeviceToHost));
    if (conv) {
        FN_CK(cudaMemcpy(cv.data(), g->conv_v.p, cv.size() * 4, cudaMemcpyDeviceToHost));
        FN_CK(cudaMemcpy(cqk.data(), g->conv_qk.p, cqk.size() * 4, cudaMemcpyDeviceToHost));
        conv_join(conv, p.nkh, p.nvh, p.ds, cv, cqk);
    }
    return 0;
}

}  // namespace fn

using namespace fn;

// nt tokens of the DeltaNet core on host buffers, tokens_per_launch at a time (1: one launch per token, as decode).
// qkv [nt][2*nkh*ds + nvh*ds], z [nt][nvh*ds], ab [nt][2*nvh] (alpha | beta), conv_w [convch][4], dt_bias and ssm_a
// [nvh], norm_w [ds]; S [nvh][ds][ds] and conv_state [3][convch] (oldest first) are read and updated in place;
// out [nt][nvh*ds].
FN_API int fn_test_gdn(int nkh, int nvh, int ds, int nt, int tokens_per_launch, const float *qkv, const float *z,
                       const float *ab, const float *conv_w, const float *dt_bias, const float *ssm_a,
                       const float *norm_w, float *S, float *conv_state, float *out) {
    if (nt < 1 || tokens_per_launch < 1) return fail("fn_test_gdn: nt and tokens_per_launch must be >= 1");
    FN_CK(cudaSetDevice(hook_device()));
    GdnH *g = gdn_build(nkh, nvh, ds, conv_w, dt_bias, ssm_a, norm_w, S, conv_state);
    if (!g) return -1;
    const int convch = 2 * nkh * ds + nvh * ds, nvd = nvh * ds;
    cudaStream_t s = hook_stream();
    DevBuf dq, dz, dab, dout;
    int rc = 0;
    if (up(dq, qkv, (size_t)nt * convch * 4) || up(dz, z, (size_t)nt * nvd * 4) || up(dab, ab, (size_t)nt * 2 * nvh * 4) ||
        cudaMalloc(&dout.p, (size_t)nt * nvd * 4) != cudaSuccess)
        rc = err().empty() ? fail("fn_test_gdn: allocation failed") : -1;
    for (int t0 = 0; !rc && t0 < nt; t0 += tokens_per_launch) {
        const int n = std::min(tokens_per_launch, nt - t0);
        rc = launch_gdn(g->p, g->st, dq.as<float>() + (size_t)t0 * convch, convch, dz.as<float>() + (size_t)t0 * nvd,
                        nvd, dab.as<float>() + (size_t)t0 * 2 * nvh, 2 * nvh, dout.as<float>() + (size_t)t0 * nvd, nvd,
                        n, /*prefetch_state=*/t0 == 0, s);  // later launches follow the previous one directly
    }
    if (!rc) {
        const cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) rc = fail(std::string("fn_test_gdn: ") + cudaGetErrorString(e));
    }
    if (!rc && cudaMemcpy(out, dout.p, (size_t)nt * nvd * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = fail("fn_test_gdn: copy out failed");
    if (!rc) rc = gdn_read_state(g, S, conv_state);
    delete g;
    return rc;
}

// Resident DeltaNet layer state + parameters on the current device (arguments as fn_test_gdn); a handle or -1.
FN_API int fn_gdn_create(int nkh, int nvh, int ds, const float *conv_w, const float *dt_bias, const float *ssm_a,
                         const float *norm_w, const float *S0, const float *conv0) {
    GdnH *g = gdn_build(nkh, nvh, ds, conv_w, dt_bias, ssm_a, norm_w, S0, conv0);
    if (!g) return -1;
    std::lock_guard<std::mutex> l(g_gdn_mu);
    g_gdn.push_back(g);
    return (int)g_gdn.size();
}

// A DeltaNet layer for `batch` independent sequences (batched decode): parameters as fn_gdn_create, every sequence's
// state and conv histories zero. Returns a handle >= 1 or -1; run it with fn_gdn_run_batch.
FN_API int fn_gdn_create_batch(int nkh, int nvh, int ds, const float *conv_w, const float *dt_bias, const float *ssm_a,
                               const float *norm_w, int batch) {
    if (batch < 1 || batch > 1024) return fail("fn_gdn_create_batch: batch out of range (1..1024)");
    const size_t nS = (size_t)nvh * ds * ds, nconv = (size_t)3 * (2 * nkh * ds + nvh * ds);
    std::vector<float> S0(nS, 0.f), c0(nconv, 0.f);
    GdnH *g = gdn_build(nkh, nvh, ds, conv_w, dt_bias, ssm_a, norm_w, S0.data(), c0.data());
    if (!g) return -1;
    g->batch = batch;
    if (batch > 1) {  // the per-sequence states, zero
        const size_t bS = (size_t)batch * nS * 4, bv = (size_t)batch * 3 * nvh * ds * 4,
                     bqk = (size_t)batch * nvh * 3 * 2 * ds * 4;
        DevBuf S, v, qk;
        if (cudaMalloc(&S.p, bS) != cudaSuccess || cudaMalloc(&v.p, bv) != cudaSuccess ||
            cudaMalloc(&qk.p, bqk) != cudaSuccess || cudaMemset(S.p, 0, bS) != cudaSuccess ||
            cudaMemset(v.p, 0, bv) != cudaSuccess || cudaMemset(qk.p, 0, bqk) != cudaSuccess) {
            delete g;
            return fail("fn_gdn_create_batch: device allocation failed");
        }
        std::swap(g->S.p, S.p);
        std::swap(g->conv_v.p, v.p);
        std::swap(g->conv_qk.p, qk.p);
        g->st.S = g->S.as<float>();
        g->st.conv_v = g->conv_v.as<float>();
        g->st.conv_qk = g->conv_qk.as<float>();
    }
    std::lock_guard<std::mutex> l(g_gdn_mu);
    g_gdn.push_back(g);
    return (int)g_gdn.size();
}

// One decode step of every sequence of a batch handle: token row b of qkv / z / ab / out (strides qs, zs, abs_, os in
// floats) is sequence b's. prefetch_state as fn_gdn_run.
FN_API int fn_gdn_run_batch(int h, const float *qkv, int qs, const float *z, int zs, const float *ab, int abs_,
                            float *out, int os, int prefetch_state, void *stream) {
    GdnH *g = gdn_get(h);
    if (!g) return fail("fn_gdn_run_batch: bad handle");
    return launch_gdn(g->p, g->st, qkv, qs, z, zs, ab, abs_, out, os, 1, prefetch_state != 0, (cudaStream_t)stream,
                      g->batch);
}

// Zero the handle's recurrent state and conv histories (the start of a new sequence), on `stream`.
FN_API int fn_gdn_reset(int h, void *stream) {
    GdnH *g = gdn_get(h);
    if (!g) return fail("fn_gdn_reset: bad handle");
    const size_t nS = (size_t)g->batch * g->p.nvh * g->p.ds * g->p.ds, nv = (size_t)g->batch * 3 * g->p.nvh * g->p.ds,
                 nqk = (size_t)g->batch * g->p.nvh * 3 * 2 * g->p.ds;
    cudaStream_t s = (cudaStream_t)stream;
    FN_CK(cudaMemsetAsync(g->st.S, 0, nS * 4, s));
    FN_CK(cudaMemsetAsync(g->st.conv_v, 0, nv * 4, s));
    FN_CK(cudaMemsetAsync(g->st.conv_qk, 0, nqk * 4, s));
    return 0;
}

FN_API int fn_gdn_free(int h) {
    GdnH *g = gdn_get(h);
    if (!g) return fail("fn_gdn_free: bad handle");
    delete g;
    std::lock_guard<std::mutex> l(g_gdn_mu);
    g_gdn[h - 1] = nullptr;
    return 0;
}

// Launch nt tokens on device pointers (token strides in floats); the handle's state advances. prefetch_state = 1
// when this handle's previous launch is two or more kernels back in the stream (its state is then complete before
// the kernel just before this one started, and is read while that kernel runs); 0 when it may be the kernel just
// before.
FN_API int fn_gdn_run(int h, const float *qkv, int qs, const float *z, int zs, const float *ab, int abs_, float *out,
                      int os, int nt, int prefetch_state, void *stream) {
    GdnH *g = gdn_get(h);
    if (!g) return fail("fn_gdn_run: bad handle");
    if (g->batch > 1) return fail("fn_gdn_run: a batch handle runs with fn_gdn_run_batch");
    return launch_gdn(g->p, g->st, qkv, qs, z, zs, ab, abs_, out, os, nt, prefetch_state != 0, (cudaStream_t)stream);
}

// Copy the handle's state to host: S [nvh][ds][ds] and conv [3][convch] (either may be NULL). Synchronous.
FN_API int fn_gdn_get_state(int h, float *S, float *conv) {
    GdnH *g = gdn_get(h);
    if (!g) return fail("fn_gdn_get_state: bad handle");
    FN_CK(cudaDeviceSynchronize());
    return gdn_read_state(g, S, conv);
}
