// One decode step of the hybrid MoE decoder as a host object: the reference's layer_forward and
// forward (engine/faie2fn.cu:2370-2490) rebuilt from this engine's resident handles. A step is the embedding row of
// tokens[*pos]; per layer the input projection, the gated-DeltaNet core or the gated attention pair, the output
// projection adding into the residual, the router GEMV and the MoE layer adding into the residual; then the lm_head
// with its fused argmax and the step counter, which feeds the argmax back as the next input once the prompt is
// consumed. Every RMSNorm is folded into the GEMVs / MoE layer that read its output (fn_w_norm, fn_moe_norm), unless
// the model asks for separate norm launches. The position and the token ids live in device memory, so a step is a
// fixed launch sequence that a CUDA graph captures once. fn_load's engine (fn_runner.cu) and the Python DecodeModel
// (flashnext/model.py) both drive it; the caller owns the handles and the buffers.
#include <cstring>
#include <mutex>
#include <vector>

#include "faie2fn.h"
#include "fn_engine.h"

namespace fn {

constexpr int DS = 128, HD = 256;  // DeltaNet head size, attention head size

struct Decoder {
    fn_model_t m;
    std::vector<fn_layer_t> L;
    int convch = 0;
};
static std::vector<Decoder *> g_dec;
static std::mutex g_dec_mu;

static Decoder *dec_get(int h) {
    std::lock_guard<std::mutex> l(g_dec_mu);
    return h >= 1 && h <= (int)g_dec.size() ? g_dec[h - 1] : nullptr;
}

#define FN_TRY(call)          \
    do {                      \
        if ((call) != 0) return -1; \
    } while (0)

// the step's launches on stream s; dbg (host, nullable): h after layer l copied to dbg + l * dbg_stride
static int decoder_step(const Decoder &d, cudaStream_t s, float *dbg, size_t dbg_stride) {
    const fn_model_t &m = d.m;
    const bool fused = m.fuse_norm != 0;
    float *h = m.hidden, *xin = fused ? m.hidden : m.xnorm;
    FN_TRY(fn_embed(m.embed_type, m.embed, m.D, m.tokens, m.pos, h, s));
    for (size_t li = 0; li < d.L.size(); ++li) {
        const fn_layer_t &L = d.L[li];
        if (!fused) FN_TRY(fn_rmsnorm(h, L.norm1, m.xnorm, m.D, m.eps, s));
        int off = 0;
        for (int i = 0; i < 3 && L.w_in[i]; ++i) {
            FN_TRY(fn_w_gemv(L.w_in[i], xin, m.D, m.proj + off, 0, 1, 0, s));
            off += L.w_in_rows[i];
        }
        if (L.kind == 0) {
            const int nv = m.nvh * DS;
            // the layer's previous core launch is a whole step back: its state is read before the wait
            FN_TRY(fn_gdn_run(L.gdn, m.proj, d.convch, m.proj + d.convch, nv, m.proj + d.convch + nv, 2 * m.nvh, m.core,
                              nv, 1, 1, s));
            FN_TRY(fn_w_gemv(L.w_out, m.core, nv, h, 0, 1, 1, s));  // h += W_out core
        } else {
            float *qg = m.proj, *k = m.proj + m.nh * 2 * HD, *v = k + m.nkv * HD;
            FN_TRY(fn_attn_decode(qg, k, v, L.q_norm, L.k_norm, m.inv_freq, m.Q, L.Kc, L.Vc, m.att, m.pos, m.nh, m.nkv,
                                  m.max_ctx, m.eps, s));
            FN_TRY(fn_w_gemv(L.w_out, m.att, m.nh * HD, h, 0, 1, 1, s));  // h += W_o o
        }
        if (!fused) FN_TRY(fn_rmsnorm(h, L.norm2, m.xnorm, m.D, m.eps, s));
        FN_TRY(fn_w_gemv(L.router, xin, m.D, m.router_out, 0, 1, 0, s));
        // h += moe(x); with the norm folded the layer reads h (final since the router GEMV's wait) beside the router
        FN_TRY(fn_moe_run(L.moe, m.router_out, m.ne + 1, xin, h, 1, fused ? 3 : 1, s));
        if (dbg && cudaMemcpyAsync(dbg + li * dbg_stride, h, (size_t)m.D * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
            return fail("decoder: debug copy failed");
    }
    if (!fused) FN_TRY(fn_rmsnorm(h, m.final_norm, m.xnorm, m.D, m.eps, s));
    FN_TRY(fn_w_gemv_argmax(m.head, xin, m.D, m.logits, 0, 1, 0, 0, m.next, nullptr, s));
    FN_TRY(fn_step_advance(m.pos, m.tokens, m.next, m.prompt_len, m.max_ctx, s));
    return 0;
}

static int decoder_launches(const Decoder &d) {
    const int norm = d.m.fuse_norm ? 0 : 1;
    const int moe = settings().moe_var == 1 ? 2 : 3;  // gate/up and down, with or without a routing kernel
    int n = 1 + norm + 2;  // embedding, final norm, lm_head, step counter
    for (const fn_layer_t &L : d.L) {
        int nin = 0;
        while (nin < 3 && L.w_in[nin]) ++nin;
        n += 2 * norm + nin + (L.kind == 0 ? 1 : 2) + 1 + 1 + moe;  // + core / attention pair, out, router, MoE
    }
    return n;
}

}  // namespace fn

using namespace fn;

// A decode step over resident handles and caller-owned device buffers (no counterpart as a symbol in the reference,
// whose step lives inside fn_forward, engine/faie2fn.cu:2466-2490). Folds the norms (fuse_norm) and sets the L2
// prefetch hints along the chain (prefetch) on the handles, which must belong to this step alone. Returns a handle
// >= 1 or -1.
FN_API int fn_decoder_create(const fn_model_t *m, const fn_layer_t *layers, int n_layers) {
    if (!m || !layers || n_layers < 1) return fail("fn_decoder_create: no model");
    if (m->D < 32 || m->D % 32 || m->nkh < 1 || m->nvh < 1 || m->nh < 1 || m->nkv < 1 || m->ne < 1 || m->vocab < 1 ||
        m->max_ctx < 1)
        return fail("fn_decoder_create: bad sizes");
    if (!m->embed || !m->head || !m->hidden || !m->proj || !m->router_out || !m->tokens || !m->pos || !m->next ||
        !m->prompt_len || (!m->fuse_norm && !m->xnorm))
        return fail("fn_decoder_create: missing buffers");
    Decoder *d = new Decoder();
    d->m = *m;
    d->L.assign(layers, layers + n_layers);
    d->convch = 2 * m->nkh * DS + m->nvh * DS;
    for (const fn_layer_t &L : d->L) {
        const bool ok = (L.kind == 0 ? L.gdn > 0 && m->core : L.Kc && L.Vc && L.q_norm && L.k_norm && m->Q && m->att &&
                                                                   m->inv_freq) &&
                        L.w_in[0] > 0 && L.w_out > 0 && L.router > 0 && L.moe > 0 && L.norm1 && L.norm2;
        if (!ok) {
            delete d;
            return fail("fn_decoder_create: incomplete layer");
        }
    }
    if (m->fuse_norm) {
        for (const fn_layer_t &L : d->L) {
            for (int i = 0; i < 3 && L.w_in[i]; ++i)
                if (fn_w_norm(L.w_in[i], L.norm1, m->eps)) {
                    delete d;
                    return -1;
                }
            if (fn_w_norm(L.router, L.norm2, m->eps) || fn_moe_norm(L.moe, L.norm2, m->eps)) {
                delete d;
                return -1;
            }
        }
        if (fn_w_norm(m->head, m->final_norm, m->eps)) {
            delete d;
            return -1;
        }
    }
    if (m->prefetch) {  // input -> output projection -> router; the MoE layer -> the next layer's input projection
        for (size_t i = 0; i < d->L.size(); ++i) {
            const fn_layer_t &L = d->L[i];
            int last_in = 0;
            for (int j = 0; j < 3 && L.w_in[j]; ++j) last_in = L.w_in[j];
            const void *p;
            uint64_t b;
            if (fn_w_weights(L.w_out, &p, &b) || fn_w_prefetch_after(last_in, p, b) || fn_w_weights(L.router, &p, &b) ||
                fn_w_prefetch_after(L.w_out, p, b)) {
                delete d;
                return -1;
            }
            if (i + 1 < d->L.size() &&
                (fn_w_weights(d->L[i + 1].w_in[0], &p, &b) || fn_moe_prefetch_after(L.moe, p, b))) {
                delete d;
                return -1;
            }
        }
    }
    std::lock_guard<std::mutex> l(g_dec_mu);
    g_dec.push_back(d);
    return (int)g_dec.size();
}

FN_API int fn_decoder_free(int h) {
    std::lock_guard<std::mutex> l(g_dec_mu);
    if (h < 1 || h > (int)g_dec.size() || !g_dec[h - 1]) return fail("fn_decoder_free: bad handle");
    delete g_dec[h - 1];
    g_dec[h - 1] = nullptr;
    return 0;
}

// One decode step on `stream` (device work only, no synchronisation; capturable as a CUDA graph). dbg (host memory,
// nullable; the step then synchronises nothing either, the copies are asynchronous on the stream): the residual h
// after layer l is copied to dbg + l * dbg_stride floats.
FN_API int fn_decoder_step(int h, void *stream, float *dbg, int64_t dbg_stride) {
    Decoder *d = dec_get(h);
    if (!d) return fail("fn_decoder_step: bad handle");
    return decoder_step(*d, (cudaStream_t)stream, dbg, (size_t)dbg_stride);
}

// Kernel launches of one step.
FN_API int fn_decoder_launches(int h) {
    Decoder *d = dec_get(h);
    if (!d) return fail("fn_decoder_launches: bad handle");
    return decoder_launches(*d);
}
