// Host launcher of the fused MoE layer (fn_moe_fused.cuh): the gate/up and down formats it is instantiated for, the
// plan of its shared memory, and the fallback signal for every other layer.
#include "fn_moe_fused.cuh"

namespace fn {

static size_t al128(size_t v) { return (v + 127) / 128 * 128; }

// The fused form of one MoE layer for one token (after its routing kernel). Returns 1 when this layer has no fused
// form (formats without an instantiation, rows too wide for one CTA's shared memory): the caller then launches the
// gate/up and down kernels. 0: launched; -1: error.
int launch_moe_fused(const MoePlan &p, const MoeWeights &w, const float *logits, const float *x, float *act,
                     const int *rsel, const float *rw, uint32_t *cnt, float *y, bool acc, bool x_early, cudaStream_t s) {
    constexpr size_t kDyn = 227 * 1024 - 4 * 1024;
    const int ks = p.k + 1, G = p.d / 32, Gd = p.ffe / 32, NW = FUSED_WARPS;
    // one SM fewer than the GPU has: the routing kernel's CTA keeps an SM while this grid starts, and a CTA placed
    // behind it would start late while the others wait for its units
    const int ctas = std::max(1, num_sms() - 1);
    if (!cnt || ks > 16 || p.lpr_down > 8 || ctas > p.d) return 1;
    const long long U = (long long)ks * p.ffe;
    const int per_cta = (int)((U + ctas - 1) / ctas), upw = (per_cta + NW - 1) / NW;
    if (upw > p.ffe) return 1;
    const int rows = (p.d + ctas - 1) / ctas;
    MoeFusedArgs a{};
    a.gu_off = 512;
    a.dw_off = (uint32_t)al128(a.gu_off + (size_t)NW * upw * 2 * p.ldw_gu);
    a.res_off = (uint32_t)al128(a.dw_off + (size_t)ks * rows * p.ldw_down);
    a.grid_off = (uint32_t)al128(a.res_off + (size_t)ks * rows * 4);
    a.xs_off = (uint32_t)al128(a.grid_off + (size_t)grid_words(p.gu_type) * 4);
    const bool xreg = G == 32 || G == 64;
    a.as_off = (uint32_t)al128(a.xs_off + (xreg ? 0 : (size_t)G * XPAD * 4));
    const size_t smem = al128(a.as_off + (size_t)ks * Gd * XPAD * 4);
    if (smem > kDyn) return 1;
    a.Wg = w.gate;
    a.Wu = w.up;
    a.Wsg = w.sh_gate;
    a.Wsu = w.sh_up;
    a.ldw_g = p.ldw_gu;
    a.Wd = w.down;
    a.Wsd = w.sh_down;
    a.ldw_d = p.ldw_down;
    {
        int qk, tb;
        type_info(p.gu_type, qk, tb);
        a.nb_g = p.d / qk;
        type_info(p.down_type, qk, tb);
        a.nb_d = p.ffe / qk;
    }
    a.ne = p.ne;
    a.k = p.k;
    a.ffe = p.ffe;
    a.d = p.d;
    a.logits = logits;
    a.ls = p.ne + 1;
    a.x = x;
    a.act = act;
    a.y = y;
    a.acc = acc ? 1 : 0;
    a.rsel = rsel;
    a.rw = rw;
    a.cnt = cnt;
    a.x_early = x_early && settings().pdl ? 1 : 0;
    a.nw = p.nw;
    a.eps = p.eps;
    a.upw = upw;
    a.rows = rows;
    a.err = dev_error_ptr();
    a.pf = p.pf;
    a.pf_bytes = p.pf_bytes;
    cudaError_t e = cudaSuccess;
    bool known = true;
    if (p.gu_type == T_IQ3_XXS && p.down_type == T_Q4_K) e = moe_fused_launch_t<T_IQ3_XXS, T_Q4_K>(a, G, p.lpr_down, ctas, smem, s);
    else if (p.gu_type == T_Q4_K && p.down_type == T_Q4_K) e = moe_fused_launch_t<T_Q4_K, T_Q4_K>(a, G, p.lpr_down, ctas, smem, s);
    else if (p.gu_type == T_IQ2_XXS && p.down_type == T_Q4_K) e = moe_fused_launch_t<T_IQ2_XXS, T_Q4_K>(a, G, p.lpr_down, ctas, smem, s);
    else if (p.gu_type == T_Q4_K && p.down_type == T_Q6_K) e = moe_fused_launch_t<T_Q4_K, T_Q6_K>(a, G, p.lpr_down, ctas, smem, s);
    else known = false;
    if (!known) return 1;
    if (e != cudaSuccess) return fail(std::string("moe fused launch: ") + cudaGetErrorString(e));
    return 0;
}

}  // namespace fn
