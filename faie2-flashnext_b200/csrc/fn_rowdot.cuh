// The row-dot core shared by the dense GEMV and the routed-expert kernels: x staging into shared memory, the
// per-lane group dot products, and the fixed-order reduction of a row's lanes.
//
// Sum order (a function of the weight's format and row length only, never of the tokens or the launch shape):
// lane l of a row (lpr lanes per row) owns the 32-value groups l, l + lpr, l + 2 lpr, ...; each group's dot product
// is one fp32 value (Fast<TY> on the plane layout, or the bit-exact generic decoder load_group reduced by four FMA
// chains on GGUF rows); the group values are accumulated in double in group order, and the row's lanes meet in a
// double butterfly (xor lpr/2, ..., 1; when a warp works on two rows the first step exchanges halves, which adds the
// same pairs). The row result is rounded to fp32 once by the caller.
#pragma once

#include "fn_decode.cuh"
#include "fn_fastdot.cuh"
#include "fn_grids.h"

namespace fn {

template <uint32_t TY> __device__ __forceinline__ const uint32_t *dev_grid() {
    if constexpr (TY == T_IQ2_XXS) return kIq2xxsGrid;
    else if constexpr (TY == T_IQ2_XS) return kIq2xsGrid;
    else if constexpr (TY == T_IQ2_S) return kIq2sGrid;
    else if constexpr (TY == T_IQ3_XXS) return kIq3xxsGrid;
    else if constexpr (TY == T_IQ3_S) return kIq3sGrid;
    else return nullptr;
}

// copy the codebook of TY (if it has one) to shared memory; every thread of the block calls this
// (IQ3_XXS: after the 256 codebook words, its signed expansion for the fast path: entry (i, s) holds the 4 values of
// codebook word i with the signs of the 4 bits of s (bit j set: value j negative) as bf16, exact for |v| <= 62, two
// per word: tab[2 (16 i + s) + h] = bf16(v[2h]) | bf16(v[2h + 1]) << 16)
template <uint32_t TY> __device__ __forceinline__ void stage_grid(uint32_t *grid) {
    if constexpr (Gguf<TY>::gridw > 0) {
        const uint32_t *g = dev_grid<TY>();
        for (int i = threadIdx.x; i < Gguf<TY>::gridw; i += blockDim.x) grid[i] = g[i];
        if constexpr (TY == T_IQ3_XXS) {  // (generated with the codebook by gen_grids.py)
            uint4 *tab = (uint4 *)(grid + Gguf<TY>::gridw);
            const uint4 *src = (const uint4 *)kIq3xxsSigned;
            for (int i = threadIdx.x; i < 8192 / 4; i += blockDim.x) tab[i] = src[i];
        }
    }
}

// the fast plane-layout path is used for TY when the weights are stored in planes
template <uint32_t TY, bool SOA> struct UseFast {
    static constexpr bool v = SOA && Fast<TY>::ok;
};
// x is staged scaled (stage_x denorm) when the fast path converts TY's bytes as denormals
template <uint32_t TY, bool SOA> struct ScaleX {
    static constexpr bool v = UseFast<TY, SOA>::v && Denorm<TY>::v;
};

constexpr int XPAD = 36;  // floats per staged x group: 32 values, the two 16-value sums, 2 spare (bank spread)

// x[t][c] (token stride xs floats, 16-byte aligned, xs % 4 == 0) -> xsm[(t * G + g) * XPAD + j], the half sums
// sum(x[16h .. 16h + 15]) (pairwise, fixed order, unscaled) at + 32 + h, and for formats that convert bytes as
// denormals (denorm) the values scaled by 2^K_t with K_t = 124 - exponent(max_c |x[t][c]|) clamped to [22, 127]
// (an exact power-of-two scaling; the products q * 2^-149 * x * 2^K_t then stay in the normal range) and
// 2^(149 - K_t) at + 34. nt <= 32. Every thread calls this; it ends with a __syncthreads.
// nw (an RMSNorm weight, nullable): the values staged are x[t][c] * nw[c], and + 35 of group g holds the sum of the
// squares of the raw x over the group's 32 values (fixed order) for norm_scale. cg: x is read through L2 only (data
// another CTA of the same grid published with a release, after this CTA's acquire).
__device__ __forceinline__ void stage_x(float *xsm, const float *x, int xs, int nt, int G, bool denorm,
                                        const float *nw = nullptr, bool cg = false) {
    __shared__ int s_xmax[32];
    if (denorm) {
        if ((int)threadIdx.x < nt) s_xmax[threadIdx.x] = 0;
        __syncthreads();
    }
    for (int idx = threadIdx.x; idx < nt * G * 2; idx += blockDim.x) {
        const int t = idx / (G * 2), r = idx - t * (G * 2), g = r >> 1, h = r & 1;
        const float4 *src = (const float4 *)(x + (size_t)t * xs + g * 32 + 16 * h);
        float *dst = xsm + ((size_t)t * G + g) * XPAD;
        float4 v[4];
        float mx = 0.0f;
        if (nw) {
            // the group's sum of squares, by the h == 0 item over both halves (16 products each, in order)
            if (h == 0) {
                float ss = 0.0f;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 f = src[q];
                    ss = __fmaf_rn(f.x, f.x, ss);
                    ss = __fmaf_rn(f.y, f.y, ss);
                    ss = __fmaf_rn(f.z, f.z, ss);
                    ss = __fmaf_rn(f.w, f.w, ss);
                }
                dst[35] = ss;
            }
            const float4 *wv = (const float4 *)(nw + g * 32 + 16 * h);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 f = src[q], w = wv[q];
                v[q] = make_float4(__fmul_rn(f.x, w.x), __fmul_rn(f.y, w.y), __fmul_rn(f.z, w.z), __fmul_rn(f.w, w.w));
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (!nw) v[q] = cg ? __ldcg(src + q) : src[q];
            *(float4 *)(dst + 16 * h + 4 * q) = v[q];
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[q].x), fabsf(v[q].y)), fmaxf(fabsf(v[q].z), fabsf(v[q].w))));
        }
        float p[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) p[q] = __fadd_rn(__fadd_rn(v[q].x, v[q].y), __fadd_rn(v[q].z, v[q].w));
        dst[32 + h] = __fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3]));
        if (denorm) atomicMax(&s_xmax[t], __float_as_int(mx));  // non-negative floats order like their bits
    }
    __syncthreads();
    if (!denorm) return;
    for (int idx = threadIdx.x; idx < nt * G * 2; idx += blockDim.x) {
        const int t = idx / (G * 2), r = idx - t * (G * 2), g = r >> 1, h = r & 1;
        const int e = ((s_xmax[t] >> 23) & 255) - 127;  // exponent of the largest |x| (0 -> -127)
        const int K = max(22, min(127, 124 - e));
        const float sc = __int_as_float((K + 127) << 23);
        float *dst = xsm + ((size_t)t * G + g) * XPAD;
#pragma unroll
        for (int q = 0; q < 16; ++q) dst[16 * h + q] = __fmul_rn(dst[16 * h + q], sc);
        if (h == 0) dst[34] = __int_as_float((149 - K + 127) << 23);
    }
    __syncthreads();
}

// RMSNorm scale of token t from stage_x's per-group sums of squares (stage_x with nw): rsqrt(sum / n + eps) with the
// sum over groups in a fixed order (lane l: groups l, l + 32, ..; then a butterfly), so every warp of every CTA gets
// the same value. Called by whole warps after stage_x.
__device__ __forceinline__ float norm_scale(const float *xsm, int G, int t, int n, float eps) {
    const int lane = threadIdx.x & 31;
    float ss = 0.0f;
    for (int g = lane; g < G; g += 32) ss = __fadd_rn(ss, xsm[((size_t)t * G + g) * XPAD + 35]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    return rsqrtf(ss / (float)n + eps);
}

// a lane's x slice in registers (one token): groups lr + LPR * i, i < GPL
template <int LPR, int GPL> struct XReg {
    float2 v[GPL][16];
    float s[GPL][2];
    float iv = 1.0f;
    // Straight from x in global memory (16-byte aligned), by one warp whose lanes together hold every group of the
    // row (LPR == 32 and GPL == G / 32): the same values, half sums and power-of-two scaling (denorm) as stage_x,
    // with the row maximum taken over the warp instead of the block, so no block barrier is needed.
    // nw (an RMSNorm weight, nullable): the values held are x * nw, and the return value is the RMSNorm scale
    // rsqrt(sum x^2 / (32 G) + eps) (the sum in group order per lane, then a butterfly: the same in every warp); else 1.
    __device__ __forceinline__ float load_global(const float *x, int lr, bool denorm, const float *nw = nullptr,
                                                 float eps = 0.0f) {
        float mx = 0.0f, ss = 0.0f;
#pragma unroll
        for (int i = 0; i < GPL; ++i) {
            const float4 *src = (const float4 *)(x + (size_t)(lr + LPR * i) * 32);
            float4 q[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) q[j] = src[j];
            if (nw) {
                const float4 *wv = (const float4 *)(nw + (size_t)(lr + LPR * i) * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 f = q[j], w = wv[j];
                    ss = __fmaf_rn(f.x, f.x, ss);
                    ss = __fmaf_rn(f.y, f.y, ss);
                    ss = __fmaf_rn(f.z, f.z, ss);
                    ss = __fmaf_rn(f.w, f.w, ss);
                    q[j] = make_float4(__fmul_rn(f.x, w.x), __fmul_rn(f.y, w.y), __fmul_rn(f.z, w.z), __fmul_rn(f.w, w.w));
                }
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float p[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float4 f = q[4 * h + u];
                    p[u] = __fadd_rn(__fadd_rn(f.x, f.y), __fadd_rn(f.z, f.w));
                    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
                }
                s[i][h] = __fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3]));
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                v[i][2 * j] = make_float2(q[j].x, q[j].y);
                v[i][2 * j + 1] = make_float2(q[j].z, q[j].w);
            }
        }
        float scale = 1.0f;
        if (nw) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
            scale = rsqrtf(ss / (float)(32 * LPR * GPL) + eps);
        }
        if (!denorm) return scale;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const int e = ((__float_as_int(mx) >> 23) & 255) - 127;
        const int K = max(22, min(127, 124 - e));
        const float sc = __int_as_float((K + 127) << 23);
#pragma unroll
        for (int i = 0; i < GPL; ++i)
#pragma unroll
            for (int j = 0; j < 16; ++j) v[i][j] = make_float2(__fmul_rn(v[i][j].x, sc), __fmul_rn(v[i][j].y, sc));
        iv = __int_as_float((149 - K + 127) << 23);
        return scale;
    }
    __device__ __forceinline__ void load(const float *xsm, int lr) {
        iv = xsm[34];
#pragma unroll
        for (int i = 0; i < GPL; ++i) {
            const float *src = xsm + (size_t)(lr + LPR * i) * XPAD;
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
                const float4 q = *(const float4 *)(src + 2 * j);
                v[i][j] = make_float2(q.x, q.y);
                v[i][j + 1] = make_float2(q.z, q.w);
            }
            s[i][0] = src[32];
            s[i][1] = src[33];
        }
    }
};

// one group of one row: fast path (planes) or generic (GGUF rows, bit-exact values in four FMA chains)
template <uint32_t TY, bool SOA, int NT, class XA>
__device__ __forceinline__ void group_dot(const uint8_t *rowp, int nb, int g, const uint32_t *grid, const XA &xa, int nt,
                                          float (&r)[NT]) {
    if constexpr (UseFast<TY, SOA>::v) {
        Fast<TY>::template group<NT>(rowp, nb, g, grid, xa, nt, r);
    } else {
        float c[NT][4];
#pragma unroll
        for (int t = 0; t < NT; ++t) c[t][0] = c[t][1] = c[t][2] = c[t][3] = 0.0f;
        const auto w = load_group<TY>(rowp, g, grid);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 v = w.quad(j);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (NT > 1 && t >= nt) break;
                const float2 x01 = xa.x2(t, j), x23 = xa.x2(t, j + 2);
                c[t][0] = __fmaf_rn(v.x, x01.x, c[t][0]);
                c[t][1] = __fmaf_rn(v.y, x01.y, c[t][1]);
                c[t][2] = __fmaf_rn(v.z, x23.x, c[t][2]);
                c[t][3] = __fmaf_rn(v.w, x23.y, c[t][3]);
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t)
            if (NT == 1 || t < nt) r[t] = __fadd_rn(__fadd_rn(c[t][0], c[t][1]), __fadd_rn(c[t][2], c[t][3]));
    }
}

// RR rows (1, or 2 when LPR == 32) of one lane group: acc[rr][t] = row rr . x[t]. After the butterfly the total of
// row rr is held by the lanes of half rr (RR == 2) or by every lane of the row (RR == 1). XREG: x from xr (one
// token); else from xsm ([t][G][XPAD], token stride G * XPAD). Invalid rows contribute zeros.
template <uint32_t TY, bool SOA, int NT, int LPR, int GPL, bool XREG, int RR>
__device__ __forceinline__ void rows_dot(const uint8_t *const (&rowp)[RR], const bool (&valid)[RR], int nb,
                                         const uint32_t *grid, const XReg<LPR, (GPL > 0 ? GPL : 1)> &xr,
                                         const float *xsm, int G, int lr, int nt, double (&acc)[RR][NT]) {
#pragma unroll
    for (int q = 0; q < RR; ++q)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[q][t] = 0.0;
    if constexpr (GPL > 0) {  // a fixed number of groups per lane (x in registers or not): unrolled
#pragma unroll
        for (int i = 0; i < GPL; ++i) {
            const int g = lr + LPR * i;
#pragma unroll
            for (int q = 0; q < RR; ++q) {
                if (!valid[q]) continue;
                float r[NT];
                if constexpr (XREG) {
                    const XRegA xa{xr.v[i], xr.s[i], xr.iv};
                    group_dot<TY, SOA, NT>(rowp[q], nb, g, grid, xa, nt, r);
                } else {
                    const XSmA xa{xsm + (size_t)g * XPAD, G * XPAD};
                    group_dot<TY, SOA, NT>(rowp[q], nb, g, grid, xa, nt, r);
                }
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    if (NT == 1 || t < nt) acc[q][t] += (double)r[t];
            }
        }
    } else {  // any row length: one decode body in a loop over (group, row), x from shared memory
        const int ni = (G + LPR - 1) / LPR;
#pragma unroll 1
        for (int it = 0; it < ni * RR; ++it) {
            const int i = it / RR, q = it - i * RR, g = lr + LPR * i;
            if (g >= G) break;
            if (!(q == 0 ? valid[0] : valid[RR - 1])) continue;
            float r[NT];
            const XSmA xa{xsm + (size_t)g * XPAD, G * XPAD};
            group_dot<TY, SOA, NT>(q == 0 ? rowp[0] : rowp[RR - 1], nb, g, grid, xa, nt, r);
#pragma unroll
            for (int t = 0; t < NT; ++t)
                if (NT == 1 || t < nt) {
                    if (q == 0) acc[0][t] += (double)r[t];
                    else acc[RR - 1][t] += (double)r[t];
                }
        }
    }
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if constexpr (RR == 2) {  // lanes 0-15 keep row 0, lanes 16-31 row 1
            const bool up = lane & 16;
            const double send = up ? acc[0][t] : acc[1][t];
            double keep = up ? acc[1][t] : acc[0][t];
            keep += __shfl_xor_sync(0xffffffffu, send, 16);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
            acc[0][t] = keep;
            acc[1][t] = keep;
        } else {
#pragma unroll
            for (int o = LPR / 2; o > 0; o >>= 1) acc[0][t] += __shfl_xor_sync(0xffffffffu, acc[0][t], o);
        }
    }
}

// Bounded wait on a stage barrier by every lane of a warp; the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, 1u << 22));
}

}  // namespace fn
