// The row-dot core shared by the dense GEMV and the routed-expert kernels: x staging into shared memory, the
// per-lane group decode + FMA chains, and the fixed-order reduction of a row's lanes.
//
// Sum order (a function of the weight's format and row length only, never of the tokens or the launch shape):
// lane l of a row (lpr lanes per row) owns the 32-value groups l, l + lpr, l + 2 lpr, ...; each group is decoded
// (Dec<TY>, bit-exact values) into four fp32 FMA chains over runs of four values (chain k takes values j + k), the
// chains are added ((c0 + c1) + (c2 + c3)) in fp32, the group sums are accumulated in double in group order, and the
// lanes meet in a double butterfly (xor lpr/2, ..., 1). The row result is rounded to fp32 once by the caller.
#pragma once

#include "fn_decode.cuh"
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
template <uint32_t TY> __device__ __forceinline__ void stage_grid(uint32_t *grid) {
    if constexpr (Dec<TY>::gridw > 0) {
        const uint32_t *g = dev_grid<TY>();
        for (int i = threadIdx.x; i < Dec<TY>::gridw; i += blockDim.x) grid[i] = g[i];
    }
}

constexpr int XPAD = 36;  // floats per staged x group (32 + 4: lanes reading consecutive groups hit distinct banks)

// x[t][c] (token stride xs floats, 16-byte aligned, xs % 4 == 0) -> xsm[(t * G + g) * XPAD + j]; every thread calls
__device__ __forceinline__ void stage_x(float *xsm, const float *x, int xs, int nt, int G) {
    for (int idx = threadIdx.x; idx < nt * G * 8; idx += blockDim.x) {
        const int t = idx / (G * 8), r = idx - t * (G * 8), g = r >> 3, q = r & 7;
        const float4 v = *(const float4 *)(x + (size_t)t * xs + g * 32 + 4 * q);
        *(float4 *)(xsm + ((size_t)t * G + g) * XPAD + 4 * q) = v;
    }
}

// a lane's x slice in registers (one token): groups lr + LPR * i, i < GPL
template <int LPR, int GPL> struct XReg {
    float v[GPL][32];
    __device__ __forceinline__ void load(const float *xsm, int lr) {
#pragma unroll
        for (int i = 0; i < GPL; ++i) {
            const float *src = xsm + (size_t)(lr + LPR * i) * XPAD;
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 q = *(const float4 *)(src + j);
                v[i][j] = q.x;
                v[i][j + 1] = q.y;
                v[i][j + 2] = q.z;
                v[i][j + 3] = q.w;
            }
        }
    }
};

// acc[t] = sum over the lane's groups of row . x[t] (t < nt), then the butterfly over the row's LPR lanes, so every
// lane of the row ends with the row total. XREG: x from xr (one token); else from xsm ([t][G][XPAD]). Lanes of
// invalid rows (valid == false) contribute zeros but still take part in the butterfly.
template <uint32_t TY, int NT, int LPR, int GPL, bool XREG>
__device__ __forceinline__ void row_dot(const uint8_t *rowp, const uint32_t *grid, const XReg<LPR, (GPL > 0 ? GPL : 1)> &xr,
                                        const float *xsm, int G, int lr, int nt, bool valid, double (&acc)[NT]) {
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.0;
    if (valid) {
        const int ni = GPL > 0 ? GPL : (G + LPR - 1) / LPR;
#pragma unroll
        for (int i = 0; i < ni; ++i) {
            const int g = lr + LPR * i;
            if (GPL == 0 && g >= G) break;
            float c[NT][4];
#pragma unroll
            for (int t = 0; t < NT; ++t) c[t][0] = c[t][1] = c[t][2] = c[t][3] = 0.0f;
            Dec<TY>::group(rowp, g, grid, [&](int j, float v0, float v1, float v2, float v3) {
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (NT > 1 && t >= nt) break;
                    float4 xv;
                    if constexpr (XREG) {
                        xv = make_float4(xr.v[i][j], xr.v[i][j + 1], xr.v[i][j + 2], xr.v[i][j + 3]);
                    } else {
                        xv = *(const float4 *)(xsm + ((size_t)t * G + g) * XPAD + j);
                    }
                    c[t][0] = __fmaf_rn(v0, xv.x, c[t][0]);
                    c[t][1] = __fmaf_rn(v1, xv.y, c[t][1]);
                    c[t][2] = __fmaf_rn(v2, xv.z, c[t][2]);
                    c[t][3] = __fmaf_rn(v3, xv.w, c[t][3]);
                }
            });
#pragma unroll
            for (int t = 0; t < NT; ++t)
                acc[t] += (double)__fadd_rn(__fadd_rn(c[t][0], c[t][1]), __fadd_rn(c[t][2], c[t][3]));
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
    }
}

// Bounded wait on a stage barrier by every lane of a warp; the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, 1u << 22));
}

}  // namespace fn
