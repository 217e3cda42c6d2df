// Argmax keys: the selection rule of the lm_head argmax (engine/faie2fn.cu:1910-1935: the largest logit wins, the
// lowest index among equal values; NaN never wins; index 0 when no logit exceeds -inf) as a 64-bit key whose integer
// maximum is the winner, so that partial results (warps, CTAs, the row slices of a split lm_head on several GPUs)
// combine by max in any order. -0 ranks as +0 (the reference compares floats with >).
#pragma once

#include <cstdint>

namespace fn {

// key of (value v, global row r): order-preserving bits of v above (2^32 - 1 - r); 0 = no candidate (NaN, -inf)
__device__ __forceinline__ unsigned long long amax_key(float v, int r) {
    if (!(v > -INFINITY)) return 0ull;
    const uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);
    const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)o << 32) | (0xFFFFFFFFu - (uint32_t)r);
}
__device__ __forceinline__ int amax_index(unsigned long long k) { return k ? (int)(0xFFFFFFFFu - (uint32_t)k) : 0; }
__device__ __forceinline__ unsigned long long kmax(unsigned long long a, unsigned long long b) { return a > b ? a : b; }
__device__ __forceinline__ unsigned long long warp_kmax(unsigned long long k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) k = kmax(k, __shfl_xor_sync(0xffffffffu, k, o));
    return k;
}

}  // namespace fn
