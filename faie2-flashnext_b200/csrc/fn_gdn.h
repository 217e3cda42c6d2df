// Host interface of the gated-DeltaNet decode core (fn_gdn.cu).
#pragma once

#include "fn_common.cuh"

namespace fn {

struct GdnParams {  // device pointers
    int nkh = 0, nvh = 0, ds = 128;
    const float *conv_w = nullptr;  // [2*nkh*ds + nvh*ds][4] conv taps, oldest input first (16-byte aligned)
    const float *dt_bias = nullptr, *ssm_a = nullptr;  // [nvh]; ssm_a = -exp(A_log)
    const float *norm_w = nullptr;                     // [ds]
};

struct GdnState {  // device pointers
    float *S = nullptr;        // [nvh][ds][ds], S[h][i][j]: i key dim, j value dim
    float *conv_v = nullptr;   // [3][nvh*ds] value-channel history, oldest first
    float *conv_qk = nullptr;  // [nvh][3][2][ds] each value head's copy of its key head's q / k history
};

// nt tokens of one layer: qkv [nt][qs], z [nt][zs], ab [nt][abs_] (alpha | beta) -> out [nt][os]; state advanced.
// prefetch_state: the state was complete before the previous kernel in the stream started (true when the layer's
// previous launch is two or more kernels back), so it may be read before the programmatic-launch wait.
// batch > 1: that many independent sequences, one token each (nt == 1), sequence b's state at b times the state size
// and its token row at b times the strides.
int launch_gdn(const GdnParams &p, const GdnState &st, const float *qkv, int qs, const float *z, int zs, const float *ab,
               int abs_, float *out, int os, int nt, bool prefetch_state, cudaStream_t s, int batch = 1);

}  // namespace fn
