// Stand-alone argmax kernels: over a logits buffer (the reference's k_argmax, engine/faie2fn.cu:1910-1935, for logits
// that did not come from the fused GEMV epilogue), and over the per-GPU keys of a row-split lm_head.
//
// B200 design: the reference reduces a 151936-logit row in one CTA, which leaves the other SMs idle; here a token's
// row is cut into chunks of 4096 logits, one 256-thread CTA per chunk, 16-byte loads (four in flight per thread).
// Each CTA folds its best key into a per-token maximum with one atomic; the CTA that takes the token's last ticket
// (release/acquire) publishes the index and clears the maximum and the ticket. The maxima and tickets are file-scope
// device arrays (no allocation), so one stand-alone argmax may run at a time per device.
#include "fn_argmax.cuh"
#include "fn_engine.h"

namespace fn {

constexpr int AMX_CHUNK = 4096, AMX_THREADS = 256, AMX_MAXT = 1024;
__device__ unsigned long long g_amx_kacc[AMX_MAXT];
__device__ unsigned int g_amx_ticket[AMX_MAXT];

__global__ void __launch_bounds__(AMX_THREADS) k_argmax(const float *__restrict__ logits, int ls, int n,
                                                        int *__restrict__ out) {
    __shared__ unsigned long long s_k[AMX_THREADS / 32];
    const int t = blockIdx.y, c0 = blockIdx.x * AMX_CHUNK, c1 = min(n, c0 + AMX_CHUNK);
    pdl_wait();
    const float *l = after_wait(logits) + (size_t)t * ls;
    pdl_trigger();
    unsigned long long k = 0;
    if (((uintptr_t)(l + c0) & 15) == 0 && c1 - c0 == AMX_CHUNK) {
        const float4 *l4 = (const float4 *)(l + c0);
        float4 v[AMX_CHUNK / 4 / AMX_THREADS];
#pragma unroll
        for (int u = 0; u < AMX_CHUNK / 4 / AMX_THREADS; ++u) v[u] = __ldcs(l4 + threadIdx.x + u * AMX_THREADS);
#pragma unroll
        for (int u = 0; u < AMX_CHUNK / 4 / AMX_THREADS; ++u) {
            const int c = c0 + 4 * (threadIdx.x + u * AMX_THREADS);
            k = kmax(k, kmax(kmax(amax_key(v[u].x, c), amax_key(v[u].y, c + 1)),
                             kmax(amax_key(v[u].z, c + 2), amax_key(v[u].w, c + 3))));
        }
    } else {
        for (int c = c0 + threadIdx.x; c < c1; c += AMX_THREADS) k = kmax(k, amax_key(l[c], c));
    }
    k = warp_kmax(k);
    if ((threadIdx.x & 31) == 0) s_k[threadIdx.x >> 5] = k;
    __syncthreads();
    if (threadIdx.x >= 32) return;
    k = warp_kmax(threadIdx.x < AMX_THREADS / 32 ? s_k[threadIdx.x] : 0ull);
    if (threadIdx.x != 0) return;
    if (k) asm volatile("red.relaxed.gpu.global.max.u64 [%0], %1;" ::"l"(g_amx_kacc + t), "l"(k) : "memory");
    uint32_t tk;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(tk) : "l"(g_amx_ticket + t) : "memory");
    if (tk != gridDim.x - 1) return;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(k) : "l"(g_amx_kacc + t) : "memory");
    out[t] = amax_index(k);
    g_amx_kacc[t] = 0ull;
    g_amx_ticket[t] = 0u;
}

__global__ void k_argmax_keys(const unsigned long long *__restrict__ keys, int nranks, int nt, int *__restrict__ out) {
    pdl_wait();
    const unsigned long long *kp = after_wait(keys);
    pdl_trigger();
    const int t = threadIdx.x;
    if (t >= nt) return;
    unsigned long long k = 0;
    for (int r = 0; r < nranks; ++r) k = kmax(k, kp[(size_t)r * nt + t]);
    out[t] = amax_index(k);
}

// KeyExchange consumer: one warp. It first waits for the kernel before it (this rank's lm_head GEMV, whose publishing
// CTA also counted this rank's own arrival), so it only ever waits on other GPUs. Every lane then polls the n
// counters with acquire loads (bounded), lane t < nt reduces the n keys of token t for this call's parity, and
// lane 0 counts the call. On a timeout the outputs are -1 and the device error word says which wait gave up.
struct KeysCombineArgs {
    const unsigned long long *keys;
    const uint32_t *counters;
    uint32_t *calls;
    int n, nt;
    int *out;
    uint32_t *err;
};

__global__ void k_keys_combine(const KeysCombineArgs a) {
    pdl_wait();
    const int lane = threadIdx.x;
    const uint32_t c = *after_wait(a.calls);
    bool ok = true;
    for (int r = 0; r < a.n && ok; ++r) ok = wait_counter_sys(a.counters + r, c + 1);
    ok = __all_sync(0xffffffffu, ok);
    pdl_trigger();
    if (!ok) {
        if (lane == 0) dev_fail(a.err, DEV_PEER_TIMEOUT);
        if (lane < a.nt) a.out[lane] = -1;
        return;
    }
    if (lane < a.nt) {
        const int par = (int)(c & 1u);
        unsigned long long k = 0;
        for (int r = 0; r < a.n; ++r) k = kmax(k, a.keys[(par * MAX_RANKS + r) * 8 + lane]);
        a.out[lane] = amax_index(k);
    }
    __syncwarp();
    if (lane == 0) *a.calls = c + 1;
}

int launch_keys_combine(const unsigned long long *keys, const uint32_t *counters, uint32_t *calls, int n, int nt,
                        int *out, cudaStream_t s) {
    if (n < 1 || n > MAX_RANKS || nt < 1 || nt > 8) return fail("keys combine: bad shape");
    KeysCombineArgs a{keys, counters, calls, n, nt, out, dev_error_ptr()};
    const cudaError_t e = launch_k(k_keys_combine, dim3(1), dim3(32), 0, s, a);
    if (e != cudaSuccess) return fail(std::string("keys combine launch: ") + cudaGetErrorString(e));
    return 0;
}

int launch_argmax(const float *logits, int ls, int n, int nt, int *out, cudaStream_t s) {
    if (nt < 1 || nt > AMX_MAXT || n < 1 || ls < n) return fail("argmax: bad shape (1 <= nt <= 1024, n <= ls)");
    const cudaError_t e = launch_k(k_argmax, dim3((n + AMX_CHUNK - 1) / AMX_CHUNK, nt), dim3(AMX_THREADS), 0, s, logits,
                                   ls, n, out);
    if (e != cudaSuccess) return fail(std::string("argmax launch: ") + cudaGetErrorString(e));
    return 0;
}

int launch_argmax_keys(const unsigned long long *keys, int nranks, int nt, int *out, cudaStream_t s) {
    if (nt < 1 || nt > 1024 || nranks < 1) return fail("argmax keys: bad shape");
    const cudaError_t e = launch_k(k_argmax_keys, dim3(1), dim3(nt < 32 ? 32 : nt), 0, s, keys, nranks, nt, out);
    if (e != cudaSuccess) return fail(std::string("argmax keys launch: ") + cudaGetErrorString(e));
    return 0;
}

}  // namespace fn
