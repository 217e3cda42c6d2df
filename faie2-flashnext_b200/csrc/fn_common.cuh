// Shared definitions of the B200 decode engine: ggml type table, device error word, mbarrier / bulk-copy
// (TMA, non-tensor) / programmatic-dependent-launch primitives. sm_100a only.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#define FN_API extern "C" __attribute__((visibility("default")))

namespace fn {

// ---------------------------------------------------------------------------------------------------------------
// ggml type ids (engine/faie2fn.cu:78-81 for the reference's 13, gguf-py GGML_QUANT_SIZES for the six it lacks)
enum : uint32_t {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11,
    T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_IQ2_XXS = 16, T_IQ2_XS = 17, T_IQ3_XXS = 18, T_IQ4_NL = 20,
    T_IQ3_S = 21, T_IQ2_S = 22, T_IQ4_XS = 23, T_BF16 = 30, T_Q2_0 = 42,
};

// values per block and bytes per block (engine/faie2fn.cu:84-103 type_info); false for types the engine does not read
inline bool type_info(uint32_t t, int &qk, int &bytes) {
    switch (t) {
        case T_Q4_0: qk = 32; bytes = 18; return true;
        case T_Q4_1: qk = 32; bytes = 20; return true;
        case T_Q5_0: qk = 32; bytes = 22; return true;
        case T_Q5_1: qk = 32; bytes = 24; return true;
        case T_Q8_0: qk = 32; bytes = 34; return true;
        case T_Q2_K: qk = 256; bytes = 84; return true;
        case T_Q3_K: qk = 256; bytes = 110; return true;
        case T_Q4_K: qk = 256; bytes = 144; return true;
        case T_Q5_K: qk = 256; bytes = 176; return true;
        case T_Q6_K: qk = 256; bytes = 210; return true;
        case T_IQ2_XXS: qk = 256; bytes = 66; return true;
        case T_IQ2_XS: qk = 256; bytes = 74; return true;
        case T_IQ3_XXS: qk = 256; bytes = 98; return true;
        case T_IQ4_NL: qk = 32; bytes = 18; return true;
        case T_IQ3_S: qk = 256; bytes = 110; return true;
        case T_IQ2_S: qk = 256; bytes = 82; return true;
        case T_IQ4_XS: qk = 256; bytes = 136; return true;
        case T_BF16: qk = 1; bytes = 2; return true;
        case T_Q2_0: qk = 64; bytes = 18; return true;
        default: return false;
    }
}

// bytes of one GGUF row of `cols` values (0: unknown type or not a whole number of blocks; engine/faie2fn.cu:105-109)
inline uint64_t row_bytes(uint32_t t, uint64_t cols) {
    int qk, b;
    if (!type_info(t, qk, b) || cols % qk) return 0;
    return cols / qk * b;
}

// shared-memory words of the IQ codebook of a format, with any table derived from it (0 for formats without one)
inline int grid_words(uint32_t t) {
    switch (t) {
        case T_IQ2_XXS: return 512;
        case T_IQ2_XS: return 1024;
        case T_IQ2_S: return 2048;
        case T_IQ3_XXS: return 256 + 8192;  // the codebook, then its signed bf16 expansion (stage_grid)
        case T_IQ3_S: return 512;
        default: return 0;
    }
}

// ---------------------------------------------------------------------------------------------------------------
// host errors: 0 ok, -1 error with the message in err() (engine/faie2fn.cu:114-118)
std::string &err();
int fail(const std::string &msg);
#define FN_CK(x)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (x);                                                                      \
        if (e_ != cudaSuccess) return ::fn::fail(std::string(#x) + " -> " + cudaGetErrorString(e_)); \
    } while (0)

// device error word: a kernel whose bounded wait ran out records a code here and returns instead of hanging
enum : uint32_t { DEV_OK = 0, DEV_WAIT_TIMEOUT = 1, DEV_BAD_ARG = 2, DEV_PEER_TIMEOUT = 3 };
// every call site that can record an error compares the word after its kernels; returns -1 with a message if set
int check_dev_error(const char *where);
uint32_t *dev_error_ptr();  // device address of the error word of the current device

// ---------------------------------------------------------------------------------------------------------------
// device primitives

__device__ __forceinline__ void dev_fail(uint32_t *errw, uint32_t code) {
    if (errw) atomicCAS(errw, 0u, code);
}

// L2 prefetch of [p, p + bytes): this CTA's even share of the grid's, by thread 0, in pieces of at most 64 KiB (p and
// bytes 16-byte multiples). A hint for data a later kernel reads: nothing waits for it.
__device__ __forceinline__ void l2_prefetch_share(const uint8_t *p, uint64_t bytes) {
    if (!p || !bytes || threadIdx.x != 0) return;
    const uint64_t nb = (uint64_t)gridDim.x * gridDim.y * gridDim.z;
    const uint64_t b = ((uint64_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    const uint64_t per = ((bytes + nb - 1) / nb + 15) & ~15ull;
    uint64_t lo = b * per;
    const uint64_t hi = lo + per < bytes ? lo + per : bytes;
    for (; lo < hi; lo += 65536) {
        const uint32_t n = (uint32_t)(hi - lo < 65536 ? hi - lo : 65536) & ~15u;
        if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p + lo), "r"(n) : "memory");
    }
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }

// one arrival that also announces `bytes` of transactions (the bulk copies that complete on this barrier)
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// Wait for the phase of `parity` to complete, giving up after ~`limit` polls (each poll may suspend the thread for a
// hardware-chosen interval). Returns false on timeout; the caller records the error and winds down.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit = 1u << 24) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// The global nanosecond timer.
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for the phase of `parity` that parks the thread in the hardware until the phase completes (try_wait with
// a suspend-time hint) instead of re-issuing polls, so waiting warps leave their scheduler's issue slots to the
// working ones; false after about a second of the global timer.
__device__ __forceinline__ bool mbar_park(uint64_t *bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    uint64_t t0 = 0;
    for (;;) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(parity), "r"(20000u)
            : "memory");
        if (done) return true;
        const uint64_t t = global_ns();
        if (t0 == 0) t0 = t;
        else if (t - t0 > 1000000000ull) return false;
    }
}

// bulk (non-tensor) copy global -> shared, completing `bytes` of transactions on `bar`. dst, src 16-byte aligned,
// bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Programmatic dependent launch. A kernel stages what does not depend on its predecessor (weights), then pdl_wait()
// before it reads activations, then pdl_trigger() so its successor may start staging. Data written by the
// predecessor is read through after_wait(p), whose value comes from an asm statement ordered after the wait, so no
// load through it can be hoisted above the wait (engine/faie2fn.cu:311-329 states the same protocol).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
template <typename P> __device__ __forceinline__ P after_wait(P p) {
    asm volatile("" : "+l"(p));
    return p;
}

// Bounded wait until the 32-bit counter at p (in this GPU's memory, written by peer GPUs with release atomics)
// reaches `target` (wrap-safe), polling with acquire loads at system scope; false after ~`limit` polls (about a second).
__device__ __forceinline__ bool wait_counter_sys(const uint32_t *p, uint32_t target, uint32_t limit = 1u << 22) {
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if ((int32_t)(v - target) >= 0) return true;
        __nanosleep(256);
    }
    return false;
}
__device__ __forceinline__ void red_release_sys_add(uint32_t *p, uint32_t v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

}  // namespace fn
