// Dequant-fused GEMV for batch-1 decode on B200 (sm_100a), and the row dequantiser.
//
// Reference behaviour: engine/faie2fn.cu:690-1042 (k_tgemv: y[t][r] (+)= sum_c W[r][c] x[t][c] for t < nt <= 8 on
// GGUF blocks, fixed-order sums that depend on the weight's shape only) and :1206-1217 (k_dequant_rows).
//
// B200 design (not the reference's): weights stay GGUF row-major, each row padded to a 16-byte stride. CTA b owns the
// contiguous rows [b*R/C, (b+1)*R/C) and streams them through a ring of `slots` shared-memory stages with bulk
// (non-tensor TMA) copies completing on mbarriers; thread 0 is the producer. Because the weights never depend on the
// previous kernel, the first `slots` stages are issued before griddepcontrol.wait, so under programmatic dependent
// launch the weight stream of this GEMV overlaps the tail of the kernel before it. x is staged once per CTA into a
// bank-conflict-free padded layout ([t][group][36] floats); for one token each lane then keeps its K-slice of x in
// registers. Lane l of a row (lpr lanes per row) owns groups l, l + lpr, ... of 32 values: it decodes each group in
// registers (Dec<TY>, bit-exact vs gguf-py) into four FMA chains, adds the chains (fp32), accumulates the group sums
// in double in group order, and the row's lanes meet in a double butterfly; the row result is rounded to fp32 once.
// A row never spans warps or CTAs, so there is no split-K scratch and no reduce kernel; the sum order is a function
// of (format, cols) alone.
#include "fn_engine.h"
#include "fn_rowdot.cuh"

#include <unordered_set>

namespace fn {

struct GemvArgs {
    const uint8_t *W;
    uint32_t ldw;
    int rows, G;
    const float *x;
    int xs;
    float *y;
    int ys, nt;
    int rps, slots;
    uint32_t stage_bytes, x_off, ring_off, grid_off;
    int acc, early;
    uint32_t *err;
};

template <uint32_t TY, int NT, int LPR, int GPL, bool XREG>
__global__ void __launch_bounds__(256, 1) k_gemv(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t *full = (uint64_t *)sm;
    uint8_t *ring = sm + a.ring_off;
    float *xsm = (float *)(sm + a.x_off);
    uint32_t *grid = (uint32_t *)(sm + a.grid_off);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const int r0 = (int)((long long)blockIdx.x * a.rows / gridDim.x);
    const int r1 = (int)((long long)(blockIdx.x + 1) * a.rows / gridDim.x);
    const int nst = (r1 - r0 + a.rps - 1) / a.rps;
    const int G = a.G;

    auto issue = [&](int st) {  // thread 0: stage st of this CTA's rows into its slot
        const int slot = st % a.slots, rr = r0 + st * a.rps, n = min(a.rps, r1 - rr);
        const uint32_t bytes = (uint32_t)n * a.ldw;
        mbar_arrive_tx(&full[slot], bytes);
        bulk_g2s(ring + (size_t)slot * a.stage_bytes, a.W + (size_t)rr * a.ldw, bytes, &full[slot]);
    };
    if (tid == 0) {
        for (int s = 0; s < a.slots; ++s) mbar_init(&full[s], 1);
        mbar_fence_init();
        for (int st = 0; st < min(nst, a.slots); ++st) issue(st);
    }
    stage_grid<TY>(grid);

    if (!a.early) pdl_wait();
    const float *x = after_wait(a.x);
    const int nt = a.nt;
    stage_x(xsm, x, a.xs, nt, G);
    __syncthreads();
    pdl_trigger();

    constexpr int RPW = 32 / LPR;  // rows a warp works on at once
    const int lr = lane % LPR, sub = lane / LPR;
    XReg<LPR, (GPL > 0 ? GPL : 1)> xr;
    if constexpr (XREG) xr.load(xsm, lr);

    int st = 0;
    for (; st < nst; ++st) {
        const int slot = st % a.slots;
        const uint32_t par = (uint32_t)(st / a.slots) & 1u;
        const bool ok = warp_wait(&full[slot], par);
        if (ok) {
            const uint8_t *sbuf = ring + (size_t)slot * a.stage_bytes;
            const int rr0 = r0 + st * a.rps, n = min(a.rps, r1 - rr0);
            for (int base = warp * RPW; base < n; base += nw * RPW) {
                const int row = base + sub;
                const bool valid = row < n;
                double acc[NT];
                row_dot<TY, NT, LPR, GPL, XREG>(sbuf + (size_t)row * a.ldw, grid, xr, xsm, G, lr, nt, valid, acc);
                if (valid && lr == 0) {
                    const int r = rr0 + row;
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        if (NT > 1 && t >= nt) break;
                        float *o = a.y + (size_t)t * a.ys + r;
                        const float v = __double2float_rn(acc[t]);
                        *o = a.acc ? __fadd_rn(*o, v) : v;
                    }
                }
            }
        }
        if (__syncthreads_or(!ok)) {
            if (tid == 0) dev_fail(a.err, DEV_WAIT_TIMEOUT);
            break;
        }
        if (tid == 0 && st + a.slots < nst) issue(st + a.slots);
    }
    if (st < nst && tid == 0) {  // wound down early: let the copies already issued land (bounded) before exiting
        for (int s2 = st; s2 < min(nst, st + a.slots); ++s2) mbar_wait(&full[s2 % a.slots], (uint32_t)(s2 / a.slots) & 1u, 1u << 16);
    }
    if (a.early) pdl_wait();
}

// ---------------------------------------------------------------------------------------------------------------
// row dequantiser: out[r][c] = dequant(W)[r][c]; one thread per 32-value group

template <uint32_t TY>
__global__ void k_dequant(const uint8_t *__restrict__ W, uint64_t rb, int rows, int G, float *__restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * G) return;
    const int r = (int)(i / G), g = (int)(i % G);
    const uint32_t *grid = dev_grid<TY>();
    float *o = out + ((size_t)r * G + g) * 32;
    Dec<TY>::group(W + (size_t)r * rb, g, grid, [&](int j, float v0, float v1, float v2, float v3) {
        *(float4 *)(o + j) = make_float4(v0, v1, v2, v3);
    });
}

int launch_dequant(uint32_t type, const uint8_t *W, uint64_t rb, int rows, int cols, float *out, cudaStream_t s) {
    if (cols % 32 || rows < 0 || row_bytes(type, cols) != rb) return fail("dequant: unsupported type/shape");
    if (rows == 0) return 0;
    const int G = cols / 32;
    const long long n = (long long)rows * G;
    const unsigned blocks = (unsigned)((n + 255) / 256);
    cudaError_t e = cudaSuccess;
    const bool known = dispatch_type(type, [&]<uint32_t TY>() { k_dequant<TY><<<blocks, 256, 0, s>>>(W, rb, rows, G, out); });
    if (!known) return fail("dequant: unsupported type " + std::to_string(type));
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail(std::string("dequant launch: ") + cudaGetErrorString(e));
    return 0;
}

// ---------------------------------------------------------------------------------------------------------------
// plan + launch

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// dynamic shared memory of a launch of plan p with nt tokens
static size_t gemv_smem(const GemvPlan &p, int nt) {
    return align_up(p.x_off + (size_t)nt * p.G * XPAD * 4, 128);
}

bool plan_gemv(GemvPlan &p, uint32_t type, int rows, int cols, int ntcap) {
    p = GemvPlan{};
    p.type = type;
    p.rows = rows;
    p.cols = cols;
    p.rb = row_bytes(type, cols);
    if (!p.rb || cols % 32 || rows < 1 || ntcap < 1 || ntcap > 8) return false;
    p.ldw = (uint32_t)align_up(p.rb, 16);
    p.G = cols / 32;
    p.ntcap = ntcap == 1 ? 1 : 8;
    p.lpr = p.G == 8 ? 8 : p.G == 16 ? 16 : 32;
    p.gpl = (p.G + p.lpr - 1) / p.lpr;
    p.xreg = p.ntcap == 1 && (p.G == 8 || p.G == 16 || p.G == 32 || p.G == 64);
    const Settings &S = settings();
    p.threads = 32 * std::max(1, std::min(S.warps_per_cta, 16));
    const int nw = p.threads / 32, rpw = 32 / p.lpr, pass = nw * rpw;
    // rows per stage: about stage_kb bytes, whole passes of the CTA's warps when a pass fits
    int rps = std::max(1, (int)((size_t)S.stage_kb * 1024 / p.ldw));
    if (rps >= pass) rps = rps / pass * pass;
    if (S.ov_rps > 0) rps = S.ov_rps;
    const int ctas_max = std::max(1, num_sms() * std::max(1, S.ctas_per_sm));
    p.ctas = std::min(ctas_max, (rows + rpw - 1) / rpw);
    const int rows_per_cta = (rows + p.ctas - 1) / p.ctas;
    p.rps = std::max(1, std::min(rps, rows_per_cta));
    p.stage_bytes = (uint32_t)align_up((size_t)p.rps * p.ldw, 128);
    const int stages_per_cta = (rows_per_cta + p.rps - 1) / p.rps;
    p.slots = (int)std::max<size_t>(2, (size_t)S.ring_kb * 1024 / p.stage_bytes);
    p.slots = std::max(1, std::min(p.slots, std::min(stages_per_cta, 16)));
    // layout: barriers | ring | codebook | x (sized per call by its token count: gemv_smem)
    p.ring_off = 128;
    p.grid_off = (uint32_t)align_up(p.ring_off + (size_t)p.slots * p.stage_bytes, 128);
    p.x_off = (uint32_t)align_up(p.grid_off + (size_t)grid_words(type) * 4, 128);
    p.smem = gemv_smem(p, p.ntcap);
    if (p.smem > 227 * 1024) p.smem = gemv_smem(p, 1);  // wide rows: fewer tokens per call fit (checked at launch)
    return p.smem <= 227 * 1024;
}

size_t plan_weight_bytes(const GemvPlan &p) { return (size_t)p.rows * p.ldw; }

template <uint32_t TY> static cudaError_t launch_t(const GemvPlan &p, const GemvArgs &a, size_t smem, cudaStream_t s) {
    void (*k)(const GemvArgs) = nullptr;
    if (p.ntcap == 1) {
        if (p.xreg) {
            if (p.lpr == 8) k = k_gemv<TY, 1, 8, 1, true>;
            else if (p.lpr == 16) k = k_gemv<TY, 1, 16, 1, true>;
            else if (p.gpl == 1) k = k_gemv<TY, 1, 32, 1, true>;
            else k = k_gemv<TY, 1, 32, 2, true>;
        } else {
            k = k_gemv<TY, 1, 32, 0, false>;
        }
    } else {
        if (p.lpr == 8) k = k_gemv<TY, 8, 8, 0, false>;
        else if (p.lpr == 16) k = k_gemv<TY, 8, 16, 0, false>;
        else k = k_gemv<TY, 8, 32, 0, false>;
    }
    static std::unordered_set<const void *> configured;  // one attribute call per kernel, outside graph capture
    if (!configured.count((const void *)k)) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured.insert((const void *)k);
    }
    return launch_k(k, dim3(p.ctas), dim3(p.threads), smem, s, a);
}

int launch_gemv(const GemvPlan &p, const uint8_t *W, const float *x, int xs, float *y, int ys, int nt, bool acc,
                bool early, cudaStream_t s) {
    if (nt < 1 || nt > p.ntcap) return fail("gemv: nt out of range for the plan");
    const size_t smem = gemv_smem(p, nt);
    if (smem > 227 * 1024) return fail("gemv: " + std::to_string(nt) + " tokens of " + std::to_string(p.cols) +
                                       " columns do not fit in shared memory");
    if (((uintptr_t)W & 15) || ((uintptr_t)x & 15) || (xs & 3)) return fail("gemv: W and x must be 16-byte aligned, xs % 4 == 0");
    GemvArgs a;
    a.W = W;
    a.ldw = p.ldw;
    a.rows = p.rows;
    a.G = p.G;
    a.x = x;
    a.xs = xs;
    a.y = y;
    a.ys = ys;
    a.nt = nt;
    a.rps = p.rps;
    a.slots = p.slots;
    a.stage_bytes = p.stage_bytes;
    a.x_off = p.x_off;
    a.ring_off = p.ring_off;
    a.grid_off = p.grid_off;
    a.acc = acc ? 1 : 0;
    a.early = early && settings().early && settings().pdl ? 1 : 0;
    a.err = dev_error_ptr();
    cudaError_t e = cudaSuccess;
    const bool known = dispatch_type(p.type, [&]<uint32_t TY>() { e = launch_t<TY>(p, a, smem, s); });
    if (!known) return fail("gemv: unsupported type " + std::to_string(p.type));
    if (e != cudaSuccess) return fail(std::string("gemv launch: ") + cudaGetErrorString(e));
    return 0;
}

}  // namespace fn
