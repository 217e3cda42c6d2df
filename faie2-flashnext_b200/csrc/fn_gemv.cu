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
// registers (load_group, bit-exact vs gguf-py) into four FMA chains, adds the chains (fp32), accumulates the group sums
// in double in group order, and the row's lanes meet in a double butterfly; the row result is rounded to fp32 once.
// A row never spans warps or CTAs, so there is no split-K scratch and no reduce kernel; the sum order is a function
// of (format, cols) alone.
#include "fn_gemv_impl.cuh"

namespace fn {

FN_GEMV_DECL(T_Q4_0) FN_GEMV_DECL(T_Q4_1) FN_GEMV_DECL(T_Q5_0) FN_GEMV_DECL(T_Q5_1) FN_GEMV_DECL(T_Q8_0)
FN_GEMV_DECL(T_Q2_K) FN_GEMV_DECL(T_Q3_K) FN_GEMV_DECL(T_Q4_K) FN_GEMV_DECL(T_Q5_K) FN_GEMV_DECL(T_Q6_K)
FN_GEMV_DECL(T_IQ2_XXS) FN_GEMV_DECL(T_IQ2_XS) FN_GEMV_DECL(T_IQ2_S) FN_GEMV_DECL(T_IQ3_XXS) FN_GEMV_DECL(T_IQ3_S)
FN_GEMV_DECL(T_IQ4_NL) FN_GEMV_DECL(T_IQ4_XS) FN_GEMV_DECL(T_BF16) FN_GEMV_DECL(T_Q2_0)

// ---------------------------------------------------------------------------------------------------------------
// plane repack at upload: GGUF rows (stride rb) -> plane rows (stride ldw), one thread per (row, block); formats
// without a plane layout are copied as they are

__global__ void k_plane_repack(const uint8_t *__restrict__ src, uint64_t rb, uint8_t *__restrict__ dst, uint32_t ldw,
                               int rows, int nb, int bytes, PlaneDesc pd) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * nb) return;
    const int r = (int)(i / nb), b = (int)(i % nb);
    const uint8_t *s = src + (size_t)r * rb + (size_t)b * bytes;
    uint8_t *d = dst + (size_t)r * ldw;
    if (pd.nf == 0) {
        for (int k = 0; k < bytes; ++k) d[(size_t)b * bytes + k] = s[k];
        return;
    }
    int plane = 0;
    for (int f = 0; f < pd.nf; ++f) {
        const Field fl = pd.f[f];
        for (int k = 0; k < fl.size; ++k) d[plane + (size_t)b * fl.size + k] = s[fl.off + k];
        plane += fl.size * nb;
    }
}

// formats with re-encoded quant planes: one thread per (row, block) writes the block's encoded planes
template <uint32_t TY>
__global__ void k_encode(const uint8_t *__restrict__ src, uint64_t rb, uint8_t *__restrict__ dst, uint32_t ldw, int rows,
                         int nb, int bytes) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * nb) return;
    const int r = (int)(i / nb), b = (int)(i % nb);
    encode_block<TY>(src + (size_t)r * rb + (size_t)b * bytes, dst + (size_t)r * ldw, b, nb);
}

int launch_plane_repack(uint32_t type, const uint8_t *src, uint64_t rb, uint8_t *dst, uint32_t ldw, int rows, int cols,
                        cudaStream_t s) {
    int qk, bytes;
    if (!type_info(type, qk, bytes) || cols % qk || row_bytes(type, cols) != rb) return fail("repack: bad type/shape");
    if (rows == 0) return 0;
    PlaneDesc pd;
    bool enc = false;
    const int nb = cols / qk;
    const long long n = (long long)rows * nb;
    const unsigned blocks = (unsigned)((n + 255) / 256);
    dispatch_type(type, [&]<uint32_t TY>() {
        pd = plane_desc<TY>();
        if constexpr (Encoded<TY>::v) {
            enc = true;
            k_encode<TY><<<blocks, 256, 0, s>>>(src, rb, dst, ldw, rows, nb, bytes);
        }
    });
    if (!enc) k_plane_repack<<<blocks, 256, 0, s>>>(src, rb, dst, ldw, rows, nb, bytes, pd);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(std::string("repack launch: ") + cudaGetErrorString(e));
    return 0;
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
    const auto v = load_group<TY>(W + (size_t)r * rb, g, grid);
#pragma unroll
    for (int j = 0; j < 32; j += 4) *(float4 *)(o + j) = v.quad(j);
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

// dynamic shared memory a GEMV may use: the SM's 227 KiB less 5 KiB for the kernel's static shared memory (x scale
// maxima, argmax keys)
constexpr size_t kDynSmem = 227 * 1024 - 5 * 1024;

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
    const int rpw = 32 / p.lpr, ru = rpw * (p.lpr == 32 ? 2 : 1);
    // every warp streams its own contiguous rows through its own ring of `slots` stages of ru rows
    p.rps = ru;
    p.stage_bytes = (uint32_t)align_up((size_t)ru * p.ldw, 128);
    // budget: x for the token capacity (one token if the capacity does not fit) and the codebook come first
    const size_t fixed = 1024 + (size_t)grid_words(type) * 4 + 128;  // barriers, codebook
    size_t xb = (size_t)p.ntcap * p.G * XPAD * 4;
    if (fixed + xb + 2 * (size_t)p.stage_bytes > kDynSmem) xb = (size_t)p.G * XPAD * 4;
    const size_t ring_budget = std::min<size_t>((size_t)S.ring_kb * 1024, kDynSmem - fixed - xb);
    // warps: the setting (S.warps_per_cta > 0), else by weight size, fewer when wide rows would leave less than two
    // stages per warp
    // (small weights: 4 warps, so that the CTAs of consecutive GEMVs fit on an SM together and overlap)
    const size_t wbytes = (size_t)rows * p.rb;
    int nw = S.warps_per_cta > 0 ? S.warps_per_cta : wbytes >= (64u << 20) ? 16 : wbytes >= (16u << 20) ? 8 : 4;
    nw = std::max(1, std::min(nw, 16));
    while (nw > 1 && (size_t)nw * 2 * p.stage_bytes > ring_budget) --nw;
    if ((size_t)nw * p.stage_bytes > ring_budget) return false;
    p.threads = 32 * nw;
    const int ctas_max = std::max(1, num_sms() * std::max(1, S.ctas_per_sm));
    p.ctas = std::min(ctas_max, (rows + ru - 1) / ru);
    const int rows_per_warp = (int)((rows + (size_t)p.ctas * nw - 1) / ((size_t)p.ctas * nw));
    const int stages_per_warp = std::max(1, (rows_per_warp + ru - 1) / ru);
    p.slots = (int)std::max<size_t>(1, ring_budget / ((size_t)nw * p.stage_bytes));
    p.slots = std::max(1, std::min(p.slots, std::min(stages_per_warp, 8)));
    // layout: barriers (nw x slots) | rings | codebook | x (sized per call by its token count: gemv_smem)
    p.ring_off = (uint32_t)align_up((size_t)nw * p.slots * 8, 128);
    p.grid_off = (uint32_t)align_up(p.ring_off + (size_t)nw * p.slots * p.stage_bytes, 128);
    p.x_off = (uint32_t)align_up(p.grid_off + (size_t)grid_words(type) * 4, 128);
    p.smem = gemv_smem(p, p.ntcap);
    if (p.smem > kDynSmem) p.smem = gemv_smem(p, 1);  // wide rows: fewer tokens per call fit (checked at launch)
    return p.smem <= kDynSmem;
}

size_t plan_weight_bytes(const GemvPlan &p) { return (size_t)p.rows * p.ldw; }

int launch_gemv(const GemvPlan &p, const uint8_t *W, const float *x, int xs, float *y, int ys, int nt, bool acc,
                bool early, cudaStream_t s, const GemvArgmax *am) {
    if (nt < 1 || nt > p.ntcap) return fail("gemv: nt out of range for the plan");
    // Q4_K / Q6_K on the tensor cores (integer products), cap tokens per launch: a token's result is the same in any
    // batch (a row-split argmax exchange counts calls, so it takes one launch or the CUDA cores)
    const int cap = settings().qmma ? qmma_cap(p.type, p.cols) : 0;
    if (cap > 0 && !(am && am->xr && nt > cap)) {
        for (int t0 = 0; t0 < nt; t0 += cap) {
            const int n = std::min(cap, nt - t0);
            GemvArgmax a2;
            if (am) {
                a2 = *am;
                if (a2.index) a2.index += t0;
                if (a2.key) a2.key += t0;
            }
            const int rc = launch_qmma(p, W, x + (size_t)t0 * xs, xs, y ? y + (size_t)t0 * ys : nullptr, ys, n, acc,
                                       early, s, am ? &a2 : nullptr);
            if (rc) return rc;
        }
        return 0;
    }
    const size_t smem = gemv_smem(p, nt);
    if (smem > kDynSmem) return fail("gemv: " + std::to_string(nt) + " tokens of " + std::to_string(p.cols) +
                                       " columns do not fit in shared memory");
    if (((uintptr_t)W & 15) || ((uintptr_t)x & 15) || (xs & 3)) return fail("gemv: W and x must be 16-byte aligned, xs % 4 == 0");
    GemvArgs a;
    a.W = W;
    a.ldw = p.ldw;
    a.rows = p.rows;
    a.G = p.G;
    int qk_, bytes_;
    type_info(p.type, qk_, bytes_);
    a.nb = p.cols / qk_;
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
    a.pf = p.pf;
    a.pf_bytes = p.pf_bytes;
    a.nw = p.nw;
    a.eps = p.eps;
    if (p.nw && ((uintptr_t)p.nw & 15)) return fail("gemv: the norm weight must be 16-byte aligned");
    a.err = dev_error_ptr();
    a.amx = 0;
    a.row0 = 0;
    a.aidx = nullptr;
    a.akey = a.kacc = nullptr;
    a.ticket = nullptr;
    a.xr = KeyExchange{};
    if (am) {
        if (!am->kacc || !am->ticket || (!am->index && !am->key && !am->xr))
            return fail("gemv argmax: missing scratch or outputs");
        if (am->row0 < 0 || (long long)am->row0 + p.rows > 0x7FFFFFFFll) return fail("gemv argmax: row0 out of range");
        a.amx = 1;
        a.row0 = am->row0;
        a.aidx = am->index;
        a.akey = am->key;
        a.kacc = am->kacc;
        a.ticket = am->ticket;
        if (am->xr) {
            const KeyExchange &x = *am->xr;
            if (x.n < 1 || x.n > MAX_RANKS || x.rank < 0 || x.rank >= x.n || !x.calls) return fail("gemv argmax: bad key exchange");
            for (int r = 0; r < x.n; ++r)
                if (!x.keys[r] || !x.counters[r]) return fail("gemv argmax: key exchange without peer memory");
            a.xr = x;
        }
    } else if (!y) {
        return fail("gemv: y is null");
    }
    cudaError_t e = cudaSuccess;
    const bool known = dispatch_type(p.type, [&]<uint32_t TY>() { e = gemv_launch_t<TY>(p, a, smem, s); });
    if (!known) return fail("gemv: unsupported type " + std::to_string(p.type));
    if (e != cudaSuccess) return fail(std::string("gemv launch: ") + cudaGetErrorString(e));
    return 0;
}

}  // namespace fn
