// Gated-DeltaNet decode core on B200 (sm_100a): conv + silu + l2norm + gates + delta rule + gated RMSNorm for nt
// tokens of one layer, in one kernel (16 key heads, 32 value heads, head dim 128).
//
// Reference behaviour: k_gdn (engine/faie2fn.cu:1349-1431); value head h reads key head h % NKH (GGUF tiled order,
// :10-11, 1374); the norm is gated with sigmoid(z) (:1424); softplus(u) = u for u > 20 (:1411).
//
// B200 design (one sequence): value head h is a cluster of GDN_SPLIT = 4 CTAs of 384 threads; CTA p owns state columns
// [32p, 32p + 32): thread (jl, c) = (tid >> 2, tid & 3) of the first 128 owns column 32p + jl, key rows [32c, 32c + 32),
// i.e. 32 fp32 values of S[h] held in registers across all tokens of the launch, so a head's 64 KB state streams
// through four SMs. The columns are independent up to the gated norm: its sum of squares over the 128 columns is the
// 16 warp partials (4 per CTA) added in column order through distributed shared memory, so every value equals the
// one-CTA-per-head arrangement's. Every CTA of a head computes the conv, silu and l2 norm of all 128 q and k channels
// (the dot products need them all) and only its own 32 value channels. The four quarter-column partial dot products
// (S^T k, S^T q) meet by two xor shuffles inside a warp, in a fixed order. When
// the caller says the state was complete before the previous kernel started (in a decode step the layer's previous
// GDN launch is several kernels back), the state is loaded BEFORE griddepcontrol.wait, so under programmatic
// dependent launch its HBM read overlaps the projection GEMVs before this kernel; back-to-back launches of one layer
// load it after the wait. The step's own inputs (qkv, z, ab) are always read after the wait.
// Conv state: the value channels keep [3][NVH*DS]; every value head keeps its own copy of its key head's q/k conv
// state ([NVH][3][2][DS]): the value heads sharing a key head would otherwise race on it (one reading the old state
// while another writes the new one); the copies stay equal. Inside a head's cluster the CTA that owns a channel's column
// block writes its history back, after the cluster barrier that follows every other CTA's read of it.
//
// B200 design (a batch of sequences, one token each): one 512-thread CTA per (value head, sequence), no cluster. The
// head's 64 KB state arrives in shared memory by one bulk copy (before griddepcontrol.wait under the same condition as
// above), is updated there and leaves by one bulk store, so a CTA needs 64 registers (40 at three CTAs per SM) and
// several CTAs share an SM, one's copy overlapping another's arithmetic. A warp's lanes take 32 consecutive columns of
// one 32-row quarter (conflict-free shared-memory rows); the quarter partials meet in shared memory in the order the
// xor shuffles give, and the gated norm adds the same partials in the same order, so the values are the same bits.
#include <cooperative_groups.h>

#include "fn_engine.h"
#include "fn_gdn.h"

namespace cg = cooperative_groups;

namespace fn {

constexpr int GDN_DS = 128;
constexpr int GDN_SPLIT = 4;                            // CTAs (one cluster) per value head of one sequence
// threads: the q, k and value conv channels (3 DS), and 4 per state column of the CTA (4 DS / SPLIT), whichever is more
constexpr int gdn_threads(int split) { return 3 * GDN_DS > 4 * GDN_DS / split ? 3 * GDN_DS : 4 * GDN_DS / split; }
constexpr int KPAD = 36;  // floats per 32-row chunk of the staged q / k (32 + 4: chunk c at bank offset 4c)

struct GdnArgs {
    const float *qkv;  // [nt][qs]: q (nkh*ds) | k (nkh*ds) | v (nvh*ds)
    int qs;
    const float *z;  // [nt][zs]
    int zs;
    const float *ab;  // [nt][abs_]: alpha (nvh) | beta (nvh)
    int abs_;
    const float4 *conv_w;  // [convch] taps (oldest .. current)
    const float *dt_bias, *ssm_a, *norm_w;
    float *S;       // [nvh][ds][ds]
    float *cst_v;   // [3][nvh*ds]
    float *cst_qk;  // [nvh][3][2][ds]
    float *out;     // [nt][os]
    int os;
    int nkh, nvh, nt;
    int prefetch;  // 1: the state was complete before the previous kernel started, so it is read before the wait
    uint32_t *err;  // device error word (a bounded wait that ran out)
};

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// SPLIT CTAs per value head: 4 (a cluster) for one sequence, whose head's state then streams through four SMs; 1 for a
// batch of sequences (one 512-thread CTA per head and sequence: the batch fills the GPU, and no cluster barriers). The
// gated norm adds the same warp partials in the same column order either way, so the results are the same bits.
// MINB: CTAs per SM the registers must allow (one CTA per head: 2 at 64 registers, or 3 at 40 for batches whose CTAs
// fill three per SM; the shared-memory state allows three)
template <int SPLIT, int MINB = 1>
__global__ void __launch_bounds__(gdn_threads(SPLIT), MINB) k_gdn(const GdnArgs a) {  // clusters of SPLIT CTAs
    constexpr int DS = GDN_DS, CW = DS / SPLIT;  // CW state columns per CTA
    constexpr int NSW = 4 * CW / 32;             // warps holding state
    __shared__ __align__(16) float qn[4 * KPAD], kn[4 * KPAD], vs[CW];
    __shared__ float red_q[4], red_k[4];
    __shared__ float red_o[2][NSW];  // this CTA's warp partials of sum o^2, by token parity (read by the cluster)
    // one CTA per head: the 4 row-quarter partials of S^T k and S^T q per column, and o^2 per column
    __shared__ float red_kv[SPLIT == 1 ? 4 * DS : 1], red_qo[SPLIT == 1 ? 4 * DS : 1], red_sq[SPLIT == 1 ? DS : 1];
    // one CTA per head: the head's whole state (64 KiB, dynamic shared memory) arrives by one bulk copy on st_bar, so
    // the load is a single request to the copy engine instead of 32 scalar loads per thread
    extern __shared__ __align__(128) float st_sm[];
    __shared__ __align__(8) uint64_t st_bar;
    cg::cluster_group cl = cg::this_cluster();
    const int p = SPLIT > 1 ? (int)cl.block_rank() : 0;  // column block: state columns [CW p, CW (p + 1)) of the head
    const int h = blockIdx.x / SPLIT, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // state threads (tid < 4 CW): column j, rows [32c, 32c + 32). A cluster CTA gives a column's 4 quarters to
    // adjacent lanes (their partials meet by xor shuffles); one CTA per head puts a warp's lanes on 32 consecutive
    // columns of one quarter, so each state load and store of a warp is one 128-byte line (the partials then meet in
    // shared memory, added in the same order)
    const int jl = SPLIT == 1 ? 32 * (warp & 3) + lane : tid >> 2, c = SPLIT == 1 ? warp >> 2 : tid & 3;
    const int j = CW * p + jl;
    const bool st_thr = tid < 4 * CW;
    const int kh = h % a.nkh, nvd = a.nvh * DS;
    // a batch of independent sequences (gridDim.y > 1, one token each): sequence blockIdx.y's state, conv histories
    // and token row
    const int bq = blockIdx.y;
    float *const stS = a.S + (size_t)bq * a.nvh * DS * DS;
    float *const stQK = a.cst_qk + (size_t)bq * a.nvh * 3 * 2 * DS;
    float *const stV = a.cst_v + (size_t)bq * 3 * nvd;
    // conv roles: threads 0..127 q channel d, 128..255 k channel d (every CTA of the head computes all 256, so each
    // has the whole normalised q and k; only the owner of d's column block writes its history back), 256..256+CW-1
    // value channel CW p + d
    const int role = tid >> 7;
    int d = tid & 127, ch = -1;
    float *stp = nullptr;
    int sst = 0;  // state stride between the 3 history slots
    bool own = false;
    if (role == 0) {
        ch = kh * DS + d;
        stp = stQK + (size_t)h * 3 * 2 * DS + d;
        sst = 2 * DS;
        own = d / CW == p;
    } else if (role == 1) {
        ch = a.nkh * DS + kh * DS + d;
        stp = stQK + (size_t)h * 3 * 2 * DS + DS + d;
        sst = 2 * DS;
        own = d / CW == p;
    } else if (role == 2 && d < CW) {
        d += CW * p;
        ch = 2 * a.nkh * DS + h * DS + d;
        stp = stV + (size_t)h * DS + d;
        sst = nvd;
        own = true;
    }
    // ---- state, conv state, parameters: read before griddepcontrol.wait when the state was complete before the
    // previous kernel started (prefetch), else after it (the previous kernel may be this layer's previous step)
    float s[SPLIT == 1 ? 1 : 32];
    float *Sh = stS + (size_t)h * DS * DS;
    float h0 = 0.f, h1 = 0.f, h2 = 0.f;
    float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (SPLIT == 1) {
        if (tid == 0) {
            mbar_init(&st_bar, 1);
            mbar_fence_init();
        }
        __syncthreads();
    }
    bool st_ok = true;  // the state copy landed within the wait's bound
    // this thread's state value i (row 32c + i of column j): in registers for a cluster CTA, in the staged shared
    // copy for one CTA per head (two CTAs then share an SM, so one's copy overlaps the other's arithmetic)
    auto sv = [&](int i) -> float & {
        if constexpr (SPLIT == 1) return st_sm[(32 * c + i) * DS + jl];
        else return s[i];
    };
    auto load_state = [&]() {
        if constexpr (SPLIT == 1) {
            if (tid == 0) {
                mbar_arrive_tx(&st_bar, DS * DS * 4);
                bulk_g2s(st_sm, Sh, DS * DS * 4, &st_bar);
            }
        } else if (st_thr) {
#pragma unroll
            for (int i = 0; i < 32; ++i) sv(i) = Sh[(size_t)(32 * c + i) * DS + j];
        }
        if (ch >= 0) {
            h0 = stp[0];
            h1 = stp[sst];
            h2 = stp[2 * sst];
        }
    };
    if (a.prefetch) load_state();
    if (ch >= 0) w = a.conv_w[ch];
    const float nwj = st_thr ? a.norm_w[j] : 0.f, dtb = a.dt_bias[h], sa = a.ssm_a[h];
    pdl_wait();
    pdl_trigger();
    if (!a.prefetch) {
        Sh = after_wait(Sh);
        if (stp) stp = after_wait(stp);
        load_state();
    }
    const float *qkv = after_wait(a.qkv) + (size_t)bq * a.qs;
    const float *zp = after_wait(a.z) + (size_t)bq * a.zs;
    const float *abp = after_wait(a.ab) + (size_t)bq * a.abs_;
    float *const outp = a.out + (size_t)bq * a.os;

    for (int t = 0; t < a.nt; ++t) {
        // conv + silu of this thread's channel; history shifts
        float y = 0.f;
        if (ch >= 0) {
            const float x = qkv[(size_t)t * a.qs + ch];
            y = silu(__fmaf_rn(w.w, x, __fmaf_rn(w.z, h2, __fmaf_rn(w.y, h1, __fmul_rn(w.x, h0)))));
            h0 = h1;
            h1 = h2;
            h2 = x;
        }
        // l2 norms of q (threads 0..127) and k (128..255): warp sums, then the 4 partials in order
        const float sq = warp_sum_f(y * y);
        if (lane == 0) {
            if (role == 0) red_q[warp] = sq;
            else if (role == 1) red_k[warp - 4] = sq;
        }
        if (role == 2 && ch >= 0) vs[d - CW * p] = y;
        __syncthreads();
        if (role <= 1) {
            const float* r = role == 0 ? red_q : red_k;
            const float inv = rsqrtf(((r[0] + r[1]) + (r[2] + r[3])) + 1e-6f);
            float *dst = role == 0 ? qn : kn;
            dst[(d >> 5) * KPAD + (d & 31)] = y * inv;
        }
        // gates of this value head
        const float beta = sigm(abp[(size_t)t * a.abs_ + a.nvh + h]);
        const float u = abp[(size_t)t * a.abs_ + h] + dtb;
        const float sp = u > 20.0f ? u : log1pf(expf(u));
        const float decay = expf(sp * sa);
        __syncthreads();
        float o = 0.f;
        if constexpr (SPLIT == 1) {
            if (t == 0) {  // the state copy landed: this thread's 32 values of column j (a warp reads 32 consecutive words)
                st_ok = mbar_park(&st_bar, 0);
                if (!st_ok) dev_fail(a.err, DEV_WAIT_TIMEOUT);
            }
        }
        if (st_thr) {
            // kv_j = sum_i S[i][j] k_i over this thread's quarter, then the 4 quarters
            const float *kq = kn + c * KPAD, *qq = qn + c * KPAD;
            float kv = 0.f;
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                const float4 kk = *(const float4 *)(kq + i);
                kv = __fmaf_rn(sv(i), kk.x, kv);
                kv = __fmaf_rn(sv(i + 1), kk.y, kv);
                kv = __fmaf_rn(sv(i + 2), kk.z, kv);
                kv = __fmaf_rn(sv(i + 3), kk.w, kv);
            }
            if constexpr (SPLIT == 1) {  // every thread holds state here: the barrier is reached by all
                red_kv[c * DS + jl] = kv;
                __syncthreads();
                kv = (red_kv[jl] + red_kv[DS + jl]) + (red_kv[2 * DS + jl] + red_kv[3 * DS + jl]);
            } else {  // lanes c = 0..3: ((p0 + p1) + (p2 + p3)) in every lane
                kv += __shfl_xor_sync(0xffffffffu, kv, 1);
                kv += __shfl_xor_sync(0xffffffffu, kv, 2);
            }
            const float delta = __fmul_rn(__fmaf_rn(-decay, kv, vs[jl]), beta);
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                const float4 kk = *(const float4 *)(kq + i), q4 = *(const float4 *)(qq + i);
                sv(i) = __fmaf_rn(decay, sv(i), __fmul_rn(kk.x, delta));
                sv(i + 1) = __fmaf_rn(decay, sv(i + 1), __fmul_rn(kk.y, delta));
                sv(i + 2) = __fmaf_rn(decay, sv(i + 2), __fmul_rn(kk.z, delta));
                sv(i + 3) = __fmaf_rn(decay, sv(i + 3), __fmul_rn(kk.w, delta));
                o = __fmaf_rn(sv(i), q4.x, o);
                o = __fmaf_rn(sv(i + 1), q4.y, o);
                o = __fmaf_rn(sv(i + 2), q4.z, o);
                o = __fmaf_rn(sv(i + 3), q4.w, o);
            }
            if constexpr (SPLIT == 1) {
                red_qo[c * DS + jl] = o;
                __syncthreads();
                o = (red_qo[jl] + red_qo[DS + jl]) + (red_qo[2 * DS + jl] + red_qo[3 * DS + jl]);
            } else {
                o += __shfl_xor_sync(0xffffffffu, o, 1);
                o += __shfl_xor_sync(0xffffffffu, o, 2);
            }
            o *= 0.08838834764831845f;  // 1 / sqrt(128)
            if constexpr (SPLIT == 1) {
                if (c == 0) red_sq[jl] = o * o;
            } else {
                // gated RMSNorm over the head's 128 columns: this warp's 8 columns (lanes with c == 0), in lane order
                const float oo = warp_sum_f(c == 0 ? o * o : 0.f);
                if (lane == 0) red_o[t & 1][warp] = oo;
            }
        }
        // the head's 16 warp partials (NSW per CTA of the cluster, CTA p holding columns [CW p, CW (p + 1))), summed in
        // column order (through distributed shared memory when the head spans a cluster)
        if constexpr (SPLIT > 1) cl.sync();
        else __syncthreads();
        if (st_thr && c == 0) {
            float ss = 0.f;
            if constexpr (SPLIT == 1) {
                // the cluster form's sum: per block of 8 columns the xor-16 / 8 / 4 butterfly over its lanes 0, 4, ..,
                // 28, i.e. ((q0 + q4) + (q2 + q6)) + ((q1 + q5) + (q3 + q7)), then the 16 blocks in column order
#pragma unroll
                for (int b = 0; b < DS / 8; ++b) {
                    const float *q8 = red_sq + 8 * b;
                    ss += ((q8[0] + q8[4]) + (q8[2] + q8[6])) + ((q8[1] + q8[5]) + (q8[3] + q8[7]));
                }
            } else {
#pragma unroll
                for (int q = 0; q < SPLIT; ++q) {
                    const float *ro = cl.map_shared_rank(&red_o[t & 1][0], q);
#pragma unroll
                    for (int i = 0; i < NSW; ++i) ss += ro[i];
                }
            }
            const float r = rsqrtf(ss / DS + 1e-6f);
            const size_t oi = (size_t)h * DS + j;
            outp[(size_t)t * a.os + oi] = o * r * nwj * sigm(zp[(size_t)t * a.zs + oi]);
        }
        __syncthreads();
    }
    if constexpr (SPLIT == 1) {
        // the updated state leaves shared memory by one bulk store: every writer orders its shared-memory writes
        // before the copy engine's reads (proxy fence + barrier); the CTA exits once the engine has read them
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(Sh), "r"(smem_u32(st_sm)),
                         "r"(DS * DS * 4)
                         : "memory");
            asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
            asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
        }
    } else if (st_thr) {
#pragma unroll
        for (int i = 0; i < 32; ++i) Sh[(size_t)(32 * c + i) * DS + j] = sv(i);
    }
    if (ch >= 0 && own) {
        stp[0] = h0;
        stp[sst] = h1;
        stp[2 * sst] = h2;
    }
    if constexpr (SPLIT > 1) cl.sync();  // no CTA leaves while another may still read its partials
    if constexpr (SPLIT == 1)
        if (!st_ok) (void)mbar_park(&st_bar, 0);  // a copy past the first bound: let it land (bounded) before exiting
}

int launch_gdn(const GdnParams &p, const GdnState &st, const float *qkv, int qs, const float *z, int zs, const float *ab,
               int abs_, float *out, int os, int nt, bool prefetch_state, cudaStream_t s, int batch) {
    if (p.ds != GDN_DS) return fail("gdn: head dim must be 128");
    if (p.nkh < 1 || p.nvh < 1 || p.nvh % p.nkh) return fail("gdn: value heads must be a multiple of key heads");
    if (nt < 1) return fail("gdn: nt < 1");
    if (batch < 1 || (batch > 1 && nt != 1)) return fail("gdn: a batch of sequences runs one token each");
    if (((uintptr_t)p.conv_w & 15)) return fail("gdn: conv weights must be 16-byte aligned");
    GdnArgs a;
    a.qkv = qkv;
    a.qs = qs;
    a.z = z;
    a.zs = zs;
    a.ab = ab;
    a.abs_ = abs_;
    a.conv_w = (const float4 *)p.conv_w;
    a.dt_bias = p.dt_bias;
    a.ssm_a = p.ssm_a;
    a.norm_w = p.norm_w;
    a.S = st.S;
    a.cst_v = st.conv_v;
    a.cst_qk = st.conv_qk;
    a.out = out;
    a.os = os;
    a.nkh = p.nkh;
    a.nvh = p.nvh;
    a.nt = nt;
    a.prefetch = prefetch_state ? 1 : 0;
    a.err = dev_error_ptr();
    // a batch: three CTAs per SM once they fill three per SM (32 sequences x 32 heads: 31.4 us against 33.7 at two),
    // else two (8 x 32: 7.8 us against 9.6 at three, which leaves SMs idle)
    void (*kb)(const GdnArgs) = p.nvh * batch >= 3 * num_sms() ? k_gdn<1, 3> : k_gdn<1, 2>;
    if (batch > 1) {
        const cudaError_t e = allow_max_dynamic_smem(kb);
        if (e != cudaSuccess) return fail(std::string("gdn attributes: ") + cudaGetErrorString(e));
    }
    const cudaError_t e = batch > 1 ? launch_k(kb, dim3(p.nvh, batch), dim3(gdn_threads(1)), GDN_DS * GDN_DS * 4, s, a)
                                    : launch_kc(k_gdn<GDN_SPLIT>, dim3(p.nvh * GDN_SPLIT, 1), dim3(gdn_threads(GDN_SPLIT)),
                                                GDN_SPLIT, 0, s, a);
    if (e != cudaSuccess) return fail(std::string("gdn launch: ") + cudaGetErrorString(e));
    return 0;
}

}  // namespace fn
