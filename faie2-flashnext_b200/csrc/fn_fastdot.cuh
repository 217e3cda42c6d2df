// Fast group dot products of the dense GEMV and the expert kernels, on the engine's plane layout.
//
// Plane layout ("SoA rows"): at upload every GGUF row is byte-permuted so that each field of the format's blocks is
// a contiguous plane: row = [field 0 of blocks 0..nb-1][field 1 of blocks 0..nb-1]..., in the field order of
// PlaneSpec<TY>. A pure permutation of the row's bytes (nothing is converted or added), chosen so the quant planes
// of every block start on 16-byte boundaries and a lane reads its 32-value group with 128-bit shared-memory loads
// even for formats whose GGUF blocks are only 2-byte aligned (Q6_K 210 B, Q8_0 34 B, IQ3_XXS 98 B, ...).
//
// Fast<TY>::group(row, nb, g, grid, xa, nt, r) adds to r[t] the dot product of the 32-value group g of a row with
// x[t], for t < nt (NT tokens at most). Arithmetic: the block's small integers q_j (plus a per-format bias) become
// exact floats with one byte permute (2^23 + q as float bits) and one packed add of -(2^23 + bias); products with x
// are accumulated by packed fp32 FMAs (__ffma2_rn) in four chains per 16-value half; each half sum is scaled by the
// sub-block's dequantisation scale and offset once: a * sum_j q_j x_j + b * sum_j x_j (x sums precomputed when x is
// staged). This equals the dot product with the exactly dequantised fp32 weights up to fp32 rounding of the same
// order as the reference's own GEMV (flashnext/test_fn_quants.py:36-37 bounds it at 1e-5, the north star at 2e-7;
// the GPU suite checks 2e-7). The result per group is one fp32 value; callers accumulate groups in double.
#pragma once

#include "fn_decode.cuh"

namespace fn {

// ---- plane specifications -------------------------------------------------------------------------------------
struct Field {
    int off, size;  // offset inside the GGUF block, bytes
};
template <uint32_t TY> struct PlaneSpec {
    static constexpr int nf = 0;  // 0: no plane layout (the generic decoder reads GGUF rows)
    static constexpr Field f[1] = {{0, 0}};
};
#define FN_PLANES(TY, ...)                                                   \
    template <> struct PlaneSpec<TY> {                                       \
        static constexpr Field f[] = {__VA_ARGS__};                          \
        static constexpr int nf = sizeof(f) / sizeof(Field);                 \
    };
FN_PLANES(T_Q4_0, {2, 16}, {0, 2})
FN_PLANES(T_Q4_1, {4, 16}, {0, 4})
FN_PLANES(T_Q5_0, {6, 16}, {2, 4}, {0, 2})
FN_PLANES(T_Q5_1, {8, 16}, {4, 4}, {0, 4})
FN_PLANES(T_Q8_0, {2, 32}, {0, 2})
FN_PLANES(T_Q2_K, {16, 64}, {0, 16}, {80, 4})
FN_PLANES(T_Q3_K, {32, 64}, {0, 32}, {96, 12}, {108, 2})
FN_PLANES(T_Q4_K, {16, 128}, {4, 12}, {0, 4})
FN_PLANES(T_Q5_K, {48, 128}, {16, 32}, {4, 12}, {0, 4})
FN_PLANES(T_Q6_K, {0, 128}, {128, 64}, {192, 16}, {208, 2})
FN_PLANES(T_IQ2_XXS, {2, 64}, {0, 2})
FN_PLANES(T_IQ3_XXS, {2, 64}, {66, 32}, {0, 2})
FN_PLANES(T_IQ4_XS, {8, 128}, {4, 4}, {0, 4})
FN_PLANES(T_IQ4_NL, {2, 16}, {0, 2})
#undef FN_PLANES

// bytes of one block's fields before field F; the byte offset of plane F of a row of nb blocks is that times nb
template <uint32_t TY, int F> __host__ __device__ constexpr int plane_prefix() {
    int o = 0;
    for (int i = 0; i < F; ++i) o += PlaneSpec<TY>::f[i].size;
    return o;
}
template <uint32_t TY, int F> __device__ __forceinline__ int plane_off(int nb) {
    constexpr int P = plane_prefix<TY, F>();
    return P * nb;
}

// ---- packed helpers --------------------------------------------------------------------------------------------
// bytes k, k+1 of w as the floats 2^23 + byte
__device__ __forceinline__ float2 mag2(uint32_t w, int k) {
    return make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u + k)),
                       __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441u + k)));
}
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float hsum2(float2 a, float2 b) { return __fadd_rn(__fadd_rn(a.x, a.y), __fadd_rn(b.x, b.y)); }

// x accessors: a lane's x for group g, token t; pairs x[j], x[j+1] (j even) and the half sums (values 0-15, 16-31)
// x2: pairs x[j], x[j+1] (j even), scaled by 2^K_t for the formats that convert bytes as denormals (Denorm<TY>);
// xs: half sums of the unscaled x; inv: 2^(149 - K_t), which turns a sum of denormal products back to q . x
struct XRegA {  // one token, x of the group in registers
    const float2 (&x)[16];
    const float (&s)[2];
    float iv;
    __device__ __forceinline__ float2 x2(int, int j) const { return x[j >> 1]; }
    __device__ __forceinline__ float xs(int, int h) const { return s[h]; }
    __device__ __forceinline__ float inv(int) const { return iv; }
};
struct XSmA {  // tokens in shared memory: token t of the group at base + t * ts (32 values, 2 half sums, inv)
    const float *base;
    int ts;
    __device__ __forceinline__ float2 x2(int t, int j) const { return *(const float2 *)(base + (size_t)t * ts + j); }
    __device__ __forceinline__ float xs(int t, int h) const { return base[(size_t)t * ts + 32 + h]; }
    __device__ __forceinline__ float inv(int t) const { return base[(size_t)t * ts + 34]; }
};

// four biased bytes q4 (value_k = byte_k - bias) times x[j + k]: chains a[t][0] (j, j+1) and a[t][1] (j+2, j+3)
template <int NT, class XA>
__device__ __forceinline__ void acc_word(uint32_t q4, float2 moff, const XA &xa, int j, int nt, float2 (&a)[NT][2]) {
    const float2 v01 = __fadd2_rn(mag2(q4, 0), moff), v23 = __fadd2_rn(mag2(q4, 2), moff);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if (NT > 1 && t >= nt) break;
        a[t][0] = __ffma2_rn(v01, xa.x2(t, j), a[t][0]);
        a[t][1] = __ffma2_rn(v23, xa.x2(t, j + 2), a[t][1]);
    }
}

// four unsigned bytes q4 as the exact denormals q * 2^-149 (no conversion instruction beyond the byte permute), times
// the scaled x (x * 2^K): the products q x 2^(K - 149) are formed exactly by the FMA, in the normal range for the K
// the staging chose; chains as acc_word
template <int NT, class XA>
__device__ __forceinline__ void acc_word_dn(uint32_t q4, const XA &xa, int j, int nt, float2 (&a)[NT][2]) {
    const float2 v01 = make_float2(__uint_as_float(__byte_perm(q4, 0, 0x4440u)), __uint_as_float(__byte_perm(q4, 0, 0x4441u)));
    const float2 v23 = make_float2(__uint_as_float(__byte_perm(q4, 0, 0x4442u)), __uint_as_float(__byte_perm(q4, 0, 0x4443u)));
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if (NT > 1 && t >= nt) break;
        a[t][0] = __ffma2_rn(v01, xa.x2(t, j), a[t][0]);
        a[t][1] = __ffma2_rn(v23, xa.x2(t, j + 2), a[t][1]);
    }
}

template <int NT> __device__ __forceinline__ void zero2(float2 (&a)[NT][2]) {
#pragma unroll
    for (int t = 0; t < NT; ++t) a[t][0] = a[t][1] = make_float2(0.f, 0.f);
}

__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *(const uint4 *)p; }
__device__ __forceinline__ uint2 lds64(const uint8_t *p) { return *(const uint2 *)p; }

// grid bytes g (< 128) with signs m (per byte 0xFF: negative) -> bytes 128 + (+-g)
__device__ __forceinline__ uint32_t signed_bias128(uint32_t g, uint32_t m) {
    return (g ^ (m & 0x7F7F7F7Fu)) + (0x80808080u ^ (m & 0x81818181u));
}

// IQ4_NL values + 128 as bytes, four per word
constexpr uint32_t KVB0 = 0x3F2D1801u, KVB1 = 0x766A5D4Fu, KVB2 = 0xA6998D81u, KVB3 = 0xF1D9C5B5u;
// the 8 nibbles of w (byte i: low nibble = value i, high nibble = value 16 + i) looked up: lo = bytes of values
// 0..3, hi = values 16..19 (relative to w's first byte)
__device__ __forceinline__ void iq4_lut(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const uint32_t idx = w & 0x77777777u, sel = 0x32103210u | ((w & 0x88888888u) >> 1);
    const uint32_t a0 = __byte_perm(KVB0, KVB1, idx), b0 = __byte_perm(KVB2, KVB3, idx);
    const uint32_t a1 = __byte_perm(KVB0, KVB1, idx >> 16), b1 = __byte_perm(KVB2, KVB3, idx >> 16);
    const uint32_t t0 = __byte_perm(a0, b0, sel), t1 = __byte_perm(a1, b1, sel >> 16);  // v0 v16 v1 v17 | v2 v18 v3 v19
    lo = __byte_perm(t0, t1, 0x6420);
    hi = __byte_perm(t0, t1, 0x7531);
}

constexpr float MAG = 8388608.0f;

template <uint32_t TY> struct Fast {
    static constexpr bool ok = false;
};
// formats whose quant planes are re-encoded at upload (Encoded) and whose bytes become denormals (Denorm)
template <uint32_t TY> struct Encoded {
    static constexpr bool v = TY == T_Q4_K || TY == T_Q5_K || TY == T_Q6_K;
};
template <uint32_t TY> struct Denorm {
    static constexpr bool v = TY == T_Q4_K || TY == T_Q5_K;
};

// ---- 32-value formats ------------------------------------------------------------------------------------------
template <> struct Fast<T_Q4_0> {
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const uint4 w = lds128(row + 16 * g);
        const float d = f16_at(row + plane_off<T_Q4_0, 1>(nb) + 2 * g);
        const float2 mo = f2(-(MAG + 8.0f));
        float2 a[NT][2], b[NT][2];
        zero2<NT>(a);
        zero2<NT>(b);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc_word<NT>(ws[k] & 0x0F0F0F0Fu, mo, xa, 4 * k, nt, a);
            acc_word<NT>((ws[k] >> 4) & 0x0F0F0F0Fu, mo, xa, 16 + 4 * k, nt, b);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) if (NT == 1 || t < nt) r[t] = __fmul_rn(d, __fadd_rn(hsum2(a[t][0], a[t][1]), hsum2(b[t][0], b[t][1])));
    }
};

template <> struct Fast<T_IQ4_NL> {
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const uint4 w = lds128(row + 16 * g);
        const float d = f16_at(row + plane_off<T_IQ4_NL, 1>(nb) + 2 * g);
        const float2 mo = f2(-(MAG + 128.0f));
        float2 a[NT][2], b[NT][2];
        zero2<NT>(a);
        zero2<NT>(b);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t lo, hi;
            iq4_lut(ws[k], lo, hi);
            acc_word<NT>(lo, mo, xa, 4 * k, nt, a);
            acc_word<NT>(hi, mo, xa, 16 + 4 * k, nt, b);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) if (NT == 1 || t < nt) r[t] = __fmul_rn(d, __fadd_rn(hsum2(a[t][0], a[t][1]), hsum2(b[t][0], b[t][1])));
    }
};

template <> struct Fast<T_Q4_1> {
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const uint4 w = lds128(row + 16 * g);
        const uint32_t dm = u32_at(row + plane_off<T_Q4_1, 1>(nb) + 4 * g);
        const float d = f16_of(dm, 0), m = f16_of(dm, 1);
        const float2 mo = f2(-MAG);
        float2 a[NT][2], b[NT][2];
        zero2<NT>(a);
        zero2<NT>(b);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc_word<NT>(ws[k] & 0x0F0F0F0Fu, mo, xa, 4 * k, nt, a);
            acc_word<NT>((ws[k] >> 4) & 0x0F0F0F0Fu, mo, xa, 16 + 4 * k, nt, b);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (NT > 1 && t >= nt) break;
            const float s = __fadd_rn(hsum2(a[t][0], a[t][1]), hsum2(b[t][0], b[t][1]));
            r[t] = __fmaf_rn(d, s, __fmul_rn(m, __fadd_rn(xa.xs(t, 0), xa.xs(t, 1))));
        }
    }
};

// the 4 qh bits n (values i..i+3) as bit 4 of each byte
__device__ __forceinline__ uint32_t spread4_b4(uint32_t n) { return (n * 0x02040810u) & 0x10101010u; }

template <> struct Fast<T_Q5_0> {
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const uint4 w = lds128(row + 16 * g);
        const uint32_t qh = u32_at(row + plane_off<T_Q5_0, 1>(nb) + 4 * g);
        const float d = f16_at(row + plane_off<T_Q5_0, 2>(nb) + 2 * g);
        const float2 mo = f2(-(MAG + 16.0f));
        float2 a[NT][2], b[NT][2];
        zero2<NT>(a);
        zero2<NT>(b);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc_word<NT>((ws[k] & 0x0F0F0F0Fu) | spread4_b4((qh >> (4 * k)) & 15u), mo, xa, 4 * k, nt, a);
            acc_word<NT>(((ws[k] >> 4) & 0x0F0F0F0Fu) | spread4_b4((qh >> (16 + 4 * k)) & 15u), mo, xa, 16 + 4 * k, nt, b);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) if (NT == 1 || t < nt) r[t] = __fmul_rn(d, __fadd_rn(hsum2(a[t][0], a[t][1]), hsum2(b[t][0], b[t][1])));
    }
};

template <> struct Fast<T_Q5_1> {
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const uint4 w = lds128(row + 16 * g);
        const uint32_t qh = u32_at(row + plane_off<T_Q5_1, 1>(nb) + 4 * g);
        const uint32_t dm = u32_at(row + plane_off<T_Q5_1, 2>(nb) + 4 * g);
        const float d = f16_of(dm, 0), m = f16_of(dm, 1);
        const float2 mo = f2(-MAG);
        float2 a[NT][2], b[NT][2];
        zero2<NT>(a);
        zero2<NT>(b);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc_word<NT>((ws[k] & 0x0F0F0F0Fu) | spread4_b4((qh >> (4 * k)) & 15u), mo, xa, 4 * k, nt, a);
            acc_word<NT>(((ws[k] >> 4) & 0x0F0F0F0Fu) | spread4_b4((qh >> (16 + 4 * k)) & 15u), mo, xa, 16 + 4 * k, nt, b);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (NT > 1 && t >= nt) break;
            const float s = __fadd_rn(hsum2(a[t][0], a[t][1]), hsum2(b[t][0], b[t][1]));
            r[t] = __fmaf_rn(d, s, __fmul_rn(m, __fadd_rn(xa.xs(t, 0), xa.xs(t, 1))));
        }
    }
};

template <> struct Fast<T_Q8_0> {
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const uint4 w0 = lds128(row + 32 * g), w1 = lds128(row + 32 * g + 16);
        const float d = f16_at(row + plane_off<T_Q8_0, 1>(nb) + 2 * g);
        const float2 mo = f2(-(MAG + 128.0f));
        float2 a[NT][2], b[NT][2];
        zero2<NT>(a);
        zero2<NT>(b);
        const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc_word<NT>(ws[k] ^ 0x80808080u, mo, xa, 4 * k, nt, a);
            acc_word<NT>(ws[4 + k] ^ 0x80808080u, mo, xa, 16 + 4 * k, nt, b);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) if (NT == 1 || t < nt) r[t] = __fmul_rn(d, __fadd_rn(hsum2(a[t][0], a[t][1]), hsum2(b[t][0], b[t][1])));
    }
};

// ---- K-quants (256-value blocks; group g = block g >> 3, sub-block g & 7) --------------------------------------
template <> struct Fast<T_Q2_K> {
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const int b = g >> 3, ib = g & 7, h = ib >> 2, s = 2 * (ib & 3);
        const uint8_t *q = row + 64 * b + 32 * h;
        const uint4 w0 = lds128(q), w1 = lds128(q + 16);
        const uint32_t sc = u16_at(row + plane_off<T_Q2_K, 1>(nb) + 16 * b + 2 * ib);
        const uint32_t dm = u32_at(row + plane_off<T_Q2_K, 2>(nb) + 4 * b);
        const float d = f16_of(dm, 0), dmin = f16_of(dm, 1);
        const float dl0 = __fmul_rn(d, __uint2float_rn(sc & 15u)), ml0 = __fmul_rn(dmin, __uint2float_rn((sc >> 4) & 15u));
        const float dl1 = __fmul_rn(d, __uint2float_rn((sc >> 8) & 15u)), ml1 = __fmul_rn(dmin, __uint2float_rn((sc >> 12) & 15u));
        const float2 mo = f2(-MAG);
        float2 a[NT][2], c[NT][2];
        zero2<NT>(a);
        zero2<NT>(c);
        const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc_word<NT>((ws[k] >> s) & 0x03030303u, mo, xa, 4 * k, nt, a);
            acc_word<NT>((ws[4 + k] >> s) & 0x03030303u, mo, xa, 16 + 4 * k, nt, c);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (NT > 1 && t >= nt) break;
            const float h0 = __fmaf_rn(dl0, hsum2(a[t][0], a[t][1]), -__fmul_rn(ml0, xa.xs(t, 0)));
            const float h1 = __fmaf_rn(dl1, hsum2(c[t][0], c[t][1]), -__fmul_rn(ml1, xa.xs(t, 1)));
            r[t] = __fadd_rn(h0, h1);
        }
    }
};

template <> struct Fast<T_Q3_K> {
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const int b = g >> 3, ib = g & 7, h = ib >> 2, s = 2 * (ib & 3);
        const uint8_t *q = row + 64 * b + 32 * h, *hm = row + plane_off<T_Q3_K, 1>(nb) + 32 * b;
        const uint4 w0 = lds128(q), w1 = lds128(q + 16), m0 = lds128(hm), m1 = lds128(hm + 16);
        const uint8_t *scp = row + plane_off<T_Q3_K, 2>(nb) + 12 * b;
        const float d = f16_at(row + plane_off<T_Q3_K, 3>(nb) + 2 * b);
        float dl[2];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int k = 2 * ib + half;
            const uint32_t lo = (scp[k & 7] >> (4 * (k >> 3))) & 15u, hi = (scp[8 + (k & 3)] >> (2 * (k >> 2))) & 3u;
            dl[half] = __fmul_rn(d, __int2float_rn((int)(lo | (hi << 4)) - 32));
        }
        const float2 mo = f2(-(MAG + 4.0f));  // q = low 2 bits + 4 * hmask bit, minus 4
        float2 a[NT][2], c[NT][2];
        zero2<NT>(a);
        zero2<NT>(c);
        const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const uint32_t ms[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc_word<NT>(((ws[k] >> s) & 0x03030303u) | (((ms[k] >> ib) & 0x01010101u) << 2), mo, xa, 4 * k, nt, a);
            acc_word<NT>(((ws[4 + k] >> s) & 0x03030303u) | (((ms[4 + k] >> ib) & 0x01010101u) << 2), mo, xa, 16 + 4 * k,
                         nt, c);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) if (NT == 1 || t < nt) r[t] = __fmaf_rn(dl[1], hsum2(c[t][0], c[t][1]), __fmul_rn(dl[0], hsum2(a[t][0], a[t][1])));
    }
};

template <> struct Fast<T_Q4_K> {
    // encoded quant plane: 16 bytes per 32-value group, byte i = q[i] | q[16 + i] << 4 (encode_block<T_Q4_K>)
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const int b = g >> 3, ib = g & 7;
        const uint4 w = lds128(row + 16 * g);
        uint32_t sc, m;
        kq_scale_min(ib, row + plane_off<T_Q4_K, 1>(nb) + 12 * b, sc, m);
        const uint32_t dm = u32_at(row + plane_off<T_Q4_K, 2>(nb) + 4 * b);
        const float dl = __fmul_rn(f16_of(dm, 0), __uint2float_rn(sc)), ml = __fmul_rn(f16_of(dm, 1), __uint2float_rn(m));
        float2 a[NT][2], c[NT][2];
        zero2<NT>(a);
        zero2<NT>(c);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc_word_dn<NT>(ws[k] & 0x0F0F0F0Fu, xa, 4 * k, nt, a);
            acc_word_dn<NT>((ws[k] >> 4) & 0x0F0F0F0Fu, xa, 16 + 4 * k, nt, c);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (NT > 1 && t >= nt) break;
            const float sq = __fmul_rn(__fadd_rn(hsum2(a[t][0], a[t][1]), hsum2(c[t][0], c[t][1])), xa.inv(t));
            r[t] = __fmaf_rn(dl, sq, -__fmul_rn(ml, __fadd_rn(xa.xs(t, 0), xa.xs(t, 1))));
        }
    }
};

template <> struct Fast<T_Q5_K> {
    // encoded planes: 16 bytes of low nibbles per group as Q4_K, and a 4-byte word per group whose byte i bit m is
    // bit 4 of q[4m + i] (encode_block<T_Q5_K>)
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const int b = g >> 3, ib = g & 7;
        const uint4 w = lds128(row + 16 * g);
        const uint32_t H = u32_at(row + plane_off<T_Q5_K, 1>(nb) + 4 * g);
        uint32_t sc, m;
        kq_scale_min(ib, row + plane_off<T_Q5_K, 2>(nb) + 12 * b, sc, m);
        const uint32_t dm = u32_at(row + plane_off<T_Q5_K, 3>(nb) + 4 * b);
        const float dl = __fmul_rn(f16_of(dm, 0), __uint2float_rn(sc)), ml = __fmul_rn(f16_of(dm, 1), __uint2float_rn(m));
        float2 a[NT][2], c[NT][2];
        zero2<NT>(a);
        zero2<NT>(c);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t tl = (H << (4 - k)) & 0x10101010u, th = (k < 4 ? (H >> k) : 0u) & 0x10101010u;
            acc_word_dn<NT>((ws[k] & 0x0F0F0F0Fu) | tl, xa, 4 * k, nt, a);
            acc_word_dn<NT>(((ws[k] >> 4) & 0x0F0F0F0Fu) | th, xa, 16 + 4 * k, nt, c);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (NT > 1 && t >= nt) break;
            const float sq = __fmul_rn(__fadd_rn(hsum2(a[t][0], a[t][1]), hsum2(c[t][0], c[t][1])), xa.inv(t));
            r[t] = __fmaf_rn(dl, sq, -__fmul_rn(ml, __fadd_rn(xa.xs(t, 0), xa.xs(t, 1))));
        }
    }
};

template <> struct Fast<T_Q6_K> {
    // encoded planes: 16 bytes of low nibbles per group (byte i = lo[i] | lo[16 + i] << 4), and 8 bytes of the 2-bit
    // highs per group: word A byte i bits 2m..2m+1 = hi[4m + i], word B the same for values 16.. (encode_block<T_Q6_K>)
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const int b = g >> 3, j8 = g & 7;
        const uint4 w = lds128(row + 16 * g);
        const uint2 hb = lds64(row + plane_off<T_Q6_K, 1>(nb) + 8 * g);
        const uint32_t sc = u16_at(row + plane_off<T_Q6_K, 2>(nb) + 16 * b + 2 * j8);
        const float d = f16_at(row + plane_off<T_Q6_K, 3>(nb) + 2 * b);
        const float ds0 = __fmul_rn(d, (float)(int8_t)(sc & 255u)), ds1 = __fmul_rn(d, (float)(int8_t)(sc >> 8));
        const float2 mo = f2(-(MAG + 32.0f));
        float2 a[NT][2], c[NT][2];
        zero2<NT>(a);
        zero2<NT>(c);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            // bits 2k..2k+1 of every byte moved to bits 4..5
            const uint32_t ta = (k < 2 ? (hb.x << (4 - 2 * k)) : (hb.x >> (2 * k - 4))) & 0x30303030u;
            const uint32_t tb = (k < 2 ? (hb.y << (4 - 2 * k)) : (hb.y >> (2 * k - 4))) & 0x30303030u;
            acc_word<NT>((ws[k] & 0x0F0F0F0Fu) | ta, mo, xa, 4 * k, nt, a);
            acc_word<NT>(((ws[k] >> 4) & 0x0F0F0F0Fu) | tb, mo, xa, 16 + 4 * k, nt, c);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t)
            if (NT == 1 || t < nt) r[t] = __fmaf_rn(ds1, hsum2(c[t][0], c[t][1]), __fmul_rn(ds0, hsum2(a[t][0], a[t][1])));
    }
};

// ---- IQ formats --------------------------------------------------------------------------------------------------
template <> struct Fast<T_IQ4_XS> {
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *, const XA &xa, int nt,
                                                 float (&r)[NT]) {
        const int b = g >> 3, ib = g & 7;
        const uint4 w = lds128(row + 128 * b + 16 * ib);
        const uint32_t sl = u32_at(row + plane_off<T_IQ4_XS, 1>(nb) + 4 * b);
        const uint32_t dsh = u32_at(row + plane_off<T_IQ4_XS, 2>(nb) + 4 * b);  // d | scales_h << 16
        const uint32_t ls = ((sl >> (4 * ib)) & 15u) | (((dsh >> (16 + 2 * ib)) & 3u) << 4);
        const float dl = __fmul_rn(f16_of(dsh, 0), __int2float_rn((int)ls - 32));
        const float2 mo = f2(-(MAG + 128.0f));
        float2 a[NT][2], c[NT][2];
        zero2<NT>(a);
        zero2<NT>(c);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t lo, hi;
            iq4_lut(ws[k], lo, hi);
            acc_word<NT>(lo, mo, xa, 4 * k, nt, a);
            acc_word<NT>(hi, mo, xa, 16 + 4 * k, nt, c);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) if (NT == 1 || t < nt) r[t] = __fmul_rn(dl, __fadd_rn(hsum2(a[t][0], a[t][1]), hsum2(c[t][0], c[t][1])));
    }
};

template <> struct Fast<T_IQ2_XXS> {
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *grid, const XA &xa,
                                                 int nt, float (&r)[NT]) {
        const int b = g >> 3, ib = g & 7;
        const uint2 w = lds64(row + 64 * b + 8 * ib);
        const float d = f16_at(row + plane_off<T_IQ2_XXS, 1>(nb) + 2 * b);
        const float db = iq_scale(d, w.y >> 28, 0.25f);
        const float2 mo = f2(-(MAG + 128.0f));
        float2 a[NT][2], c[NT][2];
        zero2<NT>(a);
        zero2<NT>(c);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint2 gw = *(const uint2 *)(grid + 2 * ((w.x >> (8 * l)) & 255u));
            const uint32_t s8 = even_signs((w.y >> (7 * l)) & 127u);
            if (l < 2) {
                acc_word<NT>(signed_bias128(gw.x, sign_mask4(s8 & 15u)), mo, xa, 8 * l, nt, a);
                acc_word<NT>(signed_bias128(gw.y, sign_mask4(s8 >> 4)), mo, xa, 8 * l + 4, nt, a);
            } else {
                acc_word<NT>(signed_bias128(gw.x, sign_mask4(s8 & 15u)), mo, xa, 8 * l, nt, c);
                acc_word<NT>(signed_bias128(gw.y, sign_mask4(s8 >> 4)), mo, xa, 8 * l + 4, nt, c);
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) if (NT == 1 || t < nt) r[t] = __fmul_rn(db, __fadd_rn(hsum2(a[t][0], a[t][1]), hsum2(c[t][0], c[t][1])));
    }
};

// four signed values as bf16 pairs (t.x: values 0, 1; t.y: values 2, 3) times x[j + k]: chains as acc_word
template <int NT, class XA>
__device__ __forceinline__ void acc_bf4(uint2 t, const XA &xa, int j, int nt, float2 (&a)[NT][2]) {
    const float2 v01 = make_float2(__uint_as_float(t.x << 16), __uint_as_float(t.x & 0xFFFF0000u));
    const float2 v23 = make_float2(__uint_as_float(t.y << 16), __uint_as_float(t.y & 0xFFFF0000u));
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) {
        if (NT > 1 && tt >= nt) break;
        a[tt][0] = __ffma2_rn(v01, xa.x2(tt, j), a[tt][0]);
        a[tt][1] = __ffma2_rn(v23, xa.x2(tt, j + 2), a[tt][1]);
    }
}

// IQ3_XXS: each codebook index and its 4 sign bits select one entry of the signed bf16 expansion staged after the
// codebook (stage_grid), so a lookup yields 4 signed values ready for the FMAs; the values and the sum order are the
// same as the byte path's (float(v) exactly), so results are unchanged
template <> struct Fast<T_IQ3_XXS> {
    static constexpr bool ok = true;
    template <int NT, class XA>
    __device__ __forceinline__ static void group(const uint8_t *row, int nb, int g, const uint32_t *grid, const XA &xa,
                                                 int nt, float (&r)[NT]) {
        const uint2 *tab = (const uint2 *)(grid + 256);
        const int b = g >> 3, ib = g & 7;
        const uint2 q = lds64(row + 64 * b + 8 * ib);
        const uint32_t aux = u32_at(row + plane_off<T_IQ3_XXS, 1>(nb) + 32 * b + 4 * ib);
        const float d = f16_at(row + plane_off<T_IQ3_XXS, 2>(nb) + 2 * b);
        const float db = iq_scale(d, aux >> 28, 0.5f);
        float2 a[NT][2], c[NT][2];
        zero2<NT>(a);
        zero2<NT>(c);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t qq = l < 2 ? q.x : q.y, s = 16 * (l & 1);
            const uint32_t code = (aux >> (7 * l)) & 127u;
            const uint32_t shi = even_signs(code) >> 4;  // signs 4..7: 3 bits and the parity
            const uint2 t0 = tab[(((qq >> s) & 255u) << 4) | (code & 15u)];
            const uint2 t1 = tab[(((qq >> (s + 8)) & 255u) << 4) | shi];
            if (l < 2) {
                acc_bf4<NT>(t0, xa, 8 * l, nt, a);
                acc_bf4<NT>(t1, xa, 8 * l + 4, nt, a);
            } else {
                acc_bf4<NT>(t0, xa, 8 * l, nt, c);
                acc_bf4<NT>(t1, xa, 8 * l + 4, nt, c);
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) if (NT == 1 || t < nt) r[t] = __fmul_rn(db, __fadd_rn(hsum2(a[t][0], a[t][1]), hsum2(c[t][0], c[t][1])));
    }
};

// ---- re-encoding of the quant planes at upload (a lossless reorder of the same bits; same byte count) -------------
// q values of one GGUF block (256), as the integers gguf-py decodes (quants.py Q4_K/Q5_K/Q6_K)
__device__ __forceinline__ int q4k_q(const uint8_t *blk, int n) {
    const int j = n >> 5, i = n & 31;
    return (blk[16 + 32 * (j >> 1) + i] >> (4 * (j & 1))) & 15;
}
__device__ __forceinline__ int q5k_q(const uint8_t *blk, int n) {
    const int j = n >> 5, i = n & 31;
    return ((blk[48 + 32 * (j >> 1) + i] >> (4 * (j & 1))) & 15) | (((blk[16 + i] >> j) & 1) << 4);
}
__device__ __forceinline__ int q6k_q(const uint8_t *blk, int n) {
    const int j = n >> 5, i = n & 31, h = j >> 2;
    const int lo = (blk[64 * h + 32 * (j & 1) + i] >> (4 * ((j >> 1) & 1))) & 15;
    const int hi = (blk[128 + 32 * h + i] >> (2 * (j & 3))) & 3;
    return lo | (hi << 4);
}
// write block b (GGUF bytes blk) of a row of nb blocks into the encoded planes of dst (the row start)
template <uint32_t TY> __device__ void encode_block(const uint8_t *blk, uint8_t *dst, int b, int nb) {
    if constexpr (TY == T_Q4_K || TY == T_Q5_K) {
        const int so = TY == T_Q4_K ? 128 * nb : 160 * nb, mo = so + 12 * nb;  // scale and d/dmin planes
        for (int g = 0; g < 8; ++g) {
            for (int i = 0; i < 16; ++i) {
                const int lo = TY == T_Q4_K ? q4k_q(blk, 32 * g + i) : q5k_q(blk, 32 * g + i);
                const int hi = TY == T_Q4_K ? q4k_q(blk, 32 * g + 16 + i) : q5k_q(blk, 32 * g + 16 + i);
                dst[128 * b + 16 * g + i] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
            }
            if constexpr (TY == T_Q5_K) {
                uint32_t H = 0;
                for (int m = 0; m < 8; ++m)
                    for (int i = 0; i < 4; ++i) H |= (uint32_t)((q5k_q(blk, 32 * g + 4 * m + i) >> 4) & 1) << (8 * i + m);
                for (int k = 0; k < 4; ++k) dst[128 * nb + 32 * b + 4 * g + k] = (uint8_t)(H >> (8 * k));
            }
        }
        for (int k = 0; k < 12; ++k) dst[so + 12 * b + k] = blk[4 + k];
        for (int k = 0; k < 4; ++k) dst[mo + 4 * b + k] = blk[k];
    } else if constexpr (TY == T_Q6_K) {
        for (int g = 0; g < 8; ++g) {
            uint32_t A = 0, B = 0;
            for (int i = 0; i < 16; ++i) {
                const int lo = q6k_q(blk, 32 * g + i), hi = q6k_q(blk, 32 * g + 16 + i);
                dst[128 * b + 16 * g + i] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
            }
            for (int m = 0; m < 4; ++m)
                for (int i = 0; i < 4; ++i) {
                    A |= (uint32_t)(q6k_q(blk, 32 * g + 4 * m + i) >> 4) << (8 * i + 2 * m);
                    B |= (uint32_t)(q6k_q(blk, 32 * g + 16 + 4 * m + i) >> 4) << (8 * i + 2 * m);
                }
            for (int k = 0; k < 4; ++k) {
                dst[128 * nb + 64 * b + 8 * g + k] = (uint8_t)(A >> (8 * k));
                dst[128 * nb + 64 * b + 8 * g + 4 + k] = (uint8_t)(B >> (8 * k));
            }
        }
        for (int k = 0; k < 16; ++k) dst[192 * nb + 16 * b + k] = blk[192 + k];
        for (int k = 0; k < 2; ++k) dst[208 * nb + 2 * b + k] = blk[208 + k];
    }
}

// ---- layout descriptor for the host (repack) ---------------------------------------------------------------------
struct PlaneDesc {
    int nf = 0;
    Field f[6];
};
template <uint32_t TY> inline PlaneDesc plane_desc() {
    PlaneDesc d;
    if constexpr (Fast<TY>::ok) {
        d.nf = PlaneSpec<TY>::nf;
        for (int i = 0; i < d.nf; ++i) d.f[i] = PlaneSpec<TY>::f[i];
    }
    return d;
}

}  // namespace fn
