// GGUF block decoding for the engine's generic paths: the row dequantiser, the embedding lookup, the tensor-core tile
// decoder and the CUDA-core GEMV of the formats without a plane layout. Written from gguf-py 0.19.0's block layouts
// and float32 arithmetic (gguf/quants.py:204-1377); Q2_0, which gguf-py lacks, from flashnext/ref_fn.py:46-52.
//
// One algebraic form covers every format but BF16. gguf-py computes each value of a 32-value group as
//     v = (A * q) + B        two float32 roundings, in this order
// with q a small signed integer (|q| <= 128: a quant, a quant minus its offset, an IQ4 table value or a signed
// codebook byte), A the float32 scale and B the float32 offset of the value's 16-value half (the K-quants' 16-value
// sub-blocks and IQ2_XS / IQ2_S's paired scales change them inside a group). Where gguf-py adds no offset B = -0.0f:
// v + (-0) == v for every float v, signed zeros included. Codebook signs go onto the integer, since
// fl(A * -g) == -fl(A * g) (round to nearest is symmetric). So a decoder is integer work only: Codes<TY>::make builds
// a Codes32 (the 32 codes as 8 words of 4 two's-complement bytes, built four at a time with byte-SIMD operations, and
// the two (A, B) pairs), and Codes32::quad turns codes into values with packed float2 operations. BF16 groups are bit
// copies (Bf16x32). load_group<TY> returns whichever applies; both give values j .. j + 3 through quad(j).
//
// Rows may sit in global or shared memory and start 16-byte aligned (every engine row and staged tile does); a block
// of a format whose size is only a multiple of 2 is read with 16-bit loads.
#pragma once

#include "fn_common.cuh"

namespace fn {

// ---- loads -------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t u16_at(const uint8_t *p) { return *(const uint16_t *)p; }
__device__ __forceinline__ uint32_t u32_at(const uint8_t *p) { return *(const uint32_t *)p; }  // 4-byte aligned
// 32 bits at a 2-byte-aligned address: two halves
__device__ __forceinline__ uint32_t u32_at2(const uint8_t *p) { return u16_at(p) | (u16_at(p + 2) << 16); }
// 32 bits at an address aligned to A bytes
template <int A> __device__ __forceinline__ uint32_t word_at(const uint8_t *p) {
    if constexpr (A >= 4) return u32_at(p);
    else return u32_at2(p);
}
__device__ __forceinline__ float f16_at(const uint8_t *p) {
    return __half2float(__ushort_as_half((unsigned short)u16_at(p)));
}
__device__ __forceinline__ float f16_of(uint32_t w, int hi) {  // half `hi` of a word holding two fp16
    return __half2float(__ushort_as_half((unsigned short)(hi ? (w >> 16) : (w & 0xFFFFu))));
}

// ---- byte-SIMD helpers -------------------------------------------------------------------------------------------
constexpr uint32_t LOW4 = 0x0F0F0F0Fu, LOW2 = 0x03030303u, BIT0 = 0x01010101u;

// bits 0..3 of n on bit 0 of bytes 0..3 (the four shifted copies of n occupy disjoint bits, so nothing carries)
__device__ __forceinline__ uint32_t spread4(uint32_t n) { return ((n & 15u) * 0x00204081u) & BIT0; }
// per-byte masks: byte k = 0xFF where bit k of n is set
__device__ __forceinline__ uint32_t sign_mask4(uint32_t n) { return spread4(n) * 0xFFu; }
// bytes of g negated where the mask byte is 0xFF: (g ^ 0xFF) - 0xFF == -g mod 256, per byte without carries
__device__ __forceinline__ uint32_t negate_where(uint32_t g, uint32_t m) { return __vsub4(g ^ m, m); }
// the four 2-bit fields of byte c on bytes 0..3, field k on byte k
__device__ __forceinline__ uint32_t pairs_of_byte(uint32_t c) { return (c | (c << 6) | (c << 12) | (c << 18)) & LOW2; }

// The IQ2_XXS / IQ3_XXS sign byte of a 7-bit index: bits 0..6 are the signs of values 0..6 and value 7's sign makes
// the count of negative values even (gguf-py IQ2_XXS.ksigns). Parity by the 16-entry nibble table 0x6996.
__device__ __forceinline__ uint32_t even_signs(uint32_t s7) {
    return s7 | (((0x6996u >> ((s7 ^ (s7 >> 4)) & 15u)) & 1u) << 7);
}

// IQ4_NL's 16 values (gguf-py IQ4_NL.kvalues) as two's-complement bytes, four per word, entry i in byte i % 4 of
// word i / 4
constexpr uint32_t iq4_word(int w) {
    constexpr int kv[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
    uint32_t r = 0;
    for (int k = 0; k < 4; ++k) r |= (uint32_t)(kv[4 * w + k] & 255) << (8 * k);
    return r;
}
// the 4 low nibbles of w's bytes looked up in the table, as 4 code bytes: two 8-entry byte permutes (entries 0..7
// and 8..15, selected by the nibbles' low 3 bits) and a per-byte choice by bit 3
__device__ __forceinline__ uint32_t iq4_codes(uint32_t w) {
    const uint32_t n7 = w & 0x07070707u, y = n7 | (n7 >> 4);
    const uint32_t sel = __byte_perm(y, 0u, 0x0020u);  // the four 3-bit indices as selector nibbles 0..3
    const uint32_t lo = __byte_perm(iq4_word(0), iq4_word(1), sel), hi = __byte_perm(iq4_word(2), iq4_word(3), sel);
    const uint32_t m = ((w >> 3) & BIT0) * 0xFFu;
    return lo ^ ((lo ^ hi) & m);
}

// K-quant 6-bit scale and min of sub-block s from the 12 packed bytes as words D = bytes 0-3, M = 4-7, X = 8-11
// (gguf-py Q4_K.get_scale_min): sub-blocks 0-3 take the low 6 bits of D / M, sub-blocks 4-7 the nibbles of X topped
// with the high 2 bits of D / M. All four of a half are built at once.
__device__ __forceinline__ void kq_scale_min(int s, uint32_t D, uint32_t M, uint32_t X, uint32_t &sc, uint32_t &mn) {
    const uint32_t scw = s < 4 ? D & 0x3F3F3F3Fu : (X & LOW4) | ((D >> 2) & 0x30303030u);
    const uint32_t mnw = s < 4 ? M & 0x3F3F3F3Fu : ((X >> 4) & LOW4) | ((M >> 2) & 0x30303030u);
    sc = (scw >> (8 * (s & 3))) & 255u;
    mn = (mnw >> (8 * (s & 3))) & 255u;
}
// the same from the 12 bytes at p (4-byte aligned)
__device__ __forceinline__ void kq_scale_min(int s, const uint8_t *p, uint32_t &sc, uint32_t &mn) {
    kq_scale_min(s, u32_at(p), u32_at(p + 4), u32_at(p + 8), sc, mn);
}

// gguf-py's IQ scale d * (0.5 + s) * f (f = 0.25 for IQ2, 0.5 for IQ3_XXS), each product rounded
__device__ __forceinline__ float iq_scale(float d, uint32_t s, float f) {
    return __fmul_rn(__fmul_rn(d, 0.5f + __uint2float_rn(s)), f);
}

// ---- the two group forms -----------------------------------------------------------------------------------------
struct Codes32 {
    float a[2], b[2];  // scale and offset of values 0-15 and 16-31
    uint32_t q[8];     // code 4i + k in byte k of q[i]
    // values j .. j + 3 (j a multiple of 4). A code c becomes a float through the bits of 2^23 + (c + 128), minus
    // 2^23 + 128, exactly; then one product and one sum, each rounded.
    __device__ __forceinline__ float4 quad(int j) const {
        const int h = j >> 4;
        const uint32_t u = q[j >> 2] ^ 0x80808080u;
        const float2 off = make_float2(-8388736.0f, -8388736.0f);
        float2 c01 = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u)),
                                 __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541u)));
        float2 c23 = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542u)),
                                 __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543u)));
        c01 = __fadd2_rn(c01, off);
        c23 = __fadd2_rn(c23, off);
        const float2 A = make_float2(a[h], a[h]), B = make_float2(b[h], b[h]);
        const float2 v01 = __fadd2_rn(__fmul2_rn(A, c01), B), v23 = __fadd2_rn(__fmul2_rn(A, c23), B);
        return make_float4(v01.x, v01.y, v23.x, v23.y);
    }
};

struct Bf16x32 {
    uint32_t w[16];  // values 2i, 2i + 1 in the low and high half of w[i]
    __device__ __forceinline__ float4 quad(int j) const {
        const uint32_t p = w[j >> 1], r = w[(j >> 1) + 1];
        return make_float4(__uint_as_float(p << 16), __uint_as_float(p & 0xFFFF0000u), __uint_as_float(r << 16),
                           __uint_as_float(r & 0xFFFF0000u));
    }
};

// scale-only group: both halves share A, no offset
__device__ __forceinline__ void set_scale(Codes32 &c, float a0, float a1) {
    c.a[0] = a0;
    c.a[1] = a1;
    c.b[0] = c.b[1] = -0.0f;
}

// ---- per-format facts: values per block, bytes per block, byte alignment of a block, codebook words ---------------
template <uint32_t TY> struct Gguf;
#define FN_GGUF(TY, QK, BYTES, ALIGN, GRIDW)                                                      \
    template <> struct Gguf<TY> {                                                                 \
        static constexpr int qk = QK, bytes = BYTES, align = ALIGN, gridw = GRIDW;                \
    };
FN_GGUF(T_Q4_0, 32, 18, 2, 0)
FN_GGUF(T_Q4_1, 32, 20, 4, 0)
FN_GGUF(T_Q5_0, 32, 22, 2, 0)
FN_GGUF(T_Q5_1, 32, 24, 4, 0)
FN_GGUF(T_Q8_0, 32, 34, 2, 0)
FN_GGUF(T_IQ4_NL, 32, 18, 2, 0)
FN_GGUF(T_Q2_0, 64, 18, 2, 0)
FN_GGUF(T_BF16, 1, 2, 16, 0)
FN_GGUF(T_Q2_K, 256, 84, 4, 0)
FN_GGUF(T_Q3_K, 256, 110, 2, 0)
FN_GGUF(T_Q4_K, 256, 144, 4, 0)
FN_GGUF(T_Q5_K, 256, 176, 4, 0)
FN_GGUF(T_Q6_K, 256, 210, 2, 0)
FN_GGUF(T_IQ2_XXS, 256, 66, 2, 512)
FN_GGUF(T_IQ2_XS, 256, 74, 2, 1024)
FN_GGUF(T_IQ2_S, 256, 82, 2, 2048)
FN_GGUF(T_IQ3_XXS, 256, 98, 2, 256)
FN_GGUF(T_IQ3_S, 256, 110, 2, 512)
FN_GGUF(T_IQ4_XS, 256, 136, 4, 0)
#undef FN_GGUF

// Codes<TY>::make(blk, s, grid, c): sub-group s of the block at blk (s = 0 for 32-value blocks, 0..1 for Q2_0, 0..7
// for 256-value blocks); grid: the format's codebook words (IQ formats), entry e of an 8-value codebook in words 2e,
// 2e + 1, of a 4-value codebook in word e, value k in byte k.
template <uint32_t TY> struct Codes;

// 32-value blocks: fp16 d, [fp16 m], [32-bit qh], 16 bytes of nibbles (byte i: value i low, value 16 + i high)
template <uint32_t TY> struct Nibble32 {
    static constexpr int A = Gguf<TY>::align;
    __device__ __forceinline__ static void make(const uint8_t *blk, int, const uint32_t *, Codes32 &c) {
        constexpr bool has_m = TY == T_Q4_1 || TY == T_Q5_1, has_h = TY == T_Q5_0 || TY == T_Q5_1;
        constexpr int qs = 2 + (has_m ? 2 : 0) + (has_h ? 4 : 0);
        const float d = f16_at(blk);
        c.a[0] = c.a[1] = d;
        c.b[0] = c.b[1] = has_m ? f16_at(blk + 2) : -0.0f;
        uint32_t qh = 0;
        if constexpr (has_h) qh = word_at<A>(blk + (has_m ? 4 : 2));
        // the offset gguf-py subtracts: 8 (Q4_0), 16 (Q5_0), none for the formats with a min
        constexpr uint32_t bias = TY == T_Q4_0 ? 0x08080808u : TY == T_Q5_0 ? 0x10101010u : 0u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w = word_at<A>(blk + qs + 4 * i);
            uint32_t lo = w & LOW4, hi = (w >> 4) & LOW4;
            if constexpr (has_h) {
                lo |= spread4(qh >> (4 * i)) << 4;
                hi |= spread4(qh >> (16 + 4 * i)) << 4;
            }
            c.q[i] = __vsub4(lo, bias);
            c.q[4 + i] = __vsub4(hi, bias);
        }
    }
};
template <> struct Codes<T_Q4_0> : Nibble32<T_Q4_0> {};
template <> struct Codes<T_Q4_1> : Nibble32<T_Q4_1> {};
template <> struct Codes<T_Q5_0> : Nibble32<T_Q5_0> {};
template <> struct Codes<T_Q5_1> : Nibble32<T_Q5_1> {};

// Q8_0: fp16 d, 32 int8 quants (gguf-py: x * d)
template <> struct Codes<T_Q8_0> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int, const uint32_t *, Codes32 &c) {
        const float d = f16_at(blk);
        set_scale(c, d, d);
#pragma unroll
        for (int i = 0; i < 8; ++i) c.q[i] = u32_at2(blk + 2 + 4 * i);
    }
};

// IQ4_NL: fp16 d, 16 bytes of nibbles indexing the non-linear table
template <> struct Codes<T_IQ4_NL> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int, const uint32_t *, Codes32 &c) {
        const float d = f16_at(blk);
        set_scale(c, d, d);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w = u32_at2(blk + 2 + 4 * i);
            c.q[i] = iq4_codes(w);
            c.q[4 + i] = iq4_codes(w >> 4);
        }
    }
};

// Q2_0 (64 values, 18 bytes): fp16 d, 16 bytes; value 4i + k of the block = ((byte i >> 2k) & 3) - 1, times d.
// Sub-group s holds bytes 8s .. 8s + 7.
template <> struct Codes<T_Q2_0> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int s, const uint32_t *, Codes32 &c) {
        const float d = f16_at(blk);
        set_scale(c, d, d);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t two = u16_at(blk + 2 + 8 * s + 2 * i);
            c.q[2 * i] = __vsub4(pairs_of_byte(two & 255u), BIT0);
            c.q[2 * i + 1] = __vsub4(pairs_of_byte(two >> 8), BIT0);
        }
    }
};

// Q2_K (84 bytes): scales[16] (low nibble: scale, high: min, one per 16 values), qs[64], fp16 d, fp16 dmin. Value
// n = 128 h + 32 k + l is bits 2k..2k+1 of qs[32 h + l]; v = (d * sc) * q - (dmin * mn).
template <> struct Codes<T_Q2_K> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int s, const uint32_t *, Codes32 &c) {
        const float d = f16_at(blk + 80), dmin = f16_at(blk + 82);
        const uint32_t sm = u16_at(blk + 2 * s);  // the two scale bytes of this group's halves
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t byte = (sm >> (8 * h)) & 255u;
            c.a[h] = __fmul_rn(d, __uint2float_rn(byte & 15u));
            c.b[h] = -__fmul_rn(dmin, __uint2float_rn(byte >> 4));
        }
        const uint8_t *qs = blk + 16 + 32 * (s >> 2);
        const int sh = 2 * (s & 3);
#pragma unroll
        for (int i = 0; i < 8; ++i) c.q[i] = (u32_at(qs + 4 * i) >> sh) & LOW2;
    }
};

// Q3_K (110 bytes): hmask[32], qs[64], scales[12], fp16 d. Value n = 32 s + l: low 2 bits as Q2_K, high bit =
// bit s of hmask[l], q = low + 4 high - 4. The 16 6-bit scales (minus 32): low nibble from byte j % 8 (high nibble for
// j >= 8), top 2 bits from byte 8 + j % 4 at bit 2 (j / 4).
template <> struct Codes<T_Q3_K> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int s, const uint32_t *, Codes32 &c) {
        const float d = f16_at(blk + 108);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = 2 * s + h;
            const uint32_t lo = (blk[96 + (j & 7)] >> (4 * (j >> 3))) & 15u;
            const uint32_t hi = (blk[104 + (j & 3)] >> (2 * (j >> 2))) & 3u;
            c.a[h] = __fmul_rn(d, __int2float_rn((int)(lo | (hi << 4)) - 32));
            c.b[h] = -0.0f;
        }
        const uint8_t *qs = blk + 32 + 32 * (s >> 2);
        const int sh = 2 * (s & 3);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t low = (u32_at2(qs + 4 * i) >> sh) & LOW2, high = (u32_at2(blk + 4 * i) >> s) & BIT0;
            c.q[i] = __vsub4(low | (high << 2), 0x04040404u);
        }
    }
};

// Q4_K (144 bytes) / Q5_K (176 bytes): fp16 d, fp16 dmin, 12 packed scale/min bytes, [qh[32]], qs[128]. Sub-block s
// takes nibble s % 2 of qs[32 (s / 2) + l] (Q5_K: plus bit s of qh[l] as bit 4); v = (d * sc) * q - (dmin * mn).
template <uint32_t TY> struct KQuant45 {
    __device__ __forceinline__ static void make(const uint8_t *blk, int s, const uint32_t *, Codes32 &c) {
        constexpr bool five = TY == T_Q5_K;
        const uint32_t dd = u32_at(blk);
        uint32_t sc, mn;
        kq_scale_min(s, blk + 4, sc, mn);
        const float a = __fmul_rn(f16_of(dd, 0), __uint2float_rn(sc)), b = -__fmul_rn(f16_of(dd, 1), __uint2float_rn(mn));
        c.a[0] = c.a[1] = a;
        c.b[0] = c.b[1] = b;
        const uint8_t *qs = blk + (five ? 48 : 16) + 32 * (s >> 1);
        const int sh = 4 * (s & 1);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint32_t q = (u32_at(qs + 4 * i) >> sh) & LOW4;
            if constexpr (five) q |= ((u32_at(blk + 16 + 4 * i) >> s) & BIT0) << 4;
            c.q[i] = q;
        }
    }
};
template <> struct Codes<T_Q4_K> : KQuant45<T_Q4_K> {};
template <> struct Codes<T_Q5_K> : KQuant45<T_Q5_K> {};

// Q6_K (210 bytes): ql[128], qh[64], int8 scales[16], fp16 d. Value n = 128 H + 32 s' + l (s' = s % 4, H = s / 4):
// low nibble = nibble (s' / 2) of ql[64 H + 32 (s' % 2) + l], high 2 bits = bits 2 s'..2 s' + 1 of qh[32 H + l],
// q = (low | high << 4) - 32; v = (d * scale[n / 16]) * q.
template <> struct Codes<T_Q6_K> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int s, const uint32_t *, Codes32 &c) {
        const float d = f16_at(blk + 208);
        const uint32_t sc = u16_at(blk + 192 + 2 * s);
        set_scale(c, __fmul_rn(d, (float)(int8_t)(sc & 255u)), __fmul_rn(d, (float)(int8_t)(sc >> 8)));
        const int H = s >> 2, sp = s & 3;
        const uint8_t *ql = blk + 64 * H + 32 * (sp & 1), *qh = blk + 128 + 32 * H;
        const int lsh = 4 * (sp >> 1), hsh = 2 * sp;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t low = (u32_at2(ql + 4 * i) >> lsh) & LOW4, high = (u32_at2(qh + 4 * i) >> hsh) & LOW2;
            c.q[i] = __vsub4(low | (high << 4), 0x20202020u);
        }
    }
};

// IQ4_XS (136 bytes): fp16 d, 16-bit scales_h, scales_l[4], qs[128]. Sub-block s: scale = (nibble s % 2 of
// scales_l[s / 2] | bits 2s..2s+1 of scales_h << 4) - 32; 16 bytes qs[16 s ..] as IQ4_NL's.
template <> struct Codes<T_IQ4_XS> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int s, const uint32_t *, Codes32 &c) {
        const uint32_t dh = u32_at(blk);  // d | scales_h << 16
        const uint32_t ls = ((blk[4 + (s >> 1)] >> (4 * (s & 1))) & 15u) | (((dh >> (16 + 2 * s)) & 3u) << 4);
        const float a = __fmul_rn(f16_of(dh, 0), __int2float_rn((int)ls - 32));
        set_scale(c, a, a);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w = u32_at(blk + 8 + 16 * s + 4 * i);
            c.q[i] = iq4_codes(w);
            c.q[4 + i] = iq4_codes(w >> 4);
        }
    }
};

// eight codebook values (the two words of an IQ2 entry) with 8 sign bits -> code words q[2e], q[2e + 1]
__device__ __forceinline__ void signed_pair(Codes32 &c, int e, uint2 gw, uint32_t s8) {
    c.q[2 * e] = negate_where(gw.x, sign_mask4(s8 & 15u));
    c.q[2 * e + 1] = negate_where(gw.y, sign_mask4(s8 >> 4));
}

// IQ2_XXS (66 bytes): fp16 d, then per sub-block two 32-bit words: the 4 codebook indices (bytes), and 4 x 7 sign
// bits (bits 7e..7e+6) with the 4-bit scale in bits 28-31; A = d (0.5 + scale) 0.25.
template <> struct Codes<T_IQ2_XXS> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int s, const uint32_t *grid, Codes32 &c) {
        const uint32_t idx = u32_at2(blk + 2 + 8 * s), aux = u32_at2(blk + 6 + 8 * s);
        const float a = iq_scale(f16_at(blk), aux >> 28, 0.25f);
        set_scale(c, a, a);
#pragma unroll
        for (int e = 0; e < 4; ++e)
            signed_pair(c, e, *(const uint2 *)(grid + 2 * ((idx >> (8 * e)) & 255u)), even_signs((aux >> (7 * e)) & 127u));
    }
};

// IQ2_XS (74 bytes): fp16 d, 32 16-bit entries (codebook index bits 0-8, 7 sign bits above), scales[8] (nibble h
// scales half h of sub-block s)
template <> struct Codes<T_IQ2_XS> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int s, const uint32_t *grid, Codes32 &c) {
        const float d = f16_at(blk);
        const uint32_t sb = blk[66 + s];
        set_scale(c, iq_scale(d, sb & 15u, 0.25f), iq_scale(d, sb >> 4, 0.25f));
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t v = u16_at(blk + 2 + 8 * s + 2 * e);
            signed_pair(c, e, *(const uint2 *)(grid + 2 * (v & 511u)), even_signs(v >> 9));
        }
    }
};

// IQ2_S (82 bytes): fp16 d, qs[32] (index low 8 bits), signs[32] (8 explicit sign bits per entry), qh[8] (2 index
// high bits per entry), scales[8] as IQ2_XS
template <> struct Codes<T_IQ2_S> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int s, const uint32_t *grid, Codes32 &c) {
        const float d = f16_at(blk);
        const uint32_t sb = blk[74 + s], qh = blk[66 + s];
        set_scale(c, iq_scale(d, sb & 15u, 0.25f), iq_scale(d, sb >> 4, 0.25f));
        const uint32_t lo8 = u32_at2(blk + 2 + 4 * s), sg = u32_at2(blk + 34 + 4 * s);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t ix = ((lo8 >> (8 * e)) & 255u) | (((qh >> (2 * e)) & 3u) << 8);
            signed_pair(c, e, *(const uint2 *)(grid + 2 * ix), (sg >> (8 * e)) & 255u);
        }
    }
};

// IQ3_XXS (98 bytes): fp16 d, qs[64] (one 4-value codebook index per byte, 8 per sub-block), then per sub-block a
// 32-bit word: 4 x 7 sign bits (one sign byte per 8 values) and the scale in bits 28-31; A = d (0.5 + scale) 0.5.
template <> struct Codes<T_IQ3_XXS> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int s, const uint32_t *grid, Codes32 &c) {
        const uint32_t i0 = u32_at2(blk + 2 + 8 * s), i1 = u32_at2(blk + 6 + 8 * s), aux = u32_at2(blk + 66 + 4 * s);
        const float a = iq_scale(f16_at(blk), aux >> 28, 0.5f);
        set_scale(c, a, a);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t ix = e < 2 ? i0 : i1, sh = 16 * (e & 1);
            const uint2 gw = make_uint2(grid[(ix >> sh) & 255u], grid[(ix >> (sh + 8)) & 255u]);
            signed_pair(c, e, gw, even_signs((aux >> (7 * e)) & 127u));
        }
    }
};

// IQ3_S (110 bytes): fp16 d, qs[64] (index low 8 bits), qh[8] (bit k of qh[s]: bit 8 of sub-block s's index k),
// signs[32] (explicit, one byte per 8 values), scales[4] (nibble s); A = d (1 + 2 scale)
template <> struct Codes<T_IQ3_S> {
    __device__ __forceinline__ static void make(const uint8_t *blk, int s, const uint32_t *grid, Codes32 &c) {
        const uint32_t scale = (blk[106 + (s >> 1)] >> (4 * (s & 1))) & 15u;
        const float a = __fmul_rn(f16_at(blk), __uint2float_rn(1u + 2u * scale));
        set_scale(c, a, a);
        const uint32_t i0 = u32_at2(blk + 2 + 8 * s), i1 = u32_at2(blk + 6 + 8 * s), qh = blk[66 + s];
        const uint32_t sg = u32_at2(blk + 74 + 4 * s);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t ix = e < 2 ? i0 : i1, sh = 16 * (e & 1);
            const uint32_t k0 = ((ix >> sh) & 255u) | (((qh >> (2 * e)) & 1u) << 8);
            const uint32_t k1 = ((ix >> (sh + 8)) & 255u) | (((qh >> (2 * e + 1)) & 1u) << 8);
            signed_pair(c, e, make_uint2(grid[k0], grid[k1]), (sg >> (8 * e)) & 255u);
        }
    }
};

// ---- the entry point -----------------------------------------------------------------------------------------------
// group g (32 values) of a row: sub-group g % (qk / 32) of block g / (qk / 32)
template <uint32_t TY> __device__ __forceinline__ auto load_group(const uint8_t *row, int g, const uint32_t *grid) {
    if constexpr (TY == T_BF16) {
        Bf16x32 v;
        const uint4 *p = (const uint4 *)(row + 64 * (size_t)g);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 u = p[i];
            v.w[4 * i] = u.x;
            v.w[4 * i + 1] = u.y;
            v.w[4 * i + 2] = u.z;
            v.w[4 * i + 3] = u.w;
        }
        return v;
    } else {
        constexpr int per = Gguf<TY>::qk / 32;
        Codes32 c;
        Codes<TY>::make(row + (size_t)(g / per) * Gguf<TY>::bytes, g % per, grid, c);
        return c;
    }
}

// run f(TY) for the runtime type id t; false if t has no decoder
template <class F> inline bool dispatch_type(uint32_t t, F &&f) {
    switch (t) {
        case T_Q4_0: f.template operator()<T_Q4_0>(); return true;
        case T_Q4_1: f.template operator()<T_Q4_1>(); return true;
        case T_Q5_0: f.template operator()<T_Q5_0>(); return true;
        case T_Q5_1: f.template operator()<T_Q5_1>(); return true;
        case T_Q8_0: f.template operator()<T_Q8_0>(); return true;
        case T_Q2_K: f.template operator()<T_Q2_K>(); return true;
        case T_Q3_K: f.template operator()<T_Q3_K>(); return true;
        case T_Q4_K: f.template operator()<T_Q4_K>(); return true;
        case T_Q5_K: f.template operator()<T_Q5_K>(); return true;
        case T_Q6_K: f.template operator()<T_Q6_K>(); return true;
        case T_IQ2_XXS: f.template operator()<T_IQ2_XXS>(); return true;
        case T_IQ2_XS: f.template operator()<T_IQ2_XS>(); return true;
        case T_IQ3_XXS: f.template operator()<T_IQ3_XXS>(); return true;
        case T_IQ4_NL: f.template operator()<T_IQ4_NL>(); return true;
        case T_IQ3_S: f.template operator()<T_IQ3_S>(); return true;
        case T_IQ2_S: f.template operator()<T_IQ2_S>(); return true;
        case T_IQ4_XS: f.template operator()<T_IQ4_XS>(); return true;
        case T_BF16: f.template operator()<T_BF16>(); return true;
        case T_Q2_0: f.template operator()<T_Q2_0>(); return true;
        default: return false;
    }
}

}  // namespace fn
