// GGUF block decoders. Dec<TY>::group(row, g, grid, f) decodes the g-th group of 32 values of a GGUF row and hands
// them to f(j, v[j], v[j+1], v[j+2], v[j+3]) in eight runs of four (j = 0, 4, ..., 28, in a format-chosen order).
// Every value is bit-identical to gguf-py 0.19.0 `quants.dequantize` (float32): each rounding step of gguf-py is one
// __fmul_rn / __fadd_rn / __fsub_rn here, so the compiler cannot contract two of them into an FMA. `row` may point
// to global or shared memory; it must be 16-byte aligned (every engine row is). Blocks of 2-byte-aligned formats
// are read with 16-bit loads only.
//
// The format semantics follow ggml's block layouts as gguf-py restates them (gguf/quants.py:220-1377) and the
// reference's decoders (engine/faie2fn.cu:343-688) for the 13 formats it carries.
#pragma once

#include "fn_common.cuh"

namespace fn {

__device__ __forceinline__ uint32_t ld8(const uint8_t *p) { return *p; }
__device__ __forceinline__ uint32_t ld16(const uint8_t *p) { return *(const uint16_t *)p; }
__device__ __forceinline__ uint32_t ld32u(const uint8_t *p) { return ld16(p) | (ld16(p + 2) << 16); }  // 2-aligned
__device__ __forceinline__ uint32_t ld32a(const uint8_t *p) { return *(const uint32_t *)p; }           // 4-aligned
__device__ __forceinline__ float ldh(const uint8_t *p) { return __half2float(__ushort_as_half((unsigned short)ld16(p))); }

// small non-negative integer u (< 2^22) as a float, exactly: 2^23 + u has u in its low mantissa bits
__device__ __forceinline__ float u2f(uint32_t u) { return __int_as_float(0x4B000000u | u) - 8388608.0f; }
// u - off as a float, exactly (u < 2^22, off small)
__device__ __forceinline__ float u2f_off(uint32_t u, float off) {
    return __int_as_float(0x4B000000u | u) - (8388608.0f + off);
}
// byte k of w, as a float
__device__ __forceinline__ float byte_f(uint32_t w, int k) { return u2f((w >> (8 * k)) & 255u); }
// value * (bit k of s ? -1 : 1): a sign-bit flip, exact
__device__ __forceinline__ float sflip(float v, uint32_t s, int k) {
    return __uint_as_float(__float_as_uint(v) ^ (((s >> k) & 1u) << 31));
}
// ggml ksigns_iq2xs[i]: the 7 sign bits i plus their parity as bit 7
__device__ __forceinline__ uint32_t ksign(uint32_t i) { return i | ((__popc(i) & 1u) << 7); }

// IQ4_NL values (-127 .. 113) + 128 as bytes, four per word: the lookup is a byte permute
constexpr uint32_t KV_W0 = 0x3F2D1801u, KV_W1 = 0x766A5D4Fu, KV_W2 = 0xA6998D81u, KV_W3 = 0xF1D9C5B5u;
__device__ __forceinline__ float iq4nl(uint32_t q) {  // q in 0..15
    const uint32_t lo = __byte_perm(KV_W0, KV_W1, q & 7), hi = __byte_perm(KV_W2, KV_W3, q & 7);
    const uint32_t b = ((q & 8) ? hi : lo) & 255u;
    return u2f_off(b, 128.0f);
}

// K-quant 6-bit scale and min of sub-block j from the 12 packed bytes at q (gguf-py Q4_K.get_scale_min)
__device__ __forceinline__ void kscale(int j, const uint8_t *q, uint32_t &sc, uint32_t &m) {
    if (j < 4) {
        sc = q[j] & 63u;
        m = q[j + 4] & 63u;
    } else {
        sc = (q[j + 4] & 15u) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

template <uint32_t TY> struct Dec;

template <> struct Dec<T_Q4_0> {
    static constexpr int qk = 32, bytes = 18, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + g * 18;
        const float d = ldh(b);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w = ld32u(b + 2 + 4 * k);
            auto lo = [&](int s) { return __fmul_rn(d, u2f_off((w >> (8 * s)) & 15u, 8.0f)); };
            auto hi = [&](int s) { return __fmul_rn(d, u2f_off((w >> (8 * s + 4)) & 15u, 8.0f)); };
            f(4 * k, lo(0), lo(1), lo(2), lo(3));
            f(16 + 4 * k, hi(0), hi(1), hi(2), hi(3));
        }
    }
};

template <> struct Dec<T_Q4_1> {
    static constexpr int qk = 32, bytes = 20, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + g * 20;
        const float d = ldh(b), m = ldh(b + 2);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w = ld32a(b + 4 + 4 * k);
            auto lo = [&](int s) { return __fadd_rn(__fmul_rn(d, u2f((w >> (8 * s)) & 15u)), m); };
            auto hi = [&](int s) { return __fadd_rn(__fmul_rn(d, u2f((w >> (8 * s + 4)) & 15u)), m); };
            f(4 * k, lo(0), lo(1), lo(2), lo(3));
            f(16 + 4 * k, hi(0), hi(1), hi(2), hi(3));
        }
    }
};

template <> struct Dec<T_Q5_0> {
    static constexpr int qk = 32, bytes = 22, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + g * 22;
        const float d = ldh(b);
        const uint32_t qh = ld32u(b + 2);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w = ld32u(b + 6 + 4 * k);
            auto lo = [&](int s) {
                const int i = 4 * k + s;
                return __fmul_rn(d, u2f_off(((w >> (8 * s)) & 15u) | (((qh >> i) & 1u) << 4), 16.0f));
            };
            auto hi = [&](int s) {
                const int i = 16 + 4 * k + s;
                return __fmul_rn(d, u2f_off(((w >> (8 * s + 4)) & 15u) | (((qh >> i) & 1u) << 4), 16.0f));
            };
            f(4 * k, lo(0), lo(1), lo(2), lo(3));
            f(16 + 4 * k, hi(0), hi(1), hi(2), hi(3));
        }
    }
};

template <> struct Dec<T_Q5_1> {
    static constexpr int qk = 32, bytes = 24, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + g * 24;
        const float d = ldh(b), m = ldh(b + 2);
        const uint32_t qh = ld32a(b + 4);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w = ld32a(b + 8 + 4 * k);
            auto lo = [&](int s) {
                const int i = 4 * k + s;
                return __fadd_rn(__fmul_rn(d, u2f(((w >> (8 * s)) & 15u) | (((qh >> i) & 1u) << 4))), m);
            };
            auto hi = [&](int s) {
                const int i = 16 + 4 * k + s;
                return __fadd_rn(__fmul_rn(d, u2f(((w >> (8 * s + 4)) & 15u) | (((qh >> i) & 1u) << 4))), m);
            };
            f(4 * k, lo(0), lo(1), lo(2), lo(3));
            f(16 + 4 * k, hi(0), hi(1), hi(2), hi(3));
        }
    }
};

template <> struct Dec<T_Q8_0> {
    static constexpr int qk = 32, bytes = 34, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + g * 34;
        const float d = ldh(b);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const uint32_t w = ld32u(b + 2 + j) ^ 0x80808080u;  // int8 + 128 as unsigned bytes
            auto v = [&](int s) { return __fmul_rn(u2f_off((w >> (8 * s)) & 255u, 128.0f), d); };
            f(j, v(0), v(1), v(2), v(3));
        }
    }
};

template <> struct Dec<T_IQ4_NL> {
    static constexpr int qk = 32, bytes = 18, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + g * 18;
        const float d = ldh(b);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w = ld32u(b + 2 + 4 * k);
            auto lo = [&](int s) { return __fmul_rn(d, iq4nl((w >> (8 * s)) & 15u)); };
            auto hi = [&](int s) { return __fmul_rn(d, iq4nl((w >> (8 * s + 4)) & 15u)); };
            f(4 * k, lo(0), lo(1), lo(2), lo(3));
            f(16 + 4 * k, hi(0), hi(1), hi(2), hi(3));
        }
    }
};

// Q2_0 (ggml type 42): 64 values per 18-byte block, value 4i + k = ((qs[i] >> 2k) & 3) - 1, times d
// (flashnext/ref_fn.py:46-52; engine/faie2fn.cu:468-481)
template <> struct Dec<T_Q2_0> {
    static constexpr int qk = 64, bytes = 18, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + (g >> 1) * 18;
        const float d = ldh(b);
        const uint8_t *qs = b + 2 + (g & 1) * 8;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w = ld16(qs + 2 * k);
            auto v = [&](int s) { return __fmul_rn(u2f_off((w >> (2 * s)) & 3u, 1.0f), d); };
            f(8 * k, v(0), v(1), v(2), v(3));
            f(8 * k + 4, v(4), v(5), v(6), v(7));
        }
    }
};

template <> struct Dec<T_BF16> {
    static constexpr int qk = 1, bytes = 2, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *p = row + g * 64;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const uint32_t a = ld32a(p + 2 * j), c = ld32a(p + 2 * j + 4);
            f(j, __uint_as_float(a << 16), __uint_as_float(a & 0xffff0000u), __uint_as_float(c << 16),
              __uint_as_float(c & 0xffff0000u));
        }
    }
};

// ---- K-quants -----------------------------------------------------------------------------------------------

template <> struct Dec<T_Q2_K> {
    static constexpr int qk = 256, bytes = 84, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + (g >> 3) * 84;
        const int ib = g & 7, h = ib >> 2, s = 2 * (ib & 3);
        const float d = ldh(b + 80), dmin = ldh(b + 82);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const uint32_t sc = b[2 * ib + half];
            const float dl = __fmul_rn(d, u2f(sc & 15u)), ml = __fmul_rn(dmin, u2f(sc >> 4));
#pragma unroll
            for (int j = 16 * half; j < 16 * half + 16; j += 4) {
                const uint32_t w = ld32a(b + 16 + 32 * h + j) >> s;
                auto v = [&](int k) { return __fsub_rn(__fmul_rn(dl, u2f((w >> (8 * k)) & 3u)), ml); };
                f(j, v(0), v(1), v(2), v(3));
            }
        }
    }
};

template <> struct Dec<T_Q3_K> {
    static constexpr int qk = 256, bytes = 110, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + (g >> 3) * 110;
        const int ib = g & 7, h = ib >> 2, s = 2 * (ib & 3);
        const float d = ldh(b + 108);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int k = 2 * ib + half;  // 16-value scale group
            const uint32_t lo = (b[96 + (k & 7)] >> (4 * (k >> 3))) & 15u;
            const uint32_t hi = (b[104 + (k & 3)] >> (2 * (k >> 2))) & 3u;
            const float dl = __fmul_rn(d, u2f_off(lo | (hi << 4), 32.0f));
#pragma unroll
            for (int j = 16 * half; j < 16 * half + 16; j += 4) {
                const uint32_t w = ld32u(b + 32 + 32 * h + j) >> s;
                const uint32_t m = ld32u(b + j) >> ib;
                // q = low 2 bits - 4 when the hmask bit is clear (gguf-py: "offset is zero when the bitmask is 1"),
                // i.e. (low + 4 * hbit) - 4
                auto v = [&](int t) {
                    const uint32_t qq = ((w >> (8 * t)) & 3u) + 4u * ((m >> (8 * t)) & 1u);
                    return __fmul_rn(dl, u2f_off(qq, 4.0f));
                };
                f(j, v(0), v(1), v(2), v(3));
            }
        }
    }
};

template <> struct Dec<T_Q4_K> {
    static constexpr int qk = 256, bytes = 144, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + (g >> 3) * 144;
        const int ib = g & 7;
        const float d = ldh(b), dmin = ldh(b + 2);
        uint32_t sc, m;
        kscale(ib, b + 4, sc, m);
        const float dl = __fmul_rn(d, u2f(sc)), ml = __fmul_rn(dmin, u2f(m));
        const uint8_t *q = b + 16 + 32 * (ib >> 1);
        const int sh = 4 * (ib & 1);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const uint32_t w = ld32a(q + j) >> sh;
            auto v = [&](int k) { return __fsub_rn(__fmul_rn(dl, u2f((w >> (8 * k)) & 15u)), ml); };
            f(j, v(0), v(1), v(2), v(3));
        }
    }
};

template <> struct Dec<T_Q5_K> {
    static constexpr int qk = 256, bytes = 176, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + (g >> 3) * 176;
        const int ib = g & 7;
        const float d = ldh(b), dmin = ldh(b + 2);
        uint32_t sc, m;
        kscale(ib, b + 4, sc, m);
        const float dl = __fmul_rn(d, u2f(sc)), ml = __fmul_rn(dmin, u2f(m));
        const uint8_t *q = b + 48 + 32 * (ib >> 1);
        const int sh = 4 * (ib & 1);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const uint32_t w = ld32a(q + j) >> sh, h = ld32a(b + 16 + j) >> ib;
            auto v = [&](int k) {
                return __fsub_rn(__fmul_rn(dl, u2f(((w >> (8 * k)) & 15u) | (((h >> (8 * k)) & 1u) << 4))), ml);
            };
            f(j, v(0), v(1), v(2), v(3));
        }
    }
};

template <> struct Dec<T_Q6_K> {
    static constexpr int qk = 256, bytes = 210, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + (g >> 3) * 210;
        const int j8 = g & 7, h = j8 >> 2;
        const uint8_t *ql = b + 64 * h + 32 * (j8 & 1);
        const uint8_t *qh = b + 128 + 32 * h;
        const int ls = 4 * ((j8 >> 1) & 1), hs = 2 * (j8 & 3);
        const float d = ldh(b + 208);
        const float ds0 = __fmul_rn(d, (float)(int8_t)b[192 + 2 * j8]);
        const float ds1 = __fmul_rn(d, (float)(int8_t)b[193 + 2 * j8]);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const uint32_t w = ld32u(ql + j) >> ls, hh = ld32u(qh + j) >> hs;
            const float ds = j < 16 ? ds0 : ds1;
            auto v = [&](int k) {
                return __fmul_rn(ds, u2f_off(((w >> (8 * k)) & 15u) | (((hh >> (8 * k)) & 3u) << 4), 32.0f));
            };
            f(j, v(0), v(1), v(2), v(3));
        }
    }
};

// ---- IQ codebook formats (grid = the codebook words, in shared or global memory) ---------------------------------

// 8 codebook bytes (words a, c) times db, signs bit k negating value k: runs j0 and j0 + 4
template <class F>
__device__ __forceinline__ void grid8(F &&f, int j0, uint32_t a, uint32_t c, float db, uint32_t signs) {
    auto v = [&](uint32_t w, int k, int sb) { return sflip(__fmul_rn(db, byte_f(w, k)), signs, sb); };
    f(j0, v(a, 0, 0), v(a, 1, 1), v(a, 2, 2), v(a, 3, 3));
    f(j0 + 4, v(c, 0, 4), v(c, 1, 5), v(c, 2, 6), v(c, 3, 7));
}

// d * (0.5 + s) * mult with gguf-py's two roundings (mult a power of two)
__device__ __forceinline__ float db_half(float d, uint32_t s, float mult) {
    return __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, u2f(s))), mult);
}

template <> struct Dec<T_IQ2_XXS> {
    static constexpr int qk = 256, bytes = 66, gridw = 512;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *grid, F &&f) {
        const uint8_t *b = row + (g >> 3) * 66;
        const int ib = g & 7;
        const float d = ldh(b);
        const uint32_t w0 = ld32u(b + 2 + 8 * ib), w1 = ld32u(b + 6 + 8 * ib);
        const float db = db_half(d, w1 >> 28, 0.25f);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t e = (w0 >> (8 * l)) & 255u;
            const uint2 gw = *(const uint2 *)(grid + 2 * e);
            grid8(f, 8 * l, gw.x, gw.y, db, ksign((w1 >> (7 * l)) & 127u));
        }
    }
};

template <> struct Dec<T_IQ2_XS> {
    static constexpr int qk = 256, bytes = 74, gridw = 1024;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *grid, F &&f) {
        const uint8_t *b = row + (g >> 3) * 74;
        const int ib = g & 7;
        const float d = ldh(b);
        const uint32_t sc = b[66 + ib];
        const float db0 = db_half(d, sc & 15u, 0.25f), db1 = db_half(d, sc >> 4, 0.25f);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t q = ld16(b + 2 + 2 * (4 * ib + l));
            const uint2 gw = *(const uint2 *)(grid + 2 * (q & 511u));
            grid8(f, 8 * l, gw.x, gw.y, l < 2 ? db0 : db1, ksign(q >> 9));
        }
    }
};

template <> struct Dec<T_IQ2_S> {
    static constexpr int qk = 256, bytes = 82, gridw = 2048;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *grid, F &&f) {
        const uint8_t *b = row + (g >> 3) * 82;
        const int ib = g & 7;
        const float d = ldh(b);
        const uint32_t qs = ld32u(b + 2 + 4 * ib), sg = ld32u(b + 34 + 4 * ib);
        const uint32_t qh = b[66 + ib], sc = b[74 + ib];
        const float db0 = db_half(d, sc & 15u, 0.25f), db1 = db_half(d, sc >> 4, 0.25f);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t e = ((qs >> (8 * l)) & 255u) | (((qh >> (2 * l)) & 3u) << 8);
            const uint2 gw = *(const uint2 *)(grid + 2 * e);
            grid8(f, 8 * l, gw.x, gw.y, l < 2 ? db0 : db1, (sg >> (8 * l)) & 255u);
        }
    }
};

template <> struct Dec<T_IQ3_XXS> {
    static constexpr int qk = 256, bytes = 98, gridw = 256;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *grid, F &&f) {
        const uint8_t *b = row + (g >> 3) * 98;
        const int ib = g & 7;
        const float d = ldh(b);
        const uint32_t q0 = ld32u(b + 2 + 8 * ib), q1 = ld32u(b + 6 + 8 * ib);
        const uint32_t aux = ld32u(b + 66 + 4 * ib);
        const float db = db_half(d, aux >> 28, 0.5f);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t qq = l < 2 ? q0 : q1, s = 16 * (l & 1);
            grid8(f, 8 * l, grid[(qq >> s) & 255u], grid[(qq >> (s + 8)) & 255u], db, ksign((aux >> (7 * l)) & 127u));
        }
    }
};

template <> struct Dec<T_IQ3_S> {
    static constexpr int qk = 256, bytes = 110, gridw = 512;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *grid, F &&f) {
        const uint8_t *b = row + (g >> 3) * 110;
        const int ib = g & 7;
        const float d = ldh(b);
        const uint32_t q0 = ld32u(b + 2 + 8 * ib), q1 = ld32u(b + 6 + 8 * ib);
        const uint32_t qh = b[66 + ib];
        const uint32_t sg = ld32u(b + 74 + 4 * ib);
        const uint32_t s4 = (b[106 + (ib >> 1)] >> (4 * (ib & 1))) & 15u;
        const float db = __fmul_rn(d, u2f(1u + 2u * s4));
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t qq = l < 2 ? q0 : q1, s = 16 * (l & 1);
            const uint32_t e0 = ((qq >> s) & 255u) | (((qh >> (2 * l)) & 1u) << 8);
            const uint32_t e1 = ((qq >> (s + 8)) & 255u) | (((qh >> (2 * l + 1)) & 1u) << 8);
            grid8(f, 8 * l, grid[e0], grid[e1], db, (sg >> (8 * l)) & 255u);
        }
    }
};

template <> struct Dec<T_IQ4_XS> {
    static constexpr int qk = 256, bytes = 136, gridw = 0;
    template <class F> __device__ __forceinline__ static void group(const uint8_t *row, int g, const uint32_t *, F &&f) {
        const uint8_t *b = row + (g >> 3) * 136;
        const int ib = g & 7;
        const float d = ldh(b);
        const uint32_t sh = ld16(b + 2);
        const uint32_t ls = ((b[4 + (ib >> 1)] >> (4 * (ib & 1))) & 15u) | (((sh >> (2 * ib)) & 3u) << 4);
        const float dl = __fmul_rn(d, u2f_off(ls, 32.0f));
        const uint8_t *qs = b + 8 + 16 * ib;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w = ld32a(qs + 4 * k);
            auto lo = [&](int s) { return __fmul_rn(dl, iq4nl((w >> (8 * s)) & 15u)); };
            auto hi = [&](int s) { return __fmul_rn(dl, iq4nl((w >> (8 * s + 4)) & 15u)); };
            f(4 * k, lo(0), lo(1), lo(2), lo(3));
            f(16 + 4 * k, hi(0), hi(1), hi(2), hi(3));
        }
    }
};

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
