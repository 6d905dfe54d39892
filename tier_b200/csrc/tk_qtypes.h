// tk_qtypes.h -- block types whose levels come from a 16-entry list or from
// base-3 packing rather than from an integer grid: IQ4_NL, IQ4_XS, MXFP4, NF4,
// FP4, TQ1_0 and TQ2_0.  Element values are bit-exact with q_val
// (tier/quant.h:69-73, 91-93, 116-119; level lists tier/quant.h:51-57 and
// tier/quant_tables.h qt_kv_iq4 / qt_kv_mxfp4).
//
// The header compiles as CUDA (the dequant and GEMV kernels include it through
// tk_device.cuh) and as plain C++ (the host check in tests/ compiles the same
// functions and compares them with the reference's own q_val).  Every product
// is a single rounded multiply and nothing is added afterwards, so there is no
// multiply-add for a compiler to fuse.
#pragma once
#include <stdint.h>
#include <string.h>
#if defined(__CUDACC__)
#include <cuda_fp16.h>
#define TKQ_FN __host__ __device__ __forceinline__
#else
#define TKQ_FN inline
#endif

namespace tkq {

// Type codes: the format's enum values (tier/quant.h:20-23).
enum : int { IQ4_NL = 20, IQ4_XS = 23, TQ1_0 = 34, TQ2_0 = 35, MXFP4 = 39, NF4 = 200, FP4 = 201 };

// (elements, bytes) per block, tier/quant.h:29-31; 0 for any other type.
TKQ_FN int elems(int t) {
    return t == IQ4_NL || t == MXFP4 ? 32 : t == NF4 || t == FP4 ? 64 : t == IQ4_XS || t == TQ1_0 || t == TQ2_0 ? 256 : 0;
}
TKQ_FN int bytes(int t) {
    switch (t) {
        case IQ4_NL: return 18;
        case MXFP4: return 17;
        case NF4: case FP4: return 36;
        case IQ4_XS: return 136;
        case TQ1_0: return 54;
        case TQ2_0: return 66;
        default: return 0;
    }
}

TKQ_FN float as_f32(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}
TKQ_FN float mul(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}
TKQ_FN uint32_t le16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// IEEE binary16 -> binary32, exact for every input (subnormals normalised,
// infinities and NaN payloads kept).
TKQ_FN float half_to_f32(uint32_t h) {
#if defined(__CUDA_ARCH__)
    return __half2float(__ushort_as_half((unsigned short)h));
#else
    const uint32_t sign = (h & 0x8000u) << 16, ex = (h >> 10) & 31u, man = h & 0x3ffu;
    if (ex == 31) return as_f32(sign | 0x7f800000u | (man << 13));
    if (ex != 0) return as_f32(sign | ((ex + 112u) << 23) | (man << 13));
    if (man == 0) return as_f32(sign);
    // subnormal: man * 2^-24, exact in fp32
    int shift = 0;
    uint32_t m = man;
    while (!(m & 0x400u)) { m <<= 1; ++shift; }
    return as_f32(sign | ((uint32_t)(113 - shift) << 23) | ((m & 0x3ffu) << 13));
#endif
}

// Non-linear 4-bit levels of IQ4_NL / IQ4_XS (the format's fixed list).
TKQ_FN int iq4_level(int v) {
    const int8_t lv[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
    return lv[v];
}
// MXFP4 element: an OCP e2m1 code with its value doubled (so every level is
// an integer): magnitudes 0, 1, 2, 3, 4, 6, 8, 12, bit 3 the sign.
TKQ_FN int mxfp4_level(int v) {
    const int mag = v & 7;
    const int a = mag < 4 ? mag : (mag == 4 ? 4 : mag == 5 ? 6 : mag == 6 ? 8 : 12);
    return (v & 8) ? -a : a;
}
// MXFP4 block scale: the E8M0 byte e as 2^(e-128) (the -1 undoes the doubled
// levels); a normal fp32 for e >= 2, a subnormal for e = 0, 1.
TKQ_FN float mxfp4_scale(uint32_t e) { return as_f32(e >= 2 ? (e - 1) << 23 : 0x00200000u << e); }
// NF4: the sixteen normal-distribution quantiles of QLoRA's NormalFloat4.
TKQ_FN float nf4_level(int v) {
    const float lv[16] = {-1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
                          -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
                          0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
                          0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};
    return lv[v];
}
// FP4 (bitsandbytes layout): magnitudes {0, 1/16, 8, 12, 4, 6, 2, 3} / 12 for
// codes 0-7, bit 3 the sign (code 8 is -0).
TKQ_FN float fp4_level(int v) {
    const float m[8] = {0.0f, 0.0625f, 8.0f, 12.0f, 4.0f, 6.0f, 2.0f, 3.0f};
    const float a = m[v & 7] / 12.0f;
    return (v & 8) ? -a : a;
}

// Value of element `col` of a row of blocks of type t (one of the codes above).
TKQ_FN float value(const uint8_t* row, int t, int col) {
    switch (t) {
        case IQ4_NL: {   // [d f16][16 B]: element i < 16 low nibble of byte i, else high nibble of byte i-16
            const uint8_t* b = row + (size_t)(col >> 5) * 18;
            const int i = col & 31, q = (b[2 + (i & 15)] >> (i & 16 ? 4 : 0)) & 15;
            return mul(half_to_f32(le16(b)), (float)iq4_level(q));
        }
        case MXFP4: {    // [e8m0 scale][16 B], nibbles as IQ4_NL
            const uint8_t* b = row + (size_t)(col >> 5) * 17;
            const int i = col & 31, q = (b[1 + (i & 15)] >> (i & 16 ? 4 : 0)) & 15;
            return mul(mxfp4_scale(b[0]), (float)mxfp4_level(q));
        }
        case NF4:
        case FP4: {      // [absmax f32][32 B]: even elements the high nibble, odd the low
            const uint8_t* b = row + (size_t)(col >> 6) * 36;
            const int i = col & 63;
            const uint32_t y = b[4 + (i >> 1)];
            const int q = (int)((i & 1) ? (y & 15u) : (y >> 4));
            const float a = as_f32(le16(b) | (le16(b + 2) << 16));
            return mul(t == NF4 ? nf4_level(q) : fp4_level(q), a);
        }
        case IQ4_XS: {   // [d f16][scales_h u16][scales_l 4 B][qs 128 B], eight 32-element sub-blocks
            const uint8_t* b = row + (size_t)(col >> 8) * 136;
            const int i = col & 255, j = i >> 5;
            const int lo = (b[4 + (j >> 1)] >> (4 * (j & 1))) & 15, hi = (int)(le16(b + 2) >> (2 * j)) & 3;
            const int sc = (lo | (hi << 4)) - 32;
            const int q = (b[8 + 16 * j + (i & 15)] >> (i & 16 ? 4 : 0)) & 15;
            return mul(mul(half_to_f32(le16(b)), (float)sc), (float)iq4_level(q));
        }
        case TQ2_0: {    // [qs 64 B][d f16]: 2-bit codes c, value d*(c-1)
            const uint8_t* b = row + (size_t)(col >> 8) * 66;
            const int i = col & 255;
            const int c = (b[32 * (i >> 7) + (i & 31)] >> (2 * ((i >> 5) & 3))) & 3;
            return mul(half_to_f32(le16(b + 64)), (float)(c - 1));
        }
        case TQ1_0: {    // [qs 48 B][qh 4 B][d f16]: five (qs) or four (qh) base-3 digits per byte
            const uint8_t* b = row + (size_t)(col >> 8) * 54;
            const int i = col & 255;
            int byte, digit;
            if (i < 160) { byte = i & 31; digit = i >> 5; }
            else if (i < 240) { byte = 32 + ((i - 160) & 15); digit = (i - 160) >> 4; }
            else { byte = 48 + ((i - 240) & 3); digit = (i - 240) >> 2; }
            const uint32_t pow3 = digit == 0 ? 1u : digit == 1 ? 3u : digit == 2 ? 9u : digit == 3 ? 27u : 81u;
            // the byte holds ceil(v * 256 / 3^n) for the n-digit number v;
            // multiplying by 3^digit (mod 256) brings the wanted digit to the
            // top, and (x * 3) >> 8 reads it
            const uint32_t x = (b[byte] * pow3) & 0xffu;
            const int c = (int)((x * 3u) >> 8);
            return mul(half_to_f32(le16(b + 52)), (float)(c - 1));
        }
        default: return 0.0f;
    }
}

}  // namespace tkq
