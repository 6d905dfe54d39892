/*
 * tk_oracle.c -- CPU oracle for the tierk frozen-weight linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (tier_b200/, libtierk.so)
 * links, loads or calls this file; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py use it, and only as the
 * checker or the timed CPU baseline.
 *
 * It restates, in plain C, the reference's arithmetic for the path:
 *   - block formats and scalar dequant       tier/quant.h:20-121 (q_val): the
 *     legacy and K-quant types plus IQ4_NL, IQ4_XS, MXFP4, NF4, FP4, TQ1_0,
 *     TQ2_0 and the IQ1/IQ2/IQ3 lattice types (tables registered by the caller)
 *   - fp16 <-> fp32 software conversion      tier/quant.h:37-42, tier/gpu_compat.h:151-190
 *   - decode GEMV summation order            tier/tier.cpp:300-306 (gemv_q), 2261-2268 (gemv<T>)
 *   - x3 activation split                    tier/tier.cpp:869-870 (split3_fp_k)
 *   - chunked LM-head running CE + dlogit    tier/tier.cpp:736-759, 3184-3266
 *
 * Parity pin: tests/golden/ holds dequant vectors produced by gguf-py 0.19.0
 * (the reference's own test oracle, tier/check_quant.py:71) and by the
 * reference's quant.h compiled from its own sources (oracle/Makefile ->
 * oracle/_ref/); tests/test_oracle.py checks this file against both.
 *
 * Build: compiled with -ffp-contract=off so that every multiply and add rounds
 * separately, exactly as the reference's host code (no FMA) does.
 */
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <math.h>

/* Block-type codes: the reference's enum values (tier/quant.h:20-23). */
enum {
    TKO_F32 = 0, TKO_F16 = 1, TKO_Q4_0 = 2, TKO_Q4_1 = 3, TKO_Q5_0 = 6, TKO_Q5_1 = 7,
    TKO_Q8_0 = 8, TKO_Q2_K = 10, TKO_Q3_K = 11, TKO_Q4_K = 12, TKO_Q5_K = 13,
    TKO_Q6_K = 14, TKO_BF16 = 30,
    TKO_IQ4_NL = 20, TKO_IQ4_XS = 23, TKO_TQ1_0 = 34, TKO_TQ2_0 = 35, TKO_MXFP4 = 39,
    TKO_NF4 = 200, TKO_FP4 = 201,
    TKO_IQ2_XXS = 16, TKO_IQ2_XS = 17, TKO_IQ3_XXS = 18, TKO_IQ1_S = 19, TKO_IQ3_S = 21, TKO_IQ2_S = 22,
    TKO_IQ1_M = 29
};

/* (elements per block, bytes per block) -- tier/quant.h:25-29 */
int tko_block_geom(int type, int *elems, int *bytes)
{
    int e = 0, b = 0;
    switch (type) {
    case TKO_F32:  e = 1;   b = 4;   break;
    case TKO_F16:  e = 1;   b = 2;   break;
    case TKO_BF16: e = 1;   b = 2;   break;
    case TKO_Q4_0: e = 32;  b = 18;  break;
    case TKO_Q4_1: e = 32;  b = 20;  break;
    case TKO_Q5_0: e = 32;  b = 22;  break;
    case TKO_Q5_1: e = 32;  b = 24;  break;
    case TKO_Q8_0: e = 32;  b = 34;  break;
    case TKO_Q2_K: e = 256; b = 84;  break;
    case TKO_Q3_K: e = 256; b = 110; break;
    case TKO_Q4_K: e = 256; b = 144; break;
    case TKO_Q5_K: e = 256; b = 176; break;
    case TKO_Q6_K: e = 256; b = 210; break;
    case TKO_IQ4_NL: e = 32; b = 18; break;
    case TKO_MXFP4: e = 32;  b = 17;  break;
    case TKO_NF4:  e = 64;  b = 36;  break;
    case TKO_FP4:  e = 64;  b = 36;  break;
    case TKO_IQ4_XS: e = 256; b = 136; break;
    case TKO_TQ1_0: e = 256; b = 54; break;
    case TKO_TQ2_0: e = 256; b = 66; break;
    case TKO_IQ2_XXS: e = 256; b = 66; break;
    case TKO_IQ2_XS: e = 256; b = 74; break;
    case TKO_IQ2_S: e = 256; b = 82; break;
    case TKO_IQ3_XXS: e = 256; b = 98; break;
    case TKO_IQ3_S: e = 256; b = 110; break;
    case TKO_IQ1_S: e = 256; b = 50; break;
    case TKO_IQ1_M: e = 256; b = 56; break;
    default: return 0;
    }
    if (elems) *elems = e;
    if (bytes) *bytes = b;
    return 1;
}

/* tier/quant.h:33 q_row_bytes */
size_t tko_row_bytes(int type, int cols)
{
    int e, b;
    if (!tko_block_geom(type, &e, &b) || cols % e) return 0;
    return (size_t)(cols / e) * (size_t)b;
}

static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static uint16_t ld16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t ld32(const uint8_t *p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* Exact half -> float, including subnormals (tier/quant.h:37-42). */
float tko_h2f(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t ex = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    if (ex == 0) {
        if (man == 0) return bits_f32(sign);
        /* subnormal: value = man * 2^-24 exactly */
        int shift = 0;
        while (!(man & 0x400u)) { man <<= 1; ++shift; }
        return bits_f32(sign | ((uint32_t)(113 - shift) << 23) | ((man & 0x3ffu) << 13));
    }
    if (ex == 31) return bits_f32(sign | 0x7f800000u | (man << 13));
    return bits_f32(sign | ((ex + 112u) << 23) | (man << 13));
}

/* Float -> half with round-to-nearest-even, subnormals and overflow to inf
 * (tier/gpu_compat.h:151-174, tier_fp16::from_float). */
uint16_t tko_f2h(float f)
{
    uint32_t u = f32_bits(f);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t ex = (u >> 23) & 0xffu, man = u & 0x7fffffu;
    if (ex == 0xffu) return (uint16_t)(sign | (man ? 0x7e00u : 0x7c00u));
    int e = (int)ex - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int sh = 14 - e;
        uint32_t q = man >> sh, rem = man & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t q = man >> 13, rem = man & 0x1fffu;
    uint32_t h = sign | ((uint32_t)e << 10) | q;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++h; /* carry may ripple into the exponent: still RNE */
    return (uint16_t)h;
}

/* Float -> bfloat16 with round-to-nearest-even (what __float2bfloat16 does;
 * hip_bfloat16 on CUDA, tier/gpu_compat.h:134-140). NaN stays NaN. */
uint16_t tko_f2bf(float f)
{
    uint32_t u = f32_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

float tko_bf2f(uint16_t b) { return bits_f32((uint32_t)b << 16); }

static float blk_d(const uint8_t *p) { return tko_h2f(ld16(p)); }

/* Q4_K / Q5_K 6-bit sub-block scale and min unpack (tier/quant.h:47-48):
 * 12 packed bytes hold 8 scales and 8 mins.  Sub-blocks 0-3 keep their low
 * 6 bits in bytes j (scale) and j+4 (min); sub-blocks 4-7 take 4 bits from
 * byte j+4 and the top 2 bits from bytes j-4 (scale) and j (min). */
static void k_scale_min(int j, const uint8_t *s, int *sc, int *mn)
{
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* One weight value, bit-exact with tier/quant.h:59-121 (q_val) for the
 * non-table block types. Each product and difference rounds to fp32. */
/* 16-level lists of the table types (tier/quant.h:51-57; tier/quant_tables.h
 * qt_kv_iq4, qt_kv_mxfp4): IQ4 non-linear levels, MXFP4 doubled e2m1 levels,
 * QLoRA NormalFloat4 quantiles, bitsandbytes FP4 magnitudes / 12. */
static const int kv_iq4[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
static const int kv_mxfp4[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
static const float kv_nf4[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f, -0.28444138169288635f,
    -0.18477343022823334f, -0.09105003625154495f, 0.0f, 0.07958029955625534f, 0.16093020141124725f,
    0.24611230194568634f, 0.33791524171829224f, 0.44070982933044434f, 0.5626170039176941f,
    0.7229568362236023f, 1.0f};
static float fp4_level(int v)
{
    static const float m[8] = {0.0f, 0.0625f, 8.0f, 12.0f, 4.0f, 6.0f, 2.0f, 3.0f};
    float a = m[v % 8] / 12.0f;
    return v >= 8 ? -a : a;
}

/* Lattice tables of the IQ1/IQ2/IQ3 types (tier/quant_tables.h), registered
 * by the caller (tko_set_iq_grids; the tests pass gguf-py's IQ*.grid).  The
 * grid types decode to NaN until then. */
static const int8_t *g_iq2xxs, *g_iq2xs, *g_iq2s, *g_iq3xxs, *g_iq3s, *g_iq1s;
void tko_set_iq_grids(const int8_t *iq2xxs, const int8_t *iq2xs, const int8_t *iq2s, const int8_t *iq3xxs,
                      const int8_t *iq3s, const int8_t *iq1s)
{
    g_iq2xxs = iq2xxs; g_iq2xs = iq2xs; g_iq2s = iq2s; g_iq3xxs = iq3xxs; g_iq3s = iq3s; g_iq1s = iq1s;
}
/* qt_ksigns[j]: the 7 sign bits j plus an eighth that makes the parity even */
static unsigned ksign(unsigned j)
{
    unsigned p = 0;
    for (unsigned t = j; t; t >>= 1) p ^= t & 1;
    return j | (p << 7);
}
static float with_sign(float v, unsigned bits, int e) { return (bits >> e) & 1 ? v * -1.0f : v; }
/* d * (0.5 + s) * f: the IQ2/IQ3_XXS block scale, left to right as q_val */
static float half_step(float d, unsigned s, float f) { float t = d * (0.5f + (float)s); return t * f; }

static float grid_q_val(const uint8_t *row, int type, int col)
{
    int i = col % 256, e = i % 8;
    if (!g_iq1s) return NAN;
    switch (type) {
    case TKO_IQ2_XXS: { /* tier/quant.h:94-96 */
        const uint8_t *b = row + (size_t)(col / 256) * 66, *grp = b + 2 + 8 * (i / 32);
        int k = (i % 32) / 8;
        uint32_t aux = ld32(grp + 4);
        float db = half_step(blk_d(b), aux >> 28, 0.25f);
        return with_sign(db * (float)g_iq2xxs[grp[k] * 8 + e], ksign((aux >> (7 * k)) & 127), e);
    }
    case TKO_IQ2_XS: { /* tier/quant.h:97-99 */
        const uint8_t *b = row + (size_t)(col / 256) * 74;
        unsigned q = ld16(b + 2 + 2 * (i / 8)), s = i / 16;
        float db = half_step(blk_d(b), (b[66 + s / 2] >> (s % 2 ? 4 : 0)) & 15, 0.25f);
        return with_sign(db * (float)g_iq2xs[(q % 512) * 8 + e], ksign(q >> 9), e);
    }
    case TKO_IQ2_S: { /* tier/quant.h:100-102 */
        const uint8_t *b = row + (size_t)(col / 256) * 82;
        int k = i / 8, s = i / 16;
        float db = half_step(blk_d(b), (b[74 + s / 2] >> (s % 2 ? 4 : 0)) & 15, 0.25f);
        int gi = b[2 + k] + 256 * ((b[66 + k / 4] >> (2 * (k % 4))) & 3);
        return with_sign(db * (float)g_iq2s[gi * 8 + e], b[34 + k], e);
    }
    case TKO_IQ3_XXS: { /* tier/quant.h:103-105 */
        const uint8_t *b = row + (size_t)(col / 256) * 98;
        uint32_t aux = ld32(b + 66 + 4 * (i / 32));
        float db = half_step(blk_d(b), aux >> 28, 0.5f);
        return with_sign(db * (float)g_iq3xxs[b[2 + i / 4] * 4 + i % 4], ksign((aux >> (7 * ((i % 32) / 8))) & 127), e);
    }
    case TKO_IQ3_S: { /* tier/quant.h:106-108 */
        const uint8_t *b = row + (size_t)(col / 256) * 110;
        int g = i / 32, k = i / 4;
        float db = blk_d(b) * (float)(1 + 2 * ((b[106 + g / 2] >> (g % 2 ? 4 : 0)) & 15));
        int gi = b[2 + k] + 256 * ((b[66 + k / 8] >> (k % 8)) & 1);
        return with_sign(db * (float)g_iq3s[gi * 4 + i % 4], b[74 + i / 8], e);
    }
    case TKO_IQ1_S: { /* tier/quant.h:109-111 */
        const uint8_t *b = row + (size_t)(col / 256) * 50;
        int k = i / 8;
        unsigned qh = ld16(b + 34 + 2 * (i / 32));
        float dl = blk_d(b) * (float)(2 * ((qh >> 12) & 7) + 1);
        float dt = (qh & 0x8000) ? -0.125f : 0.125f;
        int gi = b[2 + k] + 256 * ((qh >> (3 * (k % 4))) & 7);
        return dl * ((float)g_iq1s[gi * 8 + e] + dt);
    }
    case TKO_IQ1_M: { /* tier/quant.h:112-115 */
        const uint8_t *b = row + (size_t)(col / 256) * 56, *sc = b + 48;
        int k = i / 8, s = i / 16;
        unsigned dh = 0;
        for (int w = 0; w < 4; ++w) dh |= (unsigned)(ld16(sc + 2 * w) >> 12) << (4 * w);
        float dl = tko_h2f((uint16_t)dh) * (float)(2 * ((ld16(sc + 2 * (s / 4)) >> (3 * (s % 4))) & 7) + 1);
        int nib = (b[32 + k / 2] >> (k % 2 ? 4 : 0)) & 15;
        float dt = (nib & 8) ? -0.125f : 0.125f;
        return dl * ((float)g_iq1s[(b[k] + 256 * (nib & 7)) * 8 + e] + dt);
    }
    default: return 0.0f;
    }
}

/* element i of a 32-element block of 16 nibble bytes: low nibbles first, then high */
static int nib32(const uint8_t *qs, int i) { return (qs[i % 16] >> (i < 16 ? 0 : 4)) & 15; }

float tko_q_val(const uint8_t *row, int type, int col)
{
    switch (type) {
    case TKO_IQ2_XXS: case TKO_IQ2_XS: case TKO_IQ2_S: case TKO_IQ3_XXS: case TKO_IQ3_S:
    case TKO_IQ1_S: case TKO_IQ1_M:
        return grid_q_val(row, type, col);
    case TKO_IQ4_NL: { /* [d f16][16 B]: d * kv_iq4[q] (tier/quant.h:69) */
        const uint8_t *b = row + (size_t)(col / 32) * 18;
        return blk_d(b) * (float)kv_iq4[nib32(b + 2, col % 32)];
    }
    case TKO_MXFP4: { /* [e][16 B]: 2^(e-128) * kv_mxfp4[q] (tier/quant.h:70-71) */
        const uint8_t *b = row + (size_t)(col / 32) * 17;
        float scale = ldexpf(1.0f, (int)b[0] - 128);   /* exact, subnormal for e < 2 */
        return scale * (float)kv_mxfp4[nib32(b + 1, col % 32)];
    }
    case TKO_NF4: case TKO_FP4: { /* [absmax f32][32 B], element 2k high nibble, 2k+1 low (tier/quant.h:72-73) */
        const uint8_t *b = row + (size_t)(col / 64) * 36;
        int i = col % 64, y = b[4 + i / 2], q = (i % 2) ? (y & 15) : (y >> 4);
        float a = bits_f32(ld32(b));
        return (type == TKO_NF4 ? kv_nf4[q] : fp4_level(q)) * a;
    }
    default: break;
    }
    switch (type) {
    case TKO_F32:  return bits_f32(ld32(row + (size_t)col * 4));
    case TKO_F16:  return tko_h2f(ld16(row + (size_t)col * 2));
    case TKO_BF16: return tko_bf2f(ld16(row + (size_t)col * 2));
    case TKO_Q4_0: { /* [d f16][16 B of nibbles]; element i<16 low nibble of byte i, else high nibble of byte i-16 */
        const uint8_t *b = row + (size_t)(col / 32) * 18;
        int i = col % 32, q = (b[2 + (i % 16)] >> (i < 16 ? 0 : 4)) & 15;
        return blk_d(b) * (float)(q - 8);
    }
    case TKO_Q4_1: { /* [d f16][m f16][16 B nibbles]: d*q + m */
        const uint8_t *b = row + (size_t)(col / 32) * 20;
        int i = col % 32, q = (b[4 + (i % 16)] >> (i < 16 ? 0 : 4)) & 15;
        float t = blk_d(b) * (float)q;
        return t + blk_d(b + 2);
    }
    case TKO_Q5_0: { /* [d f16][qh u32][16 B nibbles]; fifth bit i of qh */
        const uint8_t *b = row + (size_t)(col / 32) * 22;
        int i = col % 32;
        int q = ((b[6 + (i % 16)] >> (i < 16 ? 0 : 4)) & 15) | (int)(((ld32(b + 2) >> i) & 1u) << 4);
        return blk_d(b) * (float)(q - 16);
    }
    case TKO_Q5_1: {
        const uint8_t *b = row + (size_t)(col / 32) * 24;
        int i = col % 32;
        int q = ((b[8 + (i % 16)] >> (i < 16 ? 0 : 4)) & 15) | (int)(((ld32(b + 4) >> i) & 1u) << 4);
        float t = blk_d(b) * (float)q;
        return t + blk_d(b + 2);
    }
    case TKO_Q8_0: { /* [d f16][32 x int8] */
        const uint8_t *b = row + (size_t)(col / 32) * 34;
        return blk_d(b) * (float)(int8_t)b[2 + (col % 32)];
    }
    default: break;
    }
    int i = col % 256;
    switch (type) {
    case TKO_Q2_K: { /* [scales 16][qs 64][d f16][dmin f16]: (d*(sc&15))*q - dmin*(sc>>4) */
        const uint8_t *b = row + (size_t)(col / 256) * 84;
        int half = i / 128, shift = 2 * ((i % 128) / 32), l = i % 32;
        int q = (b[16 + half * 32 + l] >> shift) & 3;
        uint8_t sc = b[i / 16];
        float a = blk_d(b + 80) * (float)(sc & 15);
        float t = a * (float)q;
        float m = blk_d(b + 82) * (float)(sc >> 4);
        return t - m;
    }
    case TKO_Q3_K: { /* [hmask 32][qs 64][scales 12][d f16] */
        const uint8_t *b = row + (size_t)(col / 256) * 110;
        const uint8_t *s = b + 96;
        int j = i / 16;
        int lo = j < 8 ? (s[j] & 15) : (s[j - 8] >> 4);
        int hi = (s[8 + (j % 4)] >> (2 * (j / 4))) & 3;
        int sc = (int)(int8_t)(uint8_t)(lo | (hi << 4)) - 32;
        int half = i / 128, shift = 2 * ((i % 128) / 32), l = i % 32;
        int ql = (b[32 + half * 32 + l] >> shift) & 3;
        int hbit = ((b[l] >> (i / 32)) & 1) ^ 1;
        float a = blk_d(b + 108) * (float)sc;
        return a * (float)(ql - (hbit << 2));
    }
    case TKO_Q4_K: { /* [d f16][dmin f16][scales 12][qs 128] */
        const uint8_t *b = row + (size_t)(col / 256) * 144;
        int g = i / 64, l = i % 64, sc, mn;
        k_scale_min(2 * g + (l >= 32), b + 4, &sc, &mn);
        uint8_t y = b[16 + g * 32 + (l % 32)];
        int q = l < 32 ? (y & 15) : (y >> 4);
        float a = blk_d(b) * (float)sc;
        float t = a * (float)q;
        float m = blk_d(b + 2) * (float)mn;
        return t - m;
    }
    case TKO_Q5_K: { /* [d f16][dmin f16][scales 12][qh 32][qs 128] */
        const uint8_t *b = row + (size_t)(col / 256) * 176;
        int g = i / 64, l = i % 64, sc, mn;
        k_scale_min(2 * g + (l >= 32), b + 4, &sc, &mn);
        uint8_t y = b[48 + g * 32 + (l % 32)];
        int q = (l < 32 ? (y & 15) : (y >> 4)) | (((b[16 + (i % 32)] >> (i / 32)) & 1) << 4);
        float a = blk_d(b) * (float)sc;
        float t = a * (float)q;
        float m = blk_d(b + 2) * (float)mn;
        return t - m;
    }
    case TKO_Q6_K: { /* [ql 128][qh 64][scales int8 16][d f16] */
        const uint8_t *b = row + (size_t)(col / 256) * 210;
        int a128 = i / 128, c = i % 64, nib = (i % 128) / 64, sh = (i % 128) / 32, l = i % 32;
        int ql = (b[a128 * 64 + c] >> (4 * nib)) & 15;
        int qh = (b[128 + a128 * 32 + l] >> (2 * sh)) & 3;
        int q = (int)(int8_t)(uint8_t)(ql | (qh << 4)) - 32;
        float a = blk_d(b + 208) * (float)(int8_t)b[192 + i / 16];
        return a * (float)q;
    }
    case TKO_IQ4_XS: { /* [d f16][sh u16][sl 4 B][qs 128 B]: (d*sc) * kv_iq4[q] (tier/quant.h:91-93) */
        const uint8_t *b = row + (size_t)(col / 256) * 136;
        int j = i / 32;
        int lo = (b[4 + j / 2] >> (j % 2 ? 4 : 0)) & 15, hi = (ld16(b + 2) >> (2 * j)) & 3;
        int sc = lo + 16 * hi - 32;
        float a = blk_d(b) * (float)sc;
        return a * (float)kv_iq4[nib32(b + 8 + 16 * j, i % 32)];
    }
    case TKO_TQ2_0: { /* [qs 64 B][d f16]: four 2-bit codes per byte, d*(c-1) (tier/quant.h:116) */
        const uint8_t *b = row + (size_t)(col / 256) * 66;
        int c = (b[(i / 128) * 32 + i % 32] >> (2 * ((i % 128) / 32))) & 3;
        return blk_d(b + 64) * (float)(c - 1);
    }
    case TKO_TQ1_0: { /* [qs 48 B][qh 4 B][d f16]: base-3 digits, d*(c-1) (tier/quant.h:117-119) */
        const uint8_t *b = row + (size_t)(col / 256) * 54;
        int byte, n;
        if (i < 160) { byte = i % 32; n = i / 32; }
        else if (i < 240) { byte = 32 + (i - 160) % 16; n = (i - 160) / 16; }
        else { byte = 48 + (i - 240) % 4; n = (i - 240) / 4; }
        unsigned p = 1;
        for (int k = 0; k < n; ++k) p *= 3;
        unsigned x = (b[byte] * p) % 256;
        int c = (int)((x * 3) / 256);
        return blk_d(b + 52) * (float)(c - 1);
    }
    default: break;
    }
    return 0.0f;
}

/* Expand rows [r0, r0+nrows) of a block matrix: out_dtype 0 = fp32,
 * 1 = fp16 (RNE of the fp32 value, tier/tier.cpp:294-296 with T=tier_fp16),
 * 2 = bf16 (RNE, T=hip_bfloat16). */
void tko_dequant(const uint8_t *W, size_t row_bytes, int type, int r0, int nrows, int cols,
                 int out_dtype, void *out)
{
    for (int r = 0; r < nrows; ++r) {
        const uint8_t *row = W + (size_t)(r0 + r) * row_bytes;
        for (int c = 0; c < cols; ++c) {
            float v = tko_q_val(row, type, c);
            size_t o = (size_t)r * cols + c;
            if (out_dtype == 0) ((float *)out)[o] = v;
            else if (out_dtype == 1) ((uint16_t *)out)[o] = tko_f2h(v);
            else ((uint16_t *)out)[o] = tko_f2bf(v);
        }
    }
}

/* Decode GEMV in the reference's summation order (tier/tier.cpp:300-306):
 * lane l of a 32-wide warp accumulates columns l, l+32, ... with a fused
 * multiply-add (nvcc contracts acc+=a*b), then the warp tree-reduces with
 * offsets 16, 8, 4, 2, 1. y[n] = sum_k q_val(W[n], k) * x[k]. */
void tko_gemv_q_warp_order(const uint8_t *W, size_t row_bytes, int type, const float *x,
                           float *y, int N, int K)
{
    float acc[32];
    for (int n = 0; n < N; ++n) {
        const uint8_t *row = W + (size_t)n * row_bytes;
        for (int l = 0; l < 32; ++l) {
            float a = 0.0f;
            for (int k = l; k < K; k += 32) a = fmaf(tko_q_val(row, type, k), x[k], a);
            acc[l] = a;
        }
        for (int off = 16; off > 0; off >>= 1)
            for (int l = 0; l < off; ++l) acc[l] = acc[l] + acc[l + off];
        y[n] = acc[0];
    }
}

/* Y[m,n] = sum_k X[m,k] * Wq(n,k) in double: the fp64 yardstick the
 * GEMV/GEMM tolerances are stated against. X fp32 row-major [M,K]. */
void tko_qgemm_f64(const uint8_t *W, size_t row_bytes, int type, const float *X,
                   double *Y, int M, int N, int K)
{
    for (int n = 0; n < N; ++n) {
        const uint8_t *row = W + (size_t)n * row_bytes;
        for (int m = 0; m < M; ++m) Y[(size_t)m * N + n] = 0.0;
        for (int k = 0; k < K; ++k) {
            double w = (double)tko_q_val(row, type, k);
            for (int m = 0; m < M; ++m) Y[(size_t)m * N + n] += w * (double)X[(size_t)m * K + k];
        }
    }
}

/* fp32 -> three fp16 parts (tier/tier.cpp:869-870, split3_fp_k):
 * h = f16(x), m = f16(x - h), l = f16((x - h) - m), every step rounded. */
void tko_split3_f16(const float *x, uint16_t *h, uint16_t *m, uint16_t *l, size_t n)
{
    for (size_t i = 0; i < n; ++i) {
        float v = x[i];
        uint16_t a = tko_f2h(v);
        float r = v - tko_h2f(a);
        uint16_t b = tko_f2h(r);
        float r2 = r - tko_h2f(b);
        h[i] = a; m[i] = b; l[i] = tko_f2h(r2);
    }
}

/* Running-CE state update for one vocab chunk (tier/tier.cpp:750-759,
 * lse_chunk_kernel): for each predicted row t with mask[t] != 0, take the
 * chunk max and its lowest index, the fp64 sum of exp(logit - chunk max),
 * merge into (rmax, rsum) and record the target logit when labels[t+1]
 * falls in [v0, v0+vc).  logits is the post-softcap chunk [T, vc]. */
void tko_lse_chunk(const float *lg, double *rmax, double *rsum, int *amax, float *tgt,
                   const int32_t *labels, const uint8_t *mask, int n_pred, int vc, int v0)
{
    for (int t = 0; t < n_pred; ++t) {
        if (!mask[t]) continue;
        const float *row = lg + (size_t)t * vc;
        float bm = -1e30f;
        int bi = 0x7fffffff;
        for (int v = 0; v < vc; ++v)
            if (row[v] > bm || (row[v] == bm && v < bi)) { bm = row[v]; bi = v; }
        /* the kernel's order: 256 threads each sum v = tid, tid+256, ...; then
         * a halving tree over the 256 partials (tier/tier.cpp:755-756) */
        double sd[256];
        for (int i = 0; i < 256; ++i) {
            double s = 0.0;
            for (int v = i; v < vc; v += 256) s += exp((double)row[v] - (double)bm);
            sd[i] = s;
        }
        for (int o = 128; o > 0; o >>= 1)
            for (int i = 0; i < o; ++i) sd[i] += sd[i + o];
        double s = sd[0];
        double om = rmax[t], nm = fmax(om, (double)bm);
        if ((double)bm > om) amax[t] = v0 + bi;
        rsum[t] = rsum[t] * exp(om - nm) + s * exp((double)bm - nm);
        rmax[t] = nm;
        int g = labels[t + 1] - v0;
        if (g >= 0 && g < vc) tgt[t] = row[g];
    }
}

/* dlogit for one chunk (tier/tier.cpp:736-748): rows t >= T-1 or masked
 * out are zero; else ((softmax - onehot) / n_loss) * (1 - y^2) * mask,
 * with softmax in fp64 and y = logit/cap when cap > 0. */
void tko_dlogit(const float *lg, const double *rmax, const double *rsum, const int32_t *labels,
                float *dl, int T, int vc, int v0, int n_loss, const uint8_t *mask, float cap)
{
    for (int t = 0; t < T; ++t) {
        for (int v = 0; v < vc; ++v) {
            size_t i = (size_t)t * vc + v;
            if (t >= T - 1 || !mask[t]) { dl[i] = 0.0f; continue; }
            double lse = rmax[t] + log(rsum[t]);
            double p = exp((double)lg[i] - lse);
            double oh = (v0 + v == labels[t + 1]) ? 1.0 : 0.0;
            float y = cap > 0.0f ? lg[i] / cap : 0.0f;
            float g = (float)((p - oh) / n_loss);
            dl[i] = g * (1.0f - y * y) * (float)mask[t];
        }
    }
}

/* Whole LM head in fp64, chunked exactly as tier/tier.cpp:3184-3266:
 * logits = softcap(Xh . W^T) per chunk, running max/sum/argmax/target,
 * loss_sum = sum over masked rows of (lse - target), then
 * dX = sum_chunks dlogit . W.  W is fp16 bits [V, H]; Xh fp32 [T, H].
 * Outputs: *loss_sum, *n_loss, amax[T-1], dX (double) [T, H].
 * All logits are computed in double and rounded to fp32 before the
 * running-state update, as the reference's fp32 GEMM output would be. */
void tko_lmhead_f64(const uint16_t *W, int V, int H, const float *X, int T,
                    const int32_t *labels, const uint8_t *mask, float cap, int chunk,
                    double *loss_sum, int *n_loss_out, int *amax, double *dX,
                    float *lg_buf /* [T*chunk] scratch */, double *rmax, double *rsum, float *tgt)
{
    int n_pred = T - 1, n_loss = 0;
    for (int t = 0; t < n_pred; ++t) n_loss += mask[t] != 0;
    for (int t = 0; t < n_pred; ++t) { rmax[t] = -1e30; rsum[t] = 0.0; amax[t] = -1; tgt[t] = 0.0f; }
    for (size_t i = 0; i < (size_t)T * H; ++i) dX[i] = 0.0;
    for (int pass = 0; pass < 2; ++pass) {
        for (int v0 = 0; v0 < V; v0 += chunk) {
            int vc = V - v0 < chunk ? V - v0 : chunk;
            for (int t = 0; t < T; ++t)
                for (int v = 0; v < vc; ++v) {
                    const uint16_t *w = W + (size_t)(v0 + v) * H;
                    const float *x = X + (size_t)t * H;
                    double s = 0.0;
                    for (int k = 0; k < H; ++k) s += (double)tko_h2f(w[k]) * (double)x[k];
                    float l = (float)s;
                    if (cap > 0.0f) l = (float)((double)cap * tanh((double)l / (double)cap));
                    lg_buf[(size_t)t * vc + v] = l;
                }
            if (pass == 0) {
                tko_lse_chunk(lg_buf, rmax, rsum, amax, tgt, labels, mask, n_pred, vc, v0);
            } else {
                for (int t = 0; t < T; ++t) {
                    if (t >= T - 1 || !mask[t]) continue;
                    double lse = rmax[t] + log(rsum[t]);
                    for (int v = 0; v < vc; ++v) {
                        double l = (double)lg_buf[(size_t)t * vc + v];
                        double p = exp(l - lse);
                        double oh = (v0 + v == labels[t + 1]) ? 1.0 : 0.0;
                        double y = cap > 0.0f ? l / cap : 0.0;
                        double g = (p - oh) / n_loss * (1.0 - y * y);
                        const uint16_t *w = W + (size_t)(v0 + v) * H;
                        double *d = dX + (size_t)t * H;
                        for (int k = 0; k < H; ++k) d[k] += g * (double)tko_h2f(w[k]);
                    }
                }
            }
        }
    }
    double tot = 0.0;
    for (int t = 0; t < n_pred; ++t)
        if (mask[t]) tot += rmax[t] + log(rsum[t]) - (double)tgt[t];
    *loss_sum = tot;
    *n_loss_out = n_loss;
}
