// tk_qgrid.h -- the lattice ("grid") block types IQ2_XXS, IQ2_XS, IQ2_S,
// IQ3_XXS, IQ3_S, IQ1_S and IQ1_M: element values bit-exact with q_val
// (tier/quant.h:94-115).  Each type looks its 8- or 4-element groups up in a
// fixed lattice table.  The tables are the format's data (tier/quant_tables.h;
// the same numbers as gguf-py's IQ*.grid).  The library does not carry them:
// the caller registers its copy once (tk_set_iq_grids) and every kernel reads
// it from one device buffer with the layout below.  The sign table is not
// registered: entry i is i with bit 7 set when i has an odd number of set
// bits, so every sign byte has even parity.
//
// Compiles as CUDA and as plain C++, like tk_qtypes.h (the host build is
// checked against the reference's q_val in tests/).  The products keep the
// reference's order, and the only additions are exact: 0.5 + a 4-bit integer,
// and a grid integer + 1/8.
#pragma once
#include "tk_qtypes.h"

namespace tkq {

enum : int { IQ2_XXS = 16, IQ2_XS = 17, IQ3_XXS = 18, IQ1_S = 19, IQ3_S = 21, IQ2_S = 22, IQ1_M = 29 };

// Offsets (bytes) into the registered table buffer.  Grid entries are int8.
enum : int {
    GRID_IQ2XXS = 0,                       // [256][8]
    GRID_IQ2XS = GRID_IQ2XXS + 256 * 8,    // [512][8]
    GRID_IQ2S = GRID_IQ2XS + 512 * 8,      // [1024][8]
    GRID_IQ3XXS = GRID_IQ2S + 1024 * 8,    // [256][4]
    GRID_IQ3S = GRID_IQ3XXS + 256 * 4,     // [512][4]
    GRID_IQ1S = GRID_IQ3S + 512 * 4,       // [2048][8], shared by IQ1_S and IQ1_M
    GRID_SIGNS = GRID_IQ1S + 2048 * 8,     // [128] uint8, filled by the library
    GRID_BYTES = GRID_SIGNS + 128
};

TKQ_FN bool is_grid(int t) {
    return t == IQ2_XXS || t == IQ2_XS || t == IQ2_S || t == IQ3_XXS || t == IQ3_S || t == IQ1_S || t == IQ1_M;
}
TKQ_FN int grid_bytes(int t) {   // bytes per 256-element block (tier/quant.h:28-29)
    switch (t) {
        case IQ2_XXS: return 66;
        case IQ2_XS: return 74;
        case IQ2_S: return 82;
        case IQ3_XXS: return 98;
        case IQ3_S: return 110;
        case IQ1_S: return 50;
        case IQ1_M: return 56;
        default: return 0;
    }
}
TKQ_FN uint8_t sign_byte(int i) {   // the value the table's GRID_SIGNS entry i holds
    int p = 0;
    for (int b = 0; b < 7; ++b) p ^= (i >> b) & 1;
    return (uint8_t)(i | (p << 7));
}
TKQ_FN uint32_t le32(const uint8_t* p) { return le16(p) | (le16(p + 2) << 16); }
TKQ_FN float flip(float v, uint32_t sign_bits, int e) { return (sign_bits >> e) & 1 ? -v : v; }

// Value of element `col` of a row of 256-element blocks of grid type t.
TKQ_FN float grid_value(const uint8_t* row, int t, int col, const int8_t* tab) {
    const int i = col & 255, e = i & 7;
    const uint8_t* signs = reinterpret_cast<const uint8_t*>(tab + GRID_SIGNS);
    switch (t) {
        case IQ2_XXS: {   // [d][8 groups x (4 grid bytes, u32: 4-bit scale | 4 x 7-bit sign index)]
            const uint8_t* b = row + (size_t)(col >> 8) * 66;
            const uint8_t* grp = b + 2 + 8 * (i >> 5);
            const int k = (i >> 3) & 3;
            const uint32_t aux = le32(grp + 4);
            const float db = mul(mul(half_to_f32(le16(b)), 0.5f + (float)(aux >> 28)), 0.25f);
            const int8_t g = tab[GRID_IQ2XXS + grp[k] * 8 + e];
            return flip(mul(db, (float)g), signs[(aux >> (7 * k)) & 127], e);
        }
        case IQ2_XS: {    // [d][32 x u16: 9-bit grid index | 7-bit sign index][8 scale bytes, two 4-bit]
            const uint8_t* b = row + (size_t)(col >> 8) * 74;
            const uint32_t q = le16(b + 2 + 2 * (i >> 3));
            const int s = i >> 4;
            const int sc = (b[66 + (s >> 1)] >> (4 * (s & 1))) & 15;
            const float db = mul(mul(half_to_f32(le16(b)), 0.5f + (float)sc), 0.25f);
            const int8_t g = tab[GRID_IQ2XS + (q & 511) * 8 + e];
            return flip(mul(db, (float)g), signs[q >> 9], e);
        }
        case IQ2_S: {     // [d][32 grid low bytes][32 sign bytes][8 bytes of 2-bit grid highs][8 scale bytes]
            const uint8_t* b = row + (size_t)(col >> 8) * 82;
            const int k = i >> 3, s = i >> 4;
            const int sc = (b[74 + (s >> 1)] >> (4 * (s & 1))) & 15;
            const float db = mul(mul(half_to_f32(le16(b)), 0.5f + (float)sc), 0.25f);
            const int gi = b[2 + k] | (((b[66 + (k >> 2)] >> (2 * (k & 3))) & 3) << 8);
            return flip(mul(db, (float)tab[GRID_IQ2S + gi * 8 + e]), b[34 + k], e);
        }
        case IQ3_XXS: {   // [d][64 grid bytes, one per 4 elements][8 x u32: 4-bit scale | 4 x 7-bit sign index]
            const uint8_t* b = row + (size_t)(col >> 8) * 98;
            const uint32_t aux = le32(b + 66 + 4 * (i >> 5));
            const float db = mul(mul(half_to_f32(le16(b)), 0.5f + (float)(aux >> 28)), 0.5f);
            const int8_t g = tab[GRID_IQ3XXS + b[2 + (i >> 2)] * 4 + (i & 3)];
            return flip(mul(db, (float)g), signs[(aux >> (7 * ((i >> 3) & 3))) & 127], e);
        }
        case IQ3_S: {     // [d][64 grid low bytes][8 bytes of grid high bits][32 sign bytes][4 scale bytes]
            const uint8_t* b = row + (size_t)(col >> 8) * 110;
            const int g = i >> 5, k = i >> 2;
            const int sc = (b[106 + (g >> 1)] >> (4 * (g & 1))) & 15;
            const float db = mul(half_to_f32(le16(b)), (float)(2 * sc + 1));
            const int gi = b[2 + k] | (((b[66 + (k >> 3)] >> (k & 7)) & 1) << 8);
            return flip(mul(db, (float)tab[GRID_IQ3S + gi * 4 + (i & 3)]), b[74 + (i >> 3)], e);
        }
        case IQ1_S: {     // [d][32 grid low bytes][8 x u16: 3 x 3-bit grid highs, 3-bit scale, delta sign]
            const uint8_t* b = row + (size_t)(col >> 8) * 50;
            const int k = i >> 3;
            const uint32_t h = le16(b + 34 + 2 * (i >> 5));
            const float dl = mul(half_to_f32(le16(b)), (float)(2 * ((h >> 12) & 7) + 1));
            const float delta = (h & 0x8000u) ? -0.125f : 0.125f;
            const int gi = b[2 + k] | (((h >> (3 * (k & 3))) & 7) << 8);
            return mul(dl, (float)tab[GRID_IQ1S + gi * 8 + e] + delta);
        }
        case IQ1_M: {     // [32 grid low bytes][16 bytes: two (3-bit high, delta sign) nibbles][4 x u16 scales]
            const uint8_t* b = row + (size_t)(col >> 8) * 56;
            const uint8_t* sc = b + 48;
            const int k = i >> 3, s = i >> 4;
            // the block's fp16 scale is spread over the top nibbles of the four scale words
            const uint32_t dbits = (le16(sc) >> 12) | ((le16(sc + 2) >> 12) << 4) | ((le16(sc + 4) >> 12) << 8) |
                                   ((le16(sc + 6) >> 12) << 12);
            const int sub = (le16(sc + 2 * (s >> 2)) >> (3 * (s & 3))) & 7;
            const float dl = mul(half_to_f32(dbits), (float)(2 * sub + 1));
            const int nib = (b[32 + (k >> 1)] >> (4 * (k & 1))) & 15;
            const float delta = (nib & 8) ? -0.125f : 0.125f;
            const int gi = b[k] | ((nib & 7) << 8);
            return mul(dl, (float)tab[GRID_IQ1S + gi * 8 + e] + delta);
        }
        default: return 0.0f;
    }
}

}  // namespace tkq
