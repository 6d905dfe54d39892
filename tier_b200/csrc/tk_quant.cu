// tk_quant.cu -- GPU quantizers, byte-exact with the reference's CPU ones
// (tier/quant.h:124-204: q_f2h, q_nearest, q8_0_row, q_qkx2, qk_minmax_row,
// q_qx, q6_k_row; dispatched by q_row, tier/quant.h:201-204, as used by
// quant_main, tier/tier.cpp:2698-2746).
//
// Byte equality needs every floating-point operation of the reference, in
// its order and in fp32 with round-to-nearest: sums stay sequential, every
// product and sum is an explicitly rounded intrinsic (__fmul_rn, __fadd_rn,
// ...), so the compiler contracts nothing into an FMA, and divisions and the
// square root are the correctly rounded ones.  The parallelism is across
// blocks and across the independent searches inside a super-block:
//   Q8_0  one thread per 32-element block;
//   Q4_K / Q5_K  eight threads per super-block, one per 32-element sub-block
//         (its q_qkx2 search), the super-block RMS computed by each of the
//         eight in the reference's order, the packed scales built from all
//         eight by every thread;
//   Q6_K  sixteen threads per super-block, one per 16-element sub-block (q_qx).
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

// float -> fp16 bits, round to nearest even, as tier/quant.h:124-131 (q_f2h).
__device__ __forceinline__ uint16_t qf2h(float f) {
    const uint32_t u = __float_as_uint(f);
    const uint32_t s = (u >> 16) & 0x8000u;
    int e = (int)((u >> 23) & 0xff) - 127 + 15;
    uint32_t m = u & 0x7fffffu;
    if (((u >> 23) & 0xff) == 0xff) return (uint16_t)(s | 0x7c00u | (m ? 0x200u : 0u));
    if (e >= 31) return (uint16_t)(s | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)s;
        m |= 0x800000u;
        const int sh = 14 - e;
        uint32_t hm = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (hm & 1))) ++hm;
        return (uint16_t)(s | hm);
    }
    const uint32_t hm = m >> 13, rem = m & 0x1fffu;
    uint32_t h = s | ((uint32_t)e << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1))) ++h;
    return (uint16_t)h;
}
// tier/quant.h:133 (q_nearest): round half to even through 1.5 * 2^23.
__device__ __forceinline__ int qnearest(float f) {
    const float v = __fadd_rn(f, 12582912.f);
    return (int)(__float_as_uint(v) & 0x007fffffu) - 0x00400000;
}
__device__ __forceinline__ float qh2f(uint16_t h) { return h2f_bits(h); }   // exact

// ---------------------------------------------------------------- Q8_0 ----
__global__ void quant_q8_0_kernel(const float* __restrict__ x, long ldx, int rows, int cols, uint8_t* __restrict__ out,
                                  size_t rb) {
    const int nb = cols / 32;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)rows * nb) return;
    const int r = (int)(i / nb), b = (int)(i - (long)r * nb);
    const float* v = x + (size_t)r * ldx + b * 32;
    uint8_t* o = out + (size_t)r * rb + (size_t)b * 34;
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) {
        const float a = fabsf(v[j]);
        amax = amax < a ? a : amax;                               // std::max(amax, a)
    }
    const float d = __fdiv_rn(amax, 127.f), id = d != 0.0f ? __fdiv_rn(1.f, d) : 0.f;
    const uint16_t hd = qf2h(d);
    o[0] = (uint8_t)hd;
    o[1] = (uint8_t)(hd >> 8);
    for (int j = 0; j < 32; ++j) o[2 + j] = (uint8_t)(int8_t)roundf(__fmul_rn(v[j], id));
}

// --------------------------------------------------------- Q4_K / Q5_K ----
// tier/quant.h:138-152 (q_qkx2) for one 32-element sub-block.
__device__ float qkx2(int nmax, const float* x, const float* w, uint8_t* L, float* the_min, uint8_t* La, float rmin,
                      float rdelta, int nstep) {
    const int n = 32;
    float mn = x[0], mx = x[0], sw = w[0], sx = __fmul_rn(sw, x[0]);
    for (int i = 1; i < n; ++i) {
        if (x[i] < mn) mn = x[i];
        if (x[i] > mx) mx = x[i];
        sw = __fadd_rn(sw, w[i]);
        sx = __fadd_rn(sx, __fmul_rn(w[i], x[i]));
    }
    if (mn > 0) mn = 0;
    if (mx == mn) {
        for (int i = 0; i < n; ++i) L[i] = 0;
        *the_min = -mn;
        return 0.f;
    }
    float iscale = __fdiv_rn((float)nmax, __fsub_rn(mx, mn)), scale = __fdiv_rn(1.f, iscale), best = 0;
    for (int i = 0; i < n; ++i) {
        int l = qnearest(__fmul_rn(iscale, __fsub_rn(x[i], mn)));
        l = max(0, min(nmax, l));
        L[i] = (uint8_t)l;
        const float df = __fsub_rn(__fadd_rn(__fmul_rn(scale, (float)L[i]), mn), x[i]);
        best = __fadd_rn(best, __fmul_rn(__fmul_rn(w[i], df), df));
    }
    for (int is = 0; is <= nstep; ++is) {
        iscale = __fdiv_rn(__fadd_rn(__fadd_rn(rmin, __fmul_rn(rdelta, (float)is)), (float)nmax), __fsub_rn(mx, mn));
        float sl = 0, sl2 = 0, sxl = 0;
        for (int i = 0; i < n; ++i) {
            int l = qnearest(__fmul_rn(iscale, __fsub_rn(x[i], mn)));
            l = max(0, min(nmax, l));
            La[i] = (uint8_t)l;
            const float fl = (float)l;
            sl = __fadd_rn(sl, __fmul_rn(w[i], fl));
            sl2 = __fadd_rn(sl2, __fmul_rn(__fmul_rn(w[i], fl), fl));
            sxl = __fadd_rn(sxl, __fmul_rn(__fmul_rn(w[i], fl), x[i]));
        }
        const float D = __fsub_rn(__fmul_rn(sw, sl2), __fmul_rn(sl, sl));
        if (D > 0) {
            float ts = __fdiv_rn(__fsub_rn(__fmul_rn(sw, sxl), __fmul_rn(sx, sl)), D);
            float tm = __fdiv_rn(__fsub_rn(__fmul_rn(sl2, sx), __fmul_rn(sl, sxl)), D);
            if (tm > 0) {
                tm = 0;
                ts = __fdiv_rn(sxl, sl2);
            }
            float mad = 0;
            for (int i = 0; i < n; ++i) {
                const float df = __fsub_rn(__fadd_rn(__fmul_rn(ts, (float)La[i]), tm), x[i]);
                mad = __fadd_rn(mad, __fmul_rn(__fmul_rn(w[i], df), df));
            }
            if (mad < best) {
                for (int i = 0; i < n; ++i) L[i] = La[i];
                best = mad;
                scale = ts;
                mn = tm;
            }
        }
    }
    *the_min = -mn;
    return scale;
}

// tier/quant.h:154-173 (qk_minmax_row): 8 threads per super-block, thread j
// = sub-block j.  Blocks of 256 threads = 32 super-blocks.
template <bool Q5>
__global__ void __launch_bounds__(256) quant_qk_kernel(const float* __restrict__ x, long ldx, int rows, int cols,
                                                       uint8_t* __restrict__ out, size_t rb) {
    constexpr int NMAX = Q5 ? 31 : 15, BB = Q5 ? 176 : 144;
    __shared__ uint8_t Ls[32][256];
    const int nsb = cols / 256;
    const int gsb = threadIdx.x >> 3, j = threadIdx.x & 7;
    const long sbi = (long)blockIdx.x * 32 + gsb;
    const bool live = sbi < (long)rows * nsb;
    const int r = live ? (int)(sbi / nsb) : 0, b = live ? (int)(sbi - (long)r * nsb) : 0;
    const float* v = x + (size_t)r * ldx + (size_t)b * 256;
    uint8_t* L = Ls[gsb];
    float scale_j = 0.f, min_j = 0.f;
    if (live) {
        float s2 = 0;   // the reference's sequential sum of squares, by each of the eight
        for (int l = 0; l < 256; ++l) s2 = __fadd_rn(s2, __fmul_rn(v[l], v[l]));
        const float av = __fsqrt_rn(__fdiv_rn(s2, 256.f));
        float w[32], xs[32];
        uint8_t La[32];
        for (int l = 0; l < 32; ++l) {
            xs[l] = v[32 * j + l];
            w[l] = __fadd_rn(av, fabsf(xs[l]));
        }
        scale_j = qkx2(NMAX, xs, w, L + 32 * j, &min_j, La, -0.5f * (Q5 ? 1 : 2), 0.1f, Q5 ? 15 : 20);
    }
    // max over the eight (max is order-free; the reference starts from 0)
    const unsigned gm = 0xffu << (8 * ((threadIdx.x & 31) >> 3));
    float ms = fmaxf(0.f, scale_j), mm = fmaxf(0.f, min_j);
    // std::max(ms, scales[j]) keeps ms when unordered; scales are finite here
    for (int o = 1; o < 8; o <<= 1) {
        ms = fmaxf(ms, __shfl_xor_sync(gm, ms, o));
        mm = fmaxf(mm, __shfl_xor_sync(gm, mm, o));
    }
    const float is = ms > 0 ? __fdiv_rn(63.f, ms) : 0.f, im = mm > 0 ? __fdiv_rn(63.f, mm) : 0.f;
    const int ls = min(63, qnearest(__fmul_rn(is, scale_j))), lm = min(63, qnearest(__fmul_rn(im, min_j)));
    int lsa[8], lma[8];
    for (int k = 0; k < 8; ++k) {
        lsa[k] = __shfl_sync(gm, ls, (threadIdx.x & 24) + k);
        lma[k] = __shfl_sync(gm, lm, (threadIdx.x & 24) + k);
    }
    uint8_t sc[12];
    for (int k = 0; k < 12; ++k) sc[k] = 0;
    for (int k = 0; k < 8; ++k) {
        if (k < 4) {
            sc[k] = (uint8_t)lsa[k];
            sc[k + 4] = (uint8_t)lma[k];
        } else {
            sc[k + 4] = (uint8_t)((lsa[k] & 0xF) | ((lma[k] & 0xF) << 4));
            sc[k - 4] |= (uint8_t)((lsa[k] >> 4) << 6);
            sc[k] |= (uint8_t)((lma[k] >> 4) << 6);
        }
    }
    const uint16_t hd = qf2h(__fdiv_rn(ms, 63.f)), hm = qf2h(__fdiv_rn(mm, 63.f));
    if (live) {
        int s, m;   // q4k_scale_min of the packed bytes (tier/quant.h:47-48)
        if (j < 4) { s = sc[j] & 63; m = sc[j + 4] & 63; }
        else { s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4); m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4); }
        const float d = __fmul_rn(qh2f(hd), (float)s);
        if (d != 0.0f) {
            const float dm = __fmul_rn(qh2f(hm), (float)m);
            for (int ii = 0; ii < 32; ++ii) {
                const int l = qnearest(__fdiv_rn(__fadd_rn(v[32 * j + ii], dm), d));
                L[32 * j + ii] = (uint8_t)max(0, min(NMAX, l));
            }
        }
    }
    __syncwarp();
    if (!live) return;
    uint8_t* o = out + (size_t)r * rb + (size_t)b * BB;
    if (j == 0) {
        o[0] = (uint8_t)hd; o[1] = (uint8_t)(hd >> 8);
        o[2] = (uint8_t)hm; o[3] = (uint8_t)(hm >> 8);
        for (int k = 0; k < 12; ++k) o[4 + k] = sc[k];
    }
    if constexpr (!Q5) {
        // 128 bytes: byte 16 + 32p + l = low nibble L[64p + l], high L[64p + l + 32]
        for (int t = 16 * j; t < 16 * j + 16; ++t) {
            const int p = t >> 5, l = t & 31;
            o[16 + t] = (uint8_t)((L[64 * p + l] & 15) | ((L[64 * p + l + 32] & 15) << 4));
        }
    } else {
        // qh[32] at 16, ql[128] at 48; thread j takes qh bytes 4j .. 4j+3
        for (int jj = 4 * j; jj < 4 * j + 4; ++jj) {
            uint8_t qh = 0;
            for (int p = 0; p < 4; ++p) {
                int l1 = L[64 * p + jj], l2 = L[64 * p + jj + 32];
                if (l1 > 15) { l1 -= 16; qh |= (uint8_t)(1 << (2 * p)); }
                if (l2 > 15) { l2 -= 16; qh |= (uint8_t)(2 << (2 * p)); }
                o[48 + 32 * p + jj] = (uint8_t)(l1 | (l2 << 4));
            }
            o[16 + jj] = qh;
        }
    }
}

// ---------------------------------------------------------------- Q6_K ----
// tier/quant.h:175-185 (q_qx) for one 16-element sub-block, nmax = 32.
__device__ float qqx(const float* x, int8_t* L) {
    const int n = 16, nmax = 32;
    float amax = 0, mx = 0;
    for (int i = 0; i < n; ++i) {
        const float a = fabsf(x[i]);
        if (a > amax) { amax = a; mx = x[i]; }
    }
    if (amax < 1e-15f) {
        for (int i = 0; i < n; ++i) L[i] = 0;
        return 0.f;
    }
    float iscale = __fdiv_rn((float)(-nmax), mx), sumlx = 0, suml2 = 0;
    for (int i = 0; i < n; ++i) {
        int l = qnearest(__fmul_rn(iscale, x[i]));
        l = max(-nmax, min(nmax - 1, l));
        L[i] = (int8_t)(l + nmax);
        const float w = __fmul_rn(x[i], x[i]);
        sumlx = __fadd_rn(sumlx, __fmul_rn(__fmul_rn(w, x[i]), (float)l));
        suml2 = __fadd_rn(suml2, __fmul_rn(__fmul_rn(w, (float)l), (float)l));
    }
    float scale = suml2 > 0 ? __fdiv_rn(sumlx, suml2) : 0.f, best = __fmul_rn(scale, sumlx);
    for (int is = -9; is <= 9; ++is) {
        if (!is) continue;
        iscale = __fdiv_rn(-__fadd_rn((float)nmax, __fmul_rn(0.1f, (float)is)), mx);
        sumlx = suml2 = 0;
        for (int i = 0; i < n; ++i) {
            int l = qnearest(__fmul_rn(iscale, x[i]));
            l = max(-nmax, min(nmax - 1, l));
            const float w = __fmul_rn(x[i], x[i]);
            sumlx = __fadd_rn(sumlx, __fmul_rn(__fmul_rn(w, x[i]), (float)l));
            suml2 = __fadd_rn(suml2, __fmul_rn(__fmul_rn(w, (float)l), (float)l));
        }
        if (suml2 > 0 && __fmul_rn(sumlx, sumlx) > __fmul_rn(best, suml2)) {
            for (int i = 0; i < n; ++i) {
                const int l = qnearest(__fmul_rn(iscale, x[i]));
                L[i] = (int8_t)(nmax + max(-nmax, min(nmax - 1, l)));
            }
            scale = __fdiv_rn(sumlx, suml2);
            best = __fmul_rn(scale, sumlx);
        }
    }
    return scale;
}

// tier/quant.h:186-199 (q6_k_row): 16 threads per super-block; blocks of 256
// threads = 16 super-blocks.
__global__ void __launch_bounds__(256) quant_q6_k_kernel(const float* __restrict__ x, long ldx, int rows, int cols,
                                                        uint8_t* __restrict__ out, size_t rb) {
    __shared__ int8_t Ls[16][256];
    const int nsb = cols / 256;
    const int gsb = threadIdx.x >> 4, j = threadIdx.x & 15;
    const long sbi = (long)blockIdx.x * 16 + gsb;
    const bool live = sbi < (long)rows * nsb;
    const int r = live ? (int)(sbi / nsb) : 0, b = live ? (int)(sbi - (long)r * nsb) : 0;
    const float* v = x + (size_t)r * ldx + (size_t)b * 256;
    int8_t* L = Ls[gsb];
    float sj = 0.f;
    if (live) {
        float xs[16];
        for (int l = 0; l < 16; ++l) xs[l] = v[16 * j + l];
        sj = qqx(xs, L + 16 * j);
    }
    const unsigned gm = 0xffffu << (16 * ((threadIdx.x & 31) >> 4));
    // the first sub-block (in order) of largest |scale|, as the reference's loop
    float sc_all[16];
    for (int k = 0; k < 16; ++k) sc_all[k] = __shfl_sync(gm, sj, (threadIdx.x & 16) + k);
    float ma = 0, ms = 0;
    for (int k = 0; k < 16; ++k) {
        const float a = fabsf(sc_all[k]);
        if (a > ma) { ma = a; ms = sc_all[k]; }
    }
    __syncwarp();
    if (!live) return;
    uint8_t* o = out + (size_t)r * rb + (size_t)b * 210;
    if (ma < 1e-15f) {   // the reference leaves the zeroed block
        for (int t = j; t < 210; t += 16) o[t] = 0;
        return;
    }
    const float is = __fdiv_rn(-128.f, ms);
    const uint16_t hd = qf2h(__fdiv_rn(1.f, is));
    const int8_t scj = (int8_t)min(127, qnearest(__fmul_rn(is, sj)));
    const float d = __fmul_rn(qh2f(hd), (float)scj);
    if (d != 0.0f) {
        for (int ii = 0; ii < 16; ++ii) {
            const int l = qnearest(__fdiv_rn(v[16 * j + ii], d));
            L[16 * j + ii] = (int8_t)(max(-32, min(31, l)) + 32);
        }
    }
    __syncwarp(gm);   // this super-block's 16 lanes (the others may have returned)
    o[192 + j] = (uint8_t)scj;
    if (j == 0) { o[208] = (uint8_t)hd; o[209] = (uint8_t)(hd >> 8); }
    // ql[128] at 0, qh[64] at 128: thread j takes l = 2j, 2j+1 of each half
    for (int h = 0; h < 2; ++h) {
        const int jb = 128 * h;
        for (int l = 2 * j; l < 2 * j + 2; ++l) {
            const int q1 = L[jb + l] & 15, q2 = L[jb + l + 32] & 15, q3 = L[jb + l + 64] & 15, q4 = L[jb + l + 96] & 15;
            o[64 * h + l] = (uint8_t)(q1 | (q3 << 4));
            o[64 * h + l + 32] = (uint8_t)(q2 | (q4 << 4));
            o[128 + 32 * h + l] = (uint8_t)((L[jb + l] >> 4) | ((L[jb + l + 32] >> 4) << 2) |
                                            ((L[jb + l + 64] >> 4) << 4) | ((L[jb + l + 96] >> 4) << 6));
        }
    }
}

// bf16 rows -> fp32 rows (exact), for quantizing bf16 sources like quant_main.
__global__ void bf16_to_f32_kernel(const uint16_t* __restrict__ src, long lds, int rows, int cols, float* dst) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)rows * cols) return;
    const int r = (int)(i / cols), c = (int)(i - (long)r * cols);
    dst[i] = __uint_as_float((uint32_t)src[(size_t)r * lds + c] << 16);
}

tk_status launch_quantize(tk_ctx* ctx, int qtype, const float* x, long ldx, int rows, int cols, uint8_t* out,
                          size_t rb, cudaStream_t s) {
    ProfScope ps(ctx, s, PK_DEQUANT);
    if (qtype == QT_Q8_0) {
        const long n = (long)rows * (cols / 32);
        quant_q8_0_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(x, ldx, rows, cols, out, rb);
    } else if (qtype == QT_Q4_K || qtype == QT_Q5_K) {
        const long n = (long)rows * (cols / 256);
        const unsigned g = (unsigned)((n + 31) / 32);
        if (qtype == QT_Q4_K) quant_qk_kernel<false><<<g, 256, 0, s>>>(x, ldx, rows, cols, out, rb);
        else quant_qk_kernel<true><<<g, 256, 0, s>>>(x, ldx, rows, cols, out, rb);
    } else if (qtype == QT_Q6_K) {
        const long n = (long)rows * (cols / 256);
        quant_q6_k_kernel<<<(unsigned)((n + 15) / 16), 256, 0, s>>>(x, ldx, rows, cols, out, rb);
    } else {
        return fail(TK_ERR_UNSUPPORTED, "tk_quantize: type " + std::to_string(qtype) +
                                            " (the reference quantizes to Q8_0, Q4_K, Q5_K, Q6_K)");
    }
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "quantize launch");
}

tk_status launch_bf16_to_f32(tk_ctx* ctx, const uint16_t* src, long lds, int rows, int cols, float* dst, cudaStream_t s) {
    const long n = (long)rows * cols;
    bf16_to_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src, lds, rows, cols, dst);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "bf16 widen launch");
}

}  // namespace tk
