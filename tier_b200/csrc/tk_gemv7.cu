// tk_gemv7.cu -- decode GEMV for 3..16 tokens on the integer tensor cores
// (mma.sync s8 x s8 -> s32) for Q8_0 / Q4_K / Q5_K / Q6_K rows, reading W once.
//
// x of 16 tokens at K = 14336 does not fit shared memory next to a weight
// ring, so x travels with the weight instead:
//
//  * A pre-pass (gw_xrec_kernel) turns x into records, one per 256-element
//    chunk: every token is scaled by a power of two (its max into [2^21,
//    2^22)) and split exactly into three signed bytes, xi = p0 * 2^16 + p1 *
//    2^8 + p2, as in tk_gemv6.cu.  A record holds the plane rows (row p * 8H +
//    token, H = 1 or 2 halves of 8 tokens, 288-byte rows so 64-bit fragment
//    loads are bank-conflict-free), one float scale per row (2^-s * 2^(16-8p))
//    and the x sums of each 32-element block per row (int16), for the K-quant
//    min term.  Rows of tokens >= M are zero.
//  * The GEMV streams (16-row group, K-chunk) slots: the weight rows of the
//    chunk and, in the same slot, the chunk's x records (one bulk copy; the
//    records stay in L2 across the SM's row groups).
//  * H teams of 16 / H warps: team h takes tokens 8h .. 8h+7 of every slot, so
//    the MMA's 8 columns are 8 tokens of one plane and the three planes of a
//    token land in the same lane: each plane's product is scaled and added into
//    the same fp32 accumulator.  The warps of a team split the slot's 64-element
//    units (Q8_0 block pairs, K-quant sub-block pairs); at the end of a row group
//    the team sums its warps' partials in a fixed order.
//  * Per unit and plane: Q8_0 one m16n8k32 MMA per block, times d; Q4_K / Q5_K
//    one per 32-element sub-block, times its 6-bit sc in int32, minus m times
//    the block's x sum, then d and dmin in fp32; Q6_K one m16n8k16 MMA per
//    16-element sub-block, times its int8 sc, then d.
// Agreement with fp64 is ~1e-7 relative.  A non-finite x element makes its
// token's y non-finite (the chunk's scale is NaN).
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

constexpr int GW_CW = 16;                        // consumer warps
constexpr int GW_THREADS = (GW_CW + 1) * 32;     // + one producer warp
constexpr int GW_MAXSLOTS = 8;
constexpr size_t GW_SMEM_MAX = 220 * 1024;
constexpr int GW_XROW = 288;                     // plane row bytes in a record (256 used; 32 mod 128)

// record of one 256-element chunk with `rows` = 24 H plane rows:
//   [rows][288] int8 planes | [rows] float scales | [8 blocks][rows] int16 x sums
__host__ __device__ constexpr int gw_rows(int nh) { return 24 * nh; }
__host__ __device__ constexpr int gw_rec_bytes(int nh) { return gw_rows(nh) * (GW_XROW + 4 + 16); }

struct GwArgs {
    const uint8_t* W;
    size_t rb;
    int N, K, M;
    const uint8_t* xr;   // records (K / 256 of them)
    float* y;
    int ldy;
    int KC;              // elements per K-chunk (slot)
    int nchunks;
    uint32_t kcb;        // weight bytes per row per chunk
    uint32_t RS;         // per-row slot stride (one copy per row)
    uint32_t CS;         // nonzero: four copies of 4 whole rows at CS-byte strides
    uint32_t xoff;       // offset of the x records in a slot
    int nslots;
    int* status;
};

__device__ __forceinline__ uint32_t w_lds16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t w_lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 w_lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float2 w_lds64f(uint32_t a) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 w_lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
// D = A (16 x 32, s8) * B (32 x 8, s8), s32, accumulator input zero
__device__ __forceinline__ void wmma32z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    const int z = 0;
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(z));
}
// D = A (16 x 16, s8) * B (16 x 8, s8), s32, accumulator input zero
__device__ __forceinline__ void wmma16z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    const int z = 0;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%7, %7, %7, %7};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(z));
}
// 32-bit load at an address that is 4-byte aligned or (odd) 2 mod 4 (Q6_K
// super-blocks are 210 bytes)
__device__ __forceinline__ uint32_t w_lds32_a(uint32_t a, bool odd) {
    if (!odd) return w_lds32(a);
    return __funnelshift_r(w_lds32(a - 2u), w_lds32(a + 2u), 16);
}
// int -> float, exact for |v| < 2^22: v added to the mantissa of 1.5 * 2^23
__device__ __forceinline__ float w_i2f22(int v) { return __int_as_float(v + 0x4B400000) - 12582912.0f; }
__device__ __forceinline__ int w_ubyte(uint32_t w, int k) { return (int)__byte_perm(w, 0u, 0x4440u | (uint32_t)k); }
__device__ __forceinline__ float w_h2f(uint32_t h) { return __half2float(__ushort_as_half((uint16_t)(h & 0xffffu))); }

// ---------------------------------------------------------------------------
// pre-pass: x [M, K] fp32 -> K / 256 records.  One warp per (token row, chunk);
// lane l takes elements 8l .. 8l+7 of the chunk.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gw_xrec_kernel(const float* __restrict__ x, int ldx, int M, int K, int nh,
                                                      uint8_t* __restrict__ rec) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int task = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int nc = K / 256, toks = 8 * nh, rows = 24 * nh;
    if (task >= toks * nc) return;
    const int m = task / nc, c = task - m * nc;
    uint8_t* r = rec + (size_t)c * gw_rec_bytes(nh);
    float* scl = reinterpret_cast<float*>(r + (size_t)rows * GW_XROW);
    int16_t* xs = reinterpret_cast<int16_t*>(r + (size_t)rows * (GW_XROW + 4));
    uint32_t w0[2] = {0u, 0u}, w1[2] = {0u, 0u}, w2[2] = {0u, 0u};
    int s0 = 0, s1 = 0, s2 = 0, s = 0;
    bool nonfin = false;
    if (m < M) {
        const float4* src = reinterpret_cast<const float4*>(x + (size_t)m * ldx + c * 256 + 8 * lane);
        const float4 v0 = __ldg(src), v1 = __ldg(src + 1);
        float mx = fmaxf(fmaxf(fmaxf(fabsf(v0.x), fabsf(v0.y)), fmaxf(fabsf(v0.z), fabsf(v0.w))),
                         fmaxf(fmaxf(fabsf(v1.x), fabsf(v1.y)), fmaxf(fabsf(v1.z), fabsf(v1.w))));
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // a non-finite x element makes the chunk's scale NaN, so y comes out
        // non-finite as the reference's fp32 sum does; its planes are zero
        nonfin = __any_sync(0xffffffffu, !(isfinite(v0.x) && isfinite(v0.y) && isfinite(v0.z) && isfinite(v0.w) &&
                                           isfinite(v1.x) && isfinite(v1.y) && isfinite(v1.z) && isfinite(v1.w)));
        if (mx > 0.0f) {
            // mx in [2^(E-127), 2^(E-126)): mx * 2^s in [2^21, 2^22); s >= -106 for finite mx
            s = 148 - (int)((__float_as_uint(mx) >> 23) & 0xffu);
            if (s > 127) s = 127;
        }
        const float up = nonfin ? 0.0f : __uint_as_float((uint32_t)(127 + s) << 23);
        const float f[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int xi = __float2int_rn(f[k] * up);      // |xi| < 2^22
            const int b2 = (int)((uint32_t)xi << 24) >> 24;
            const int r1 = (xi - b2) >> 8;
            const int b1 = (int)((uint32_t)r1 << 24) >> 24;
            const int b0 = (r1 - b1) >> 8;                 // |b0| <= 64
            s0 += b0;
            s1 += b1;
            s2 += b2;
            w0[k >> 2] |= ((uint32_t)b0 & 0xffu) << (8 * (k & 3));
            w1[k >> 2] |= ((uint32_t)b1 & 0xffu) << (8 * (k & 3));
            w2[k >> 2] |= ((uint32_t)b2 & 0xffu) << (8 * (k & 3));
        }
    }
    *reinterpret_cast<uint2*>(r + (size_t)(0 * toks + m) * GW_XROW + 8 * lane) = make_uint2(w0[0], w0[1]);
    *reinterpret_cast<uint2*>(r + (size_t)(1 * toks + m) * GW_XROW + 8 * lane) = make_uint2(w1[0], w1[1]);
    *reinterpret_cast<uint2*>(r + (size_t)(2 * toks + m) * GW_XROW + 8 * lane) = make_uint2(w2[0], w2[1]);
    if (lane < 3) scl[lane * toks + m] = m >= M ? 0.0f : nonfin ? __uint_as_float(0x7fc00000u) : ldexpf(1.0f, 16 - 8 * lane - s);
    // x sums of each 32-element block (4 lanes)
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        s0 += __shfl_xor_sync(0xffffffffu, s0, o);
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if ((lane & 3) == 0) {
        const int b = lane >> 2;
        xs[b * rows + 0 * toks + m] = (int16_t)s0;
        xs[b * rows + 1 * toks + m] = (int16_t)s1;
        xs[b * rows + 2 * toks + m] = (int16_t)s2;
    }
}

template <int T, int NH>
__global__ void __launch_bounds__(GW_THREADS, 1) gemv_wide_kernel(const __grid_constant__ GwArgs a) {
    constexpr int TOKS = 8 * NH, ROWS = 24 * NH, REC = gw_rec_bytes(NH);
    constexpr int TW = GW_CW / NH;                  // warps per team
    extern __shared__ uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const uint32_t slot_bytes = a.xoff + (uint32_t)(a.KC / 256) * REC;
    uint8_t* ring = sm;
    float* part = reinterpret_cast<float*>(ring + (size_t)a.nslots * slot_bytes);   // [team][2][TW][16][8]
    uint64_t* full = reinterpret_cast<uint64_t*>(part + 2 * GW_CW * 128);
    uint64_t* empty = full + a.nslots;

    const int r_begin = (int)((long long)a.N * blockIdx.x / gridDim.x);
    const int r_end = (int)((long long)a.N * (blockIdx.x + 1) / gridDim.x);
    const int nrows = r_end - r_begin;
    const int ngroups = (nrows + 15) / 16;
    const int nslot_total = ngroups * a.nchunks;

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (int i = 0; i < a.nslots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], GW_CW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    // the x records come from the kernel just before (and W may be written by
    // earlier ones): nothing is read before it completes
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp == GW_CW) {
        // ---------------- producer: weight rows + the chunk's x records per slot ----------------
        bool ok = true;
        int slot = 0, issued = 0;
        const uint32_t xbytes = (uint32_t)(a.KC / 256) * REC;
        for (int s = 0; s < nslot_total; ++s) {
            const int grp = s / a.nchunks, c = s - grp * a.nchunks;
            const int row0 = r_begin + grp * 16;
            const int nv = r_end - row0 < 16 ? r_end - row0 : 16;
            if (lane == 0) {
                if (ok && s >= a.nslots)
                    ok = mbar_wait(&empty[slot], (uint32_t)((s / a.nslots) - 1) & 1u, a.status);
                if (ok) mbar_arrive_expect_tx(&full[slot], (uint32_t)nv * a.kcb + xbytes);
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            uint8_t* sb = ring + (size_t)slot * slot_bytes;
            if (a.CS) {
                if (lane < 4 && 4 * lane < nv) {
                    const int nr = nv - 4 * lane < 4 ? nv - 4 * lane : 4;
                    bulk_load(sb + (size_t)lane * a.CS, a.W + (size_t)(row0 + 4 * lane) * a.rb, (uint32_t)nr * a.kcb,
                              &full[slot]);
                }
            } else if (lane < nv) {
                bulk_load(sb + (size_t)lane * a.RS, a.W + (size_t)(row0 + lane) * a.rb + (size_t)c * a.kcb, a.kcb,
                          &full[slot]);
            }
            if (lane == 31) bulk_load(sb + a.xoff, a.xr + (size_t)c * xbytes, xbytes, &full[slot]);
            issued = s + 1;
            if (++slot == a.nslots) slot = 0;
        }
        if (!ok && lane == 0) {
            // copies already issued land before the block exits (bounded): the
            // last nslots uses issued (earlier ones were consumed before reuse)
            const int first = issued > a.nslots ? issued - a.nslots : 0;
            for (int s = first; s < issued; ++s)
                (void)mbar_wait(&full[s % a.nslots], (uint32_t)(s / a.nslots) & 1u, a.status);
        }
        return;
    }

    // ---------------- consumers: team h = tokens 8h .. 8h+7 of every slot ----------------
    const int team = warp / TW, tw = warp - team * TW;
    const uint32_t offA = a.CS ? (uint32_t)(g & 3) * a.CS + (uint32_t)(g >> 2) * a.kcb : (uint32_t)g * a.RS;
    const uint32_t offB = a.CS ? (uint32_t)(g & 3) * a.CS + (uint32_t)(2 + (g >> 2)) * a.kcb : (uint32_t)(g + 8) * a.RS;
    // x record offsets: B column g = token 8 team + g of plane p (row p * TOKS + 8 team + g);
    // this lane's output columns 2q, 2q+1 = tokens 8 team + 2q, +1
    const uint32_t xb_row = (uint32_t)(8 * team + g) * GW_XROW + 8u * q;       // + p * TOKS * 288
    const uint32_t cs_col = (uint32_t)ROWS * GW_XROW + (uint32_t)(8 * team + 2 * q) * 4u;   // + p * TOKS * 4
    const uint32_t sx_col = (uint32_t)ROWS * (GW_XROW + 4) + (uint32_t)(8 * team + 2 * q) * 2u;   // + (b * ROWS + p * TOKS) * 2
    const uint32_t ring_u = smem_u32(ring);

    int slot = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int grp = 0; grp < ngroups; ++grp) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};     // rows g, g+8 x tokens 2q, 2q+1 (of the team's half)
        for (int c = 0; c < a.nchunks; ++c) {
            if (ok) {
                const bool w = mbar_wait(&full[slot], ph, a.status);
                ok = __all_sync(0xffffffffu, w);
            }
            if (ok) {
                const uint32_t sbase = ring_u + (uint32_t)slot * slot_bytes;
                const uint32_t rA = sbase + offA, rB = sbase + offB;
                const uint32_t xbase = sbase + a.xoff;
                const int nunits = a.KC / 64;
                for (int u = tw; u < nunits; u += TW) {
                    const uint32_t rec = xbase + (uint32_t)(u >> 2) * REC;      // record of this unit
                    const uint32_t eo = 64u * (uint32_t)(u & 3);              // element offset in the record
                    if constexpr (T == QT_Q8_0) {
                        // block pair u: the even block's quants start at 2 mod 4, the odd one's at 0 mod 4
                        const uint32_t pA = rA + 68u * u, pB = rB + 68u * u;
                        const uint32_t oe = 8u * q;
                        const uint32_t a0w = w_lds32(pA + oe), a1w = w_lds32(pA + oe + 4), a2w = w_lds32(pA + oe + 8);
                        const uint32_t b0w = w_lds32(pB + oe), b1w = w_lds32(pB + oe + 4), b2w = w_lds32(pB + oe + 8);
                        const uint32_t aE0 = __funnelshift_r(a0w, a1w, 16), aE2 = __funnelshift_r(a1w, a2w, 16);
                        const uint32_t bE0 = __funnelshift_r(b0w, b1w, 16), bE2 = __funnelshift_r(b1w, b2w, 16);
                        const uint32_t oo = 36u + 8u * q;
                        const uint32_t aO0 = w_lds32(pA + oo), aO2 = w_lds32(pA + oo + 4);
                        const uint32_t bO0 = w_lds32(pB + oo), bO2 = w_lds32(pB + oo + 4);
                        const float dAe = w_h2f(w_lds16(pA)), dBe = w_h2f(w_lds16(pB));
                        const float dAo = w_h2f(w_lds16(pA + 34u)), dBo = w_h2f(w_lds16(pB + 34u));
#pragma unroll
                        for (int p = 0; p < 3; ++p) {
                            const uint32_t xr = rec + (uint32_t)(p * TOKS) * GW_XROW + xb_row + eo;
                            const uint2 xe = w_lds64(xr), xo = w_lds64(xr + 32u);
                            int ce[4], co[4];
                            wmma32z(ce, aE0, bE0, aE2, bE2, xe.x, xe.y);
                            wmma32z(co, aO0, bO0, aO2, bO2, xo.x, xo.y);
                            const float2 sc = w_lds64f(rec + cs_col + (uint32_t)(p * TOKS) * 4u);
                            acc[0] = fmaf(sc.x, fmaf(dAo, w_i2f22(co[0]), dAe * w_i2f22(ce[0])), acc[0]);
                            acc[1] = fmaf(sc.y, fmaf(dAo, w_i2f22(co[1]), dAe * w_i2f22(ce[1])), acc[1]);
                            acc[2] = fmaf(sc.x, fmaf(dBo, w_i2f22(co[2]), dBe * w_i2f22(ce[2])), acc[2]);
                            acc[3] = fmaf(sc.y, fmaf(dBo, w_i2f22(co[3]), dBe * w_i2f22(ce[3])), acc[3]);
                        }
                    } else if constexpr (T == QT_Q6_K) {
                        // Q6_K (tier/quant.h:88-90): unit u is elements 64j .. 64j+63 of
                        // super-block u / 4, i.e. 16-element sub-blocks 4j+t (t < 4), one
                        // m16n8k16 MMA each; thread q takes elements 4q .. 4q+3 of each.
                        // In half ha = j / 2: ql bytes 64ha + 16t + 4q (nibble j & 1), qh
                        // bytes 128 + 32ha + 16 (t & 1) + 4q (bits 2 (2 (j & 1) + t / 2)).
                        const int j = u & 3, sbi = u >> 2, ha = j >> 1, nb = j & 1;
                        const uint32_t sA = rA + 210u * (uint32_t)sbi, sB = rB + 210u * (uint32_t)sbi;
                        const bool odd = (sbi & 1) != 0;
                        const uint32_t scwA = w_lds32_a(sA + 192u + 4u * j, odd), scwB = w_lds32_a(sB + 192u + 4u * j, odd);
                        const float dA = w_h2f(w_lds16(sA + 208u)), dB = w_h2f(w_lds16(sB + 208u));
                        uint32_t vA[4], vB[4];
                        {
                            const uint32_t hA0 = w_lds32_a(sA + 128u + 32u * ha + 4u * q, odd);
                            const uint32_t hA1 = w_lds32_a(sA + 128u + 32u * ha + 16u + 4u * q, odd);
                            const uint32_t hB0 = w_lds32_a(sB + 128u + 32u * ha + 4u * q, odd);
                            const uint32_t hB1 = w_lds32_a(sB + 128u + 32u * ha + 16u + 4u * q, odd);
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                const uint32_t o = 64u * ha + 16u * t + 4u * q;
                                const int sh = 2 * (2 * nb + (t >> 1));
                                const uint32_t uA = ((w_lds32_a(sA + o, odd) >> (4 * nb)) & 0x0F0F0F0Fu) |
                                                    ((((t & 1) ? hA1 : hA0) >> sh) & 0x03030303u) << 4;
                                const uint32_t uB = ((w_lds32_a(sB + o, odd) >> (4 * nb)) & 0x0F0F0F0Fu) |
                                                    ((((t & 1) ? hB1 : hB0) >> sh) & 0x03030303u) << 4;
                                // bytes u - 32 (u < 64): no borrow crosses a byte
                                vA[t] = ((uA | 0x80808080u) - 0x20202020u) ^ 0x80808080u;
                                vB[t] = ((uB | 0x80808080u) - 0x20202020u) ^ 0x80808080u;
                            }
                        }
#pragma unroll
                        for (int p = 0; p < 3; ++p) {
                            // + 16 t: thread q's x bytes 4q .. 4q+3 of sub-block t
                            const uint32_t xr = rec + (uint32_t)(p * TOKS) * GW_XROW + xb_row - 4u * q + eo;
                            int I1[4] = {0, 0, 0, 0};
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                int cc[4];
                                wmma16z(cc, vA[t], vB[t], w_lds32(xr + 16u * t));
                                const int sa = (int)(scwA << (24 - 8 * t)) >> 24, sb = (int)(scwB << (24 - 8 * t)) >> 24;
                                I1[0] += sa * cc[0];
                                I1[1] += sa * cc[1];
                                I1[2] += sb * cc[2];
                                I1[3] += sb * cc[3];
                            }
                            const float2 sc = w_lds64f(rec + cs_col + (uint32_t)(p * TOKS) * 4u);
                            acc[0] = fmaf(sc.x, dA * __int2float_rn(I1[0]), acc[0]);
                            acc[1] = fmaf(sc.y, dA * __int2float_rn(I1[1]), acc[1]);
                            acc[2] = fmaf(sc.x, dB * __int2float_rn(I1[2]), acc[2]);
                            acc[3] = fmaf(sc.y, dB * __int2float_rn(I1[3]), acc[3]);
                        }
                    } else {
                        // Q4_K / Q5_K: unit u is sub-blocks 2j, 2j+1 of super-block u / 4
                        // (tier/quant.h:83-87; sc / m packing tier/quant.h:47-48)
                        constexpr uint32_t SB = T == QT_Q4_K ? 144u : 176u;
                        constexpr uint32_t QS = T == QT_Q4_K ? 16u : 48u;
                        const int j = u & 3;
                        const uint32_t sA = rA + SB * (uint32_t)(u >> 2), sB = rB + SB * (uint32_t)(u >> 2);
                        const uint4 hA = w_lds128(sA), hB = w_lds128(sB);
                        // 6-bit sc / m of sub-blocks 2j, 2j+1 (bytes of the packed words)
                        const uint32_t scA = j < 2 ? (hA.y & 0x3F3F3F3Fu)
                                                   : ((hA.w & 0x0F0F0F0Fu) | ((hA.y >> 2) & 0x30303030u));
                        const uint32_t mA = j < 2 ? (hA.z & 0x3F3F3F3Fu)
                                                  : (((hA.w >> 4) & 0x0F0F0F0Fu) | ((hA.z >> 2) & 0x30303030u));
                        const uint32_t scB = j < 2 ? (hB.y & 0x3F3F3F3Fu)
                                                   : ((hB.w & 0x0F0F0F0Fu) | ((hB.y >> 2) & 0x30303030u));
                        const uint32_t mB = j < 2 ? (hB.z & 0x3F3F3F3Fu)
                                                  : (((hB.w >> 4) & 0x0F0F0F0Fu) | ((hB.z >> 2) & 0x30303030u));
                        const int k0 = (2 * j) & 3, k1 = (2 * j + 1) & 3;
                        const int sAl = w_ubyte(scA, k0), sAh = w_ubyte(scA, k1), mAl = w_ubyte(mA, k0), mAh = w_ubyte(mA, k1);
                        const int sBl = w_ubyte(scB, k0), sBh = w_ubyte(scB, k1), mBl = w_ubyte(mB, k0), mBh = w_ubyte(mB, k1);
                        const float dA = w_h2f(hA.x), dmA = w_h2f(hA.x >> 16);
                        const float dB = w_h2f(hB.x), dmB = w_h2f(hB.x >> 16);
                        const uint2 wA = w_lds64(sA + QS + 32u * j + 8u * q), wB = w_lds64(sB + QS + 32u * j + 8u * q);
                        uint32_t lA0 = wA.x & 0x0F0F0F0Fu, lA2 = wA.y & 0x0F0F0F0Fu;
                        uint32_t lB0 = wB.x & 0x0F0F0F0Fu, lB2 = wB.y & 0x0F0F0F0Fu;
                        uint32_t hA0 = (wA.x >> 4) & 0x0F0F0F0Fu, hA2 = (wA.y >> 4) & 0x0F0F0F0Fu;
                        uint32_t hB0 = (wB.x >> 4) & 0x0F0F0F0Fu, hB2 = (wB.y >> 4) & 0x0F0F0F0Fu;
                        if constexpr (T == QT_Q5_K) {
                            const uint2 qhA = w_lds64(sA + 16u + 8u * q), qhB = w_lds64(sB + 16u + 8u * q);
                            lA0 |= ((qhA.x >> (2 * j)) & 0x01010101u) << 4;
                            lA2 |= ((qhA.y >> (2 * j)) & 0x01010101u) << 4;
                            lB0 |= ((qhB.x >> (2 * j)) & 0x01010101u) << 4;
                            lB2 |= ((qhB.y >> (2 * j)) & 0x01010101u) << 4;
                            hA0 |= ((qhA.x >> (2 * j + 1)) & 0x01010101u) << 4;
                            hA2 |= ((qhA.y >> (2 * j + 1)) & 0x01010101u) << 4;
                            hB0 |= ((qhB.x >> (2 * j + 1)) & 0x01010101u) << 4;
                            hB2 |= ((qhB.y >> (2 * j + 1)) & 0x01010101u) << 4;
                        }
#pragma unroll
                        for (int p = 0; p < 3; ++p) {
                            const uint32_t xr = rec + (uint32_t)(p * TOKS) * GW_XROW + xb_row + eo;
                            const uint2 xl = w_lds64(xr), xh = w_lds64(xr + 32u);
                            int cl[4], ch[4];
                            wmma32z(cl, lA0, lB0, lA2, lB2, xl.x, xl.y);
                            wmma32z(ch, hA0, hB0, hA2, hB2, xh.x, xh.y);
                            // x sums of blocks 2j, 2j+1 for tokens 2q, 2q+1 (int16 pairs)
                            const uint32_t sxa = rec + sx_col + (uint32_t)(((2 * j) * ROWS + p * TOKS) * 2);
                            const uint32_t S0 = w_lds32(sxa), S1 = w_lds32(sxa + (uint32_t)ROWS * 2u);
                            const int S0a = (int)(S0 << 16) >> 16, S0b = (int)S0 >> 16;
                            const int S1a = (int)(S1 << 16) >> 16, S1b = (int)S1 >> 16;
                            const int iA0 = sAl * cl[0] + sAh * ch[0], iA1 = sAl * cl[1] + sAh * ch[1];
                            const int iB0 = sBl * cl[2] + sBh * ch[2], iB1 = sBl * cl[3] + sBh * ch[3];
                            const int mA0 = mAl * S0a + mAh * S1a, mA1 = mAl * S0b + mAh * S1b;
                            const int mB0 = mBl * S0a + mBh * S1a, mB1 = mBl * S0b + mBh * S1b;
                            const float2 sc = w_lds64f(rec + cs_col + (uint32_t)(p * TOKS) * 4u);
                            acc[0] = fmaf(sc.x, fmaf(dA, __int2float_rn(iA0), -dmA * __int2float_rn(mA0)), acc[0]);
                            acc[1] = fmaf(sc.y, fmaf(dA, __int2float_rn(iA1), -dmA * __int2float_rn(mA1)), acc[1]);
                            acc[2] = fmaf(sc.x, fmaf(dB, __int2float_rn(iB0), -dmB * __int2float_rn(mB0)), acc[2]);
                            acc[3] = fmaf(sc.y, fmaf(dB, __int2float_rn(iB1), -dmB * __int2float_rn(mB1)), acc[3]);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            if (++slot == a.nslots) { slot = 0; ph ^= 1u; }
        }
        // ---- the team's partials, summed over its warps in a fixed order ----
        float* pb = part + ((size_t)team * 2 + (grp & 1)) * TW * 128;
        *reinterpret_cast<float2*>(pb + tw * 128 + g * 8 + 2 * q) = make_float2(acc[0], acc[1]);
        *reinterpret_cast<float2*>(pb + tw * 128 + (g + 8) * 8 + 2 * q) = make_float2(acc[2], acc[3]);
        asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "r"(TW * 32) : "memory");
        const int tt = threadIdx.x - team * TW * 32;
        if (ok && tt < 128) {
            const int r = tt & 15, m = tt >> 4;
            const int row = r_begin + grp * 16 + (a.CS ? 4 * (r & 3) + (r >> 2) : r);
            const int tok = 8 * team + m;
            if (row < r_end && tok < a.M) {
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < TW; ++w) sum += pb[w * 128 + r * 8 + m];
                a.y[(size_t)tok * a.ldy + row] = sum;
            }
        }
        // the next group writes the other partial buffer; the team barrier of
        // the group after orders these reads before its reuse
    }
}

// ---- host side ----
struct GwPlan {
    int KC, nchunks, nslots;
    uint32_t kcb, RS, CS, xoff;
    size_t smem;
};

static uint32_t gw_block_bytes(int t) { return t == QT_Q8_0 ? 34u : t == QT_Q4_K ? 144u : t == QT_Q5_K ? 176u : 210u; }
static int gw_block_elems(int t) { return t == QT_Q8_0 ? 32 : 256; }

// The fewest K-chunks (largest copies) that give two slots, with at least
// one 64-element unit per warp of a team.
static bool gw_plan(int t, int N, int K, size_t rb, int M, int grid, GwPlan& p) {
    if (K % 256 || M < 3 || M > 16) return false;
    const int nh = M > 8 ? 2 : 1;
    const int rows_blk = (N + grid - 1) / grid;
    const int ngroups = (rows_blk + 15) / 16;
    const size_t fixed = 128 + 2 * GW_CW * 16 * 8 * 4 + 2 * GW_MAXSLOTS * 8 + 64;
    const int units = K / 256;
    bool found = false;
    int best_ns = 0;
    for (int need_ns = 2; need_ns >= 2 && !found; --need_ns) {
        for (int nc = 1; nc <= units; ++nc) {
            if (units % nc) continue;
            const int KC = K / nc;
            if (KC / 64 < GW_CW / nh) break;              // every warp of a team gets a unit
            const uint32_t kcb = (uint32_t)((size_t)KC / gw_block_elems(t) * gw_block_bytes(t));
            if (kcb % 16u) continue;
            uint32_t RS = (kcb + 15u) & ~15u;
            while (RS % 128u != (t == QT_Q6_K ? 16u : 32u)) RS += 16u;    // 32-bit (Q6_K) or 64-bit fragment loads
            const uint32_t CS = (nc == 1 && rb == kcb) ? ((4u * kcb + 127u) & ~127u) + 32u : 0u;
            const size_t wpart = CS ? 4u * (size_t)CS : 16u * (size_t)RS;
            const uint32_t xoff = (uint32_t)((wpart + 127) & ~size_t(127));
            const size_t slot = xoff + (size_t)(KC / 256) * gw_rec_bytes(nh);
            int ns = (int)((GW_SMEM_MAX - fixed) / slot);
            if (ns > GW_MAXSLOTS) ns = GW_MAXSLOTS;
            if (ns < need_ns) continue;
            p.KC = KC;
            p.nchunks = nc;
            p.kcb = kcb;
            p.RS = RS;
            p.CS = CS;
            p.xoff = xoff;
            best_ns = ns;
            found = true;
            break;
        }
    }
    if (!found) return false;
    const int need = ngroups * p.nchunks;
    int ns = best_ns < need ? best_ns : need;
    if (ns < 1) ns = 1;
    p.nslots = ns;
    p.smem = fixed + (size_t)ns * (p.xoff + (size_t)(p.KC / 256) * gw_rec_bytes(nh));
    return p.smem <= GW_SMEM_MAX + 1024;
}

bool gemv_wide_ok(int t, size_t rb, int K, int M) {
    if (t != QT_Q8_0 && t != QT_Q4_K && t != QT_Q5_K && t != QT_Q6_K) return false;
    if (M < 3 || M > 16 || rb % 16 || K % 256) return false;
    GwPlan p;
    return gw_plan(t, 148 * 64, K, rb, M, 148, p);
}

template <int T, int NH>
static tk_status go_wide(tk_ctx* ctx, const uint8_t* W, size_t rb, int N, int K, int M, const uint8_t* xr, float* y,
                         int ldy, cudaStream_t s) {
    const int grid = ctx->num_sms < N ? ctx->num_sms : N;
    GwPlan p;
    if (!gw_plan(T, N, K, rb, M, grid, p)) return fail(TK_ERR_UNSUPPORTED, "gemv wide: shape does not fit shared memory");
    auto kern = gemv_wide_kernel<T, NH>;
    static std::atomic<uint64_t> attr_done{0};   // per instantiation, one bit per device
    {
        const cudaError_t e = smem_attr_once(kern, (int)GW_SMEM_MAX + 1024, ctx->device, attr_done);
        if (e != cudaSuccess) return cuda_fail(e, "gemv wide smem attribute");
    }
    GwArgs a;
    a.W = W; a.rb = rb; a.N = N; a.K = K; a.M = M; a.xr = xr; a.y = y; a.ldy = ldy;
    a.KC = p.KC; a.nchunks = p.nchunks; a.kcb = p.kcb; a.RS = p.RS; a.CS = p.CS; a.xoff = p.xoff;
    a.nslots = p.nslots;
    a.status = ctx->status;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(GW_THREADS, 1, 1);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ProfScope ps(ctx, s, PK_GEMV);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    ctx->launches++;
    if (e != cudaSuccess) return cuda_fail(e, "gemv wide launch");
    return cuda_fail(cudaGetLastError(), "gemv wide launch");
}

tk_status launch_gemv_wide(tk_ctx* ctx, int t, const void* Wv, size_t rb, int N, int K, const float* x, int ldx, int M,
                           float* y, int ldy, cudaStream_t s) {
    const int nh = M > 8 ? 2 : 1;
    const size_t rec_bytes = (size_t)(K / 256) * gw_rec_bytes(nh);
    tk_status st = ws_ensure(ctx, rec_bytes, s);
    if (st != TK_OK) return st;
    uint8_t* xr = static_cast<uint8_t*>(ctx->ws);
    {
        const int tasks = 8 * nh * (K / 256);
        ProfScope ps(ctx, s, PK_GEMV);
        gw_xrec_kernel<<<(tasks + 7) / 8, 256, 0, s>>>(x, ldx, M, K, nh, xr);
        ctx->launches++;
        st = cuda_fail(cudaGetLastError(), "gemv x-record launch");
        if (st != TK_OK) return st;
    }
    const uint8_t* W = static_cast<const uint8_t*>(Wv);
    if (nh == 1) {
        if (t == QT_Q8_0) return go_wide<QT_Q8_0, 1>(ctx, W, rb, N, K, M, xr, y, ldy, s);
        if (t == QT_Q4_K) return go_wide<QT_Q4_K, 1>(ctx, W, rb, N, K, M, xr, y, ldy, s);
        if (t == QT_Q5_K) return go_wide<QT_Q5_K, 1>(ctx, W, rb, N, K, M, xr, y, ldy, s);
        if (t == QT_Q6_K) return go_wide<QT_Q6_K, 1>(ctx, W, rb, N, K, M, xr, y, ldy, s);
    } else {
        if (t == QT_Q8_0) return go_wide<QT_Q8_0, 2>(ctx, W, rb, N, K, M, xr, y, ldy, s);
        if (t == QT_Q4_K) return go_wide<QT_Q4_K, 2>(ctx, W, rb, N, K, M, xr, y, ldy, s);
        if (t == QT_Q5_K) return go_wide<QT_Q5_K, 2>(ctx, W, rb, N, K, M, xr, y, ldy, s);
        if (t == QT_Q6_K) return go_wide<QT_Q6_K, 2>(ctx, W, rb, N, K, M, xr, y, ldy, s);
    }
    return fail(TK_ERR_UNSUPPORTED, "gemv wide: type");
}

}  // namespace tk
