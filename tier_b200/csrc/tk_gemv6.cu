// tk_gemv6.cu -- decode GEMV for one or two tokens on the integer tensor
// cores (mma.sync s8 x s8 -> s32) for Q8_0 / Q4_K / Q5_K / Q6_K rows.
//
// y[m, n] = sum_k W(n, k) x[m, k], M <= 2.  The decode GEMV is meant to be
// HBM-bound; with fp16 MMAs (tk_gemv5.cu) the per-weight conversions (byte
// permutes, f16x2 subtractions) and the per-sub-block fp32 scaling fill the
// issue slots first.  Here the quants enter the MMA as the integers they are:
//
//  * x: every 256-element chunk of every token is scaled by a power of two
//    (its max into [2^21, 2^22)), rounded to an integer xi and split exactly
//    into three signed bytes, xi = p0 * 2^16 + p1 * 2^8 + p2.  The planes are
//    the MMA's B columns: column 3m + p is plane p of token m (6 of 8 columns
//    at M = 2).  Relative to the chunk's max, x is kept to 2^-22.
//  * W: Q8_0 quants are int8 already; Q4_K / Q5_K quants (0..15 / 0..31) are
//    masked out of their nibbles into bytes; Q6_K quants are (ql | qh << 4) -
//    32, one byte-wise add.  No per-weight float conversion.
//  * Products are exact in int32.  Q4_K / Q5_K: one m16n8k32 MMA per
//    32-element sub-block, scaled by its 6-bit sc in int32 and summed over the
//    super-block; the min term (sum over sub-blocks of m times the sub-block's
//    x sum) is one more MMA pair per super-block, with the x sums split into
//    two bytes.  The super-block's result is d * I1 - dmin * I2 in fp32.
//    Q6_K: one m16n8k16 MMA per 16-element sub-block, times its int8 sc, d *
//    I1 per super-block.  Q8_0: one m16n8k32 MMA per block, times d in fp32.
//  * Rows, slots, producer warp, ring of bulk copies and programmatic
//    dependent launch are those of tk_gemv5.cu.  The consumer warps form two
//    teams of eight that take alternate 16-row groups, so one team's group-end
//    barrier and fixed-order reduction overlap the other team's MMAs.  At the
//    end of a row group the three plane columns of each token are summed with
//    two warp shuffles.
// The result agrees with fp64 to ~1e-7 relative.  A non-finite x element makes
// its token's y non-finite (the chunk's scale is NaN).
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

constexpr int GI_CW = 16;                        // consumer warps
constexpr int GI_THREADS = (GI_CW + 1) * 32;     // + one producer warp
constexpr int GI_MAXSLOTS = 8;
constexpr size_t GI_SMEM_MAX = 220 * 1024;

struct GiArgs {
    const uint8_t* W;
    size_t rb;
    int N, K, M;
    const float* x;
    int ldx;
    float* y;
    int ldy;
    int KC;           // elements per K-chunk (slot)
    int nchunks;
    uint32_t kcb;     // bytes per row per chunk
    uint32_t RS;      // shared-memory row stride in a slot (one copy per row)
    uint32_t CS;      // nonzero: a slot is four copies of 4 whole rows, at CS-byte strides
    int nslots;       // slots per team ring
    int teams;        // consumer teams (1 or 2), on alternate row groups
    int XQ;           // x plane row stride in bytes
    int frozen;
    int* status;
    // several weights sharing x (tk_gemv_multi): rows [seg_end[i-1], seg_end[i])
    // are rows of Ws[i] with outputs ys[i]; nseg == 1 uses W, y, ldy
    int nseg;
    int seg_end[TK_GEMV_MAXSEG];
    const uint8_t* Ws[TK_GEMV_MAXSEG];
    float* ys[TK_GEMV_MAXSEG];
    int ldys[TK_GEMV_MAXSEG];
};

// segment of a row of the concatenated weights and the row within it
__device__ __forceinline__ int gi_seg(const GiArgs& a, int row, int& local) {
    int sg = 0;
    while (sg + 1 < a.nseg && row >= a.seg_end[sg]) ++sg;
    local = row - (sg ? a.seg_end[sg - 1] : 0);
    return sg;
}

__device__ __forceinline__ uint32_t i_lds16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t i_lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 i_lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float2 i_lds64f(uint32_t a) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 i_lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
// 32-bit load at an address that is 4-byte aligned or (odd) 2 mod 4: Q6_K
// super-blocks are 210 bytes, so every other one starts at 2 mod 4.
__device__ __forceinline__ uint32_t i_lds32_a(uint32_t a, bool odd) {
    if (!odd) return i_lds32(a);
    return __funnelshift_r(i_lds32(a - 2u), i_lds32(a + 2u), 16);
}
// D = A (16 x 32, s8) * B (32 x 8, s8), s32 (accumulator input zero: no
// per-MMA register clearing)
__device__ __forceinline__ void imma32z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    const int z = 0;
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(z));
}
__device__ __forceinline__ void imma16z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    const int z = 0;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%7, %7, %7, %7};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(z));
}
// int -> float, exact for |v| < 2^22: v added to the mantissa of 1.5 * 2^23
__device__ __forceinline__ float i2f22(int v) { return __int_as_float(v + 0x4B400000) - 12582912.0f; }
// byte k of w, zero-extended (one byte permute) or sign-extended
__device__ __forceinline__ int ubyte(uint32_t w, int k) { return (int)__byte_perm(w, 0u, 0x4440u | (uint32_t)k); }
__device__ __forceinline__ int sbyte(uint32_t w, int k) { return (int)(w << (24 - 8 * k)) >> 24; }
__device__ __forceinline__ float h2f_lo(uint32_t w) { return __half2float(__ushort_as_half((uint16_t)(w & 0xffffu))); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return __half2float(__ushort_as_half((uint16_t)(w >> 16))); }
__device__ __forceinline__ void gi_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void gi_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <int T>
__global__ void __launch_bounds__(GI_THREADS, 1) gemv_imma_kernel(const __grid_constant__ GiArgs a) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int nc256 = a.K / 256;
    const int ncol = 3 * a.M;
    const uint32_t slot_bytes = a.CS ? 4u * a.CS : 16u * a.RS;
    uint8_t* ring = sm;
    const int nteams = a.teams, TWn = GI_CW / nteams;
    uint8_t* xq = ring + (size_t)nteams * a.nslots * slot_bytes;               // [3M][XQ] int8 planes
    float* cs = reinterpret_cast<float*>(xq + (size_t)ncol * a.XQ);             // [nc256][8] column scales
    uint8_t* sb8 = reinterpret_cast<uint8_t*>(cs + (size_t)nc256 * 8);          // [nc256][lo, hi][8 cols][8 sub]
    float* part = reinterpret_cast<float*>(sb8 + (size_t)nc256 * 128);          // [team][2][TW][16 rows][8]
    uint64_t* full = reinterpret_cast<uint64_t*>(part + 2 * GI_CW * 128);
    uint64_t* empty = full + nteams * a.nslots;

    const int r_begin = (int)((long long)a.N * blockIdx.x / gridDim.x);
    const int r_end = (int)((long long)a.N * (blockIdx.x + 1) / gridDim.x);
    const int nrows = r_end - r_begin;
    const int ngroups = (nrows + 15) / 16;
    const int nslot_total = ngroups * a.nchunks;

    gi_launch_dependents();
    if (threadIdx.x == 0) {
        for (int i = 0; i < nteams * a.nslots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], TWn);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (!(a.frozen && warp == GI_CW)) gi_wait_prior();

    if (warp == GI_CW) {
        // ---------------- producer: one bulk copy per row of each slot ----------------
        // Uses in (group, chunk) order.  Group grp goes to team grp % TEAMS, whose
        // ring sees the team's uses in order (use u: slot u % nslots, phase
        // u / nslots), so every wait below is at most one phase ahead.
        bool ok = true;
        int issued = 0;
        for (int s = 0; s < nslot_total; ++s) {
            const int grp = s / a.nchunks, c = s - grp * a.nchunks;
            const int t = grp % nteams;
            const int u = (grp / nteams) * a.nchunks + c;
            const int slot = t * a.nslots + u % a.nslots;
            const int row0 = r_begin + grp * 16;
            const int nv = r_end - row0 < 16 ? r_end - row0 : 16;
            if (lane == 0) {
                if (ok && u >= a.nslots)
                    ok = mbar_wait(&empty[slot], (uint32_t)((u / a.nslots) - 1) & 1u, a.status);
                if (ok) mbar_arrive_expect_tx(&full[slot], (uint32_t)nv * a.kcb);
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            if (a.CS) {
                // whole rows, contiguous in W: rows 4i .. 4i+3 of the group in one copy
                if (lane < 4 && 4 * lane < nv) {
                    const int nr = nv - 4 * lane < 4 ? nv - 4 * lane : 4;
                    bulk_load(ring + (size_t)slot * slot_bytes + (size_t)lane * a.CS,
                              a.W + (size_t)(row0 + 4 * lane) * a.rb, (uint32_t)nr * a.kcb, &full[slot]);
                }
            } else if (lane < nv) {
                const uint8_t* src = a.W + (size_t)(row0 + lane) * a.rb;
                if (a.nseg > 1) {
                    int lr;
                    const int sg = gi_seg(a, row0 + lane, lr);
                    src = a.Ws[sg] + (size_t)lr * a.rb;
                }
                bulk_load(ring + (size_t)slot * slot_bytes + (size_t)lane * a.RS, src + (size_t)c * a.kcb, a.kcb,
                          &full[slot]);
            }
            issued = s + 1;
        }
        if (!ok && lane == 0) {
            // copies already issued land before the block exits (bounded): the
            // latest use of every slot
            int cnt[2] = {0, 0};
            for (int s = 0; s < issued; ++s) ++cnt[(s / a.nchunks) % nteams];
            for (int s = 0; s < issued; ++s) {
                const int grp = s / a.nchunks, c = s - grp * a.nchunks;
                const int t = grp % nteams;
                const int u = (grp / nteams) * a.nchunks + c;
                if (u + a.nslots >= cnt[t])
                    (void)mbar_wait(&full[t * a.nslots + u % a.nslots], (uint32_t)(u / a.nslots) & 1u, a.status);
            }
        }
        return;
    }

    // ---------------- consumers: x -> three int8 planes per (token, 256-chunk) ----------------
    for (int i = threadIdx.x; i < nc256 * 8; i += GI_CW * 32)
        if ((i & 7) >= ncol) cs[i] = 0.0f;                  // unused columns contribute 0
    for (int task = warp; task < a.M * nc256; task += GI_CW) {
        const int m = task / nc256, c = task - m * nc256;
        const float4* src = reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx + c * 256 + 8 * lane);
        const float4 v0 = __ldg(src), v1 = __ldg(src + 1);
        float mx = fmaxf(fmaxf(fmaxf(fabsf(v0.x), fabsf(v0.y)), fmaxf(fabsf(v0.z), fabsf(v0.w))),
                         fmaxf(fmaxf(fabsf(v1.x), fabsf(v1.y)), fmaxf(fabsf(v1.z), fabsf(v1.w))));
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // a non-finite x element makes the chunk's scale NaN, so y comes out
        // non-finite as the reference's fp32 sum does; its planes are zero
        const bool nonfin = __any_sync(0xffffffffu, !(isfinite(v0.x) && isfinite(v0.y) && isfinite(v0.z) &&
                                                      isfinite(v0.w) && isfinite(v1.x) && isfinite(v1.y) &&
                                                      isfinite(v1.z) && isfinite(v1.w)));
        int s = 0;
        if (mx > 0.0f) {
            // mx in [2^(E-127), 2^(E-126)): mx * 2^s in [2^21, 2^22); s >= -106 for finite mx
            s = 148 - (int)((__float_as_uint(mx) >> 23) & 0xffu);
            if (s > 127) s = 127;
        }
        const float up = nonfin ? 0.0f : __uint_as_float((uint32_t)(127 + s) << 23);
        const float f[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        uint32_t w0[2] = {0u, 0u}, w1[2] = {0u, 0u}, w2[2] = {0u, 0u};
        int s0 = 0, s1 = 0, s2 = 0;
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
        uint8_t* xrow = xq + (size_t)(3 * m) * a.XQ + c * 256 + 8 * lane;
        *reinterpret_cast<uint2*>(xrow) = make_uint2(w0[0], w0[1]);
        *reinterpret_cast<uint2*>(xrow + a.XQ) = make_uint2(w1[0], w1[1]);
        *reinterpret_cast<uint2*>(xrow + 2 * a.XQ) = make_uint2(w2[0], w2[1]);
        if (lane < 3) cs[c * 8 + 3 * m + lane] = nonfin ? __uint_as_float(0x7fc00000u) : ldexpf(1.0f, 16 - 8 * lane - s);
        if constexpr (T == QT_Q4_K || T == QT_Q5_K) {
            // x sums of each 32-element block (4 lanes), split S = hi * 128 + lo
#pragma unroll
            for (int o = 1; o <= 2; o <<= 1) {
                s0 += __shfl_xor_sync(0xffffffffu, s0, o);
                s1 += __shfl_xor_sync(0xffffffffu, s1, o);
                s2 += __shfl_xor_sync(0xffffffffu, s2, o);
            }
            if ((lane & 3) == 0) {
                const int b = lane >> 2;
                uint8_t* sbc = sb8 + (size_t)c * 128 + (3 * m) * 8 + b;
                sbc[0] = (uint8_t)(s0 & 127);
                sbc[8] = (uint8_t)(s1 & 127);
                sbc[16] = (uint8_t)(s2 & 127);
                sbc[64] = (uint8_t)(s0 >> 7);
                sbc[72] = (uint8_t)(s1 >> 7);
                sbc[80] = (uint8_t)(s2 >> 7);
            }
        }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(GI_CW * 32) : "memory");

    // this lane's B column (any valid one for columns >= 3M: dropped)
    const int colg = g < ncol ? g : 0;
    const uint32_t xq_b = smem_u32(xq + (size_t)colg * a.XQ);
    const uint32_t cs_q = smem_u32(cs) + 8u * q;                    // + 32 * chunk: columns 2q, 2q+1
    const uint32_t sb_g = smem_u32(sb8) + 8u * colg + 4u * q;       // + 128 * chunk (+ 64: high bytes)
    const uint32_t ring_u = smem_u32(ring);
    // slot offsets of the MMA tile's rows g and g+8.  Four-copy slots: tile row
    // i is row 4 (i & 3) + (i >> 2) of the group, so the four rows a half-warp
    // reads sit in four copies, 32 bytes apart in bank terms.
    const uint32_t offA = a.CS ? (uint32_t)(g & 3) * a.CS + (uint32_t)(g >> 2) * a.kcb : (uint32_t)g * a.RS;
    const uint32_t offB = a.CS ? (uint32_t)(g & 3) * a.CS + (uint32_t)(2 + (g >> 2)) * a.kcb : (uint32_t)(g + 8) * a.RS;

    // team t takes row groups t, t + TEAMS, ... from its own ring
    const int team = warp / TWn, tw = warp - team * TWn;
    bool ok = true;
    for (int grp = team; grp < ngroups; grp += nteams) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};     // rows g, g+8 x columns 2q, 2q+1
        for (int c = 0; c < a.nchunks; ++c) {
            const int u = (grp / nteams) * a.nchunks + c;        // use of this team's ring
            const int slot = team * a.nslots + u % a.nslots;
            const uint32_t ph = (uint32_t)(u / a.nslots) & 1u;
            if (ok) {
                const bool w = mbar_wait(&full[slot], ph, a.status);
                ok = __all_sync(0xffffffffu, w);
            }
            if (ok) {
                const uint32_t rA = ring_u + (uint32_t)slot * slot_bytes + offA;
                const uint32_t rB = ring_u + (uint32_t)slot * slot_bytes + offB;
                const int kc0 = c * a.KC;                 // first element of the chunk
                if constexpr (T == QT_Q8_0) {
                    // block pairs (68 bytes): the even block's quants start at 2 mod 4,
                    // the odd block's at 0 mod 4.  Thread q takes quants 8q .. 8q+7
                    // (MMA k 4q .. 4q+3 and 16+4q .. 16+4q+3; x uses the same order).
                    const int npairs = a.KC / 64;
                    for (int p = tw; p < npairs; p += TWn) {
                        const uint32_t pA = rA + 68u * p, pB = rB + 68u * p;
                        const int e0 = kc0 + 64 * p;
                        const uint32_t oe = 8u * q;
                        const uint32_t a0w = i_lds32(pA + oe), a1w = i_lds32(pA + oe + 4), a2w = i_lds32(pA + oe + 8);
                        const uint32_t b0w = i_lds32(pB + oe), b1w = i_lds32(pB + oe + 4), b2w = i_lds32(pB + oe + 8);
                        const uint32_t oo = 36u + 8u * q;
                        const uint32_t aO0 = i_lds32(pA + oo), aO2 = i_lds32(pA + oo + 4);
                        const uint32_t bO0 = i_lds32(pB + oo), bO2 = i_lds32(pB + oo + 4);
                        const uint2 xe = i_lds64(xq_b + (uint32_t)e0 + 8u * q);
                        const uint2 xo = i_lds64(xq_b + (uint32_t)e0 + 32u + 8u * q);
                        int ce[4], co[4];
                        imma32z(ce, __funnelshift_r(a0w, a1w, 16), __funnelshift_r(b0w, b1w, 16),
                               __funnelshift_r(a1w, a2w, 16), __funnelshift_r(b1w, b2w, 16), xe.x, xe.y);
                        imma32z(co, aO0, bO0, aO2, bO2, xo.x, xo.y);
                        const float dAe = __half2float(__ushort_as_half((uint16_t)i_lds16(pA)));
                        const float dBe = __half2float(__ushort_as_half((uint16_t)i_lds16(pB)));
                        const float dAo = __half2float(__ushort_as_half((uint16_t)i_lds16(pA + 34u)));
                        const float dBo = __half2float(__ushort_as_half((uint16_t)i_lds16(pB + 34u)));
                        const float2 sc = i_lds64f(cs_q + 32u * (uint32_t)(e0 >> 8));
                        acc[0] = fmaf(sc.x, fmaf(dAo, i2f22(co[0]), dAe * i2f22(ce[0])), acc[0]);
                        acc[1] = fmaf(sc.y, fmaf(dAo, i2f22(co[1]), dAe * i2f22(ce[1])), acc[1]);
                        acc[2] = fmaf(sc.x, fmaf(dBo, i2f22(co[2]), dBe * i2f22(ce[2])), acc[2]);
                        acc[3] = fmaf(sc.y, fmaf(dBo, i2f22(co[3]), dBe * i2f22(ce[3])), acc[3]);
                    }
                } else if constexpr (T == QT_Q6_K) {
                    // super-block (tier/quant.h:88-90): ql[128] low nibbles, qh[64]
                    // 2-bit high parts, sc[16] int8 per 16 elements, d fp16 at 208.
                    // Element e of half h (e < 128): ql byte 64h + (e & 63), nibble
                    // e >> 6; qh byte 128 + 32h + (e & 31), bits 2 (e >> 5).  One
                    // m16n8k16 MMA per 16-element sub-block; thread q takes its
                    // elements 4q .. 4q+3.
                    const int nsb = a.KC / 256;
                    for (int sbi = tw; sbi < nsb; sbi += TWn) {
                        const uint32_t sA = rA + 210u * sbi, sB = rB + 210u * sbi;
                        const bool odd = (sbi & 1) != 0;
                        const int e0 = kc0 + 256 * sbi;
                        uint32_t scA[4], scB[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            scA[k] = i_lds32_a(sA + 192u + 4u * k, odd);
                            scB[k] = i_lds32_a(sB + 192u + 4u * k, odd);
                        }
                        int I1[4] = {0, 0, 0, 0};
#pragma unroll
                        for (int ha = 0; ha < 2; ++ha) {
#pragma unroll
                            for (int w = 0; w < 2; ++w) {
                                const uint32_t o = 64u * ha + 16u * w + 4u * q;
                                const uint32_t ho = 128u + 32u * ha + 16u * w + 4u * q;
                                const uint32_t l0A = i_lds32_a(sA + o, odd), l1A = i_lds32_a(sA + o + 32u, odd);
                                const uint32_t l0B = i_lds32_a(sB + o, odd), l1B = i_lds32_a(sB + o + 32u, odd);
                                const uint32_t hA = i_lds32_a(sA + ho, odd), hB = i_lds32_a(sB + ho, odd);
#pragma unroll
                                for (int gq = 0; gq < 4; ++gq) {
                                    const uint32_t lA = gq & 1 ? l1A : l0A, lB = gq & 1 ? l1B : l0B;
                                    const uint32_t uA = ((lA >> (4 * (gq >> 1))) & 0x0F0F0F0Fu) |
                                                        (((hA >> (2 * gq)) & 0x03030303u) << 4);
                                    const uint32_t uB = ((lB >> (4 * (gq >> 1))) & 0x0F0F0F0Fu) |
                                                        (((hB >> (2 * gq)) & 0x03030303u) << 4);
                                    // bytes u - 32 (u < 64): no borrow crosses a byte
                                    const uint32_t vA = ((uA | 0x80808080u) - 0x20202020u) ^ 0x80808080u;
                                    const uint32_t vB = ((uB | 0x80808080u) - 0x20202020u) ^ 0x80808080u;
                                    const int e = e0 + 128 * ha + 32 * gq + 16 * w;
                                    int cc[4];
                                    imma16z(cc, vA, vB, i_lds32(xq_b + (uint32_t)e + 4u * q));
                                    const int sub = 8 * ha + 2 * gq + w;
                                    const int sa = sbyte(scA[sub >> 2], sub & 3), sb = sbyte(scB[sub >> 2], sub & 3);
                                    I1[0] += sa * cc[0];
                                    I1[1] += sa * cc[1];
                                    I1[2] += sb * cc[2];
                                    I1[3] += sb * cc[3];
                                }
                            }
                        }
                        const float dA = __half2float(__ushort_as_half((uint16_t)i_lds16(sA + 208u)));
                        const float dB = __half2float(__ushort_as_half((uint16_t)i_lds16(sB + 208u)));
                        const float2 sc = i_lds64f(cs_q + 32u * (uint32_t)(e0 >> 8));
                        acc[0] = fmaf(sc.x, dA * __int2float_rn(I1[0]), acc[0]);
                        acc[1] = fmaf(sc.y, dA * __int2float_rn(I1[1]), acc[1]);
                        acc[2] = fmaf(sc.x, dB * __int2float_rn(I1[2]), acc[2]);
                        acc[3] = fmaf(sc.y, dB * __int2float_rn(I1[3]), acc[3]);
                    }
                } else {
                    // Q4_K / Q5_K super-block (tier/quant.h:83-87): d, dmin fp16, 12
                    // bytes of packed 6-bit sc / m (tier/quant.h:47-48), Q5_K qh[32],
                    // qs[128]: sub-block 2j is the low nibbles of qs[32j .. 32j+31],
                    // 2j+1 the high ones.  Thread q takes elements 8q .. 8q+7.
                    constexpr uint32_t SB = T == QT_Q4_K ? 144u : 176u;
                    constexpr uint32_t QS = T == QT_Q4_K ? 16u : 48u;
                    const int nsb = a.KC / 256;
                    for (int sbi = tw; sbi < nsb; sbi += TWn) {
                        const uint32_t sA = rA + SB * sbi, sB = rB + SB * sbi;
                        const int e0 = kc0 + 256 * sbi;
                        const int ch = e0 >> 8;
                        const uint4 hA = i_lds128(sA), hB = i_lds128(sB);
                        // sc[0..3], sc[4..7], m[0..3], m[4..7] as bytes
                        const uint32_t scA0 = hA.y & 0x3F3F3F3Fu;
                        const uint32_t scA1 = (hA.w & 0x0F0F0F0Fu) | ((hA.y >> 2) & 0x30303030u);
                        const uint32_t mA0 = hA.z & 0x3F3F3F3Fu;
                        const uint32_t mA1 = ((hA.w >> 4) & 0x0F0F0F0Fu) | ((hA.z >> 2) & 0x30303030u);
                        const uint32_t scB0 = hB.y & 0x3F3F3F3Fu;
                        const uint32_t scB1 = (hB.w & 0x0F0F0F0Fu) | ((hB.y >> 2) & 0x30303030u);
                        const uint32_t mB0 = hB.z & 0x3F3F3F3Fu;
                        const uint32_t mB1 = ((hB.w >> 4) & 0x0F0F0F0Fu) | ((hB.z >> 2) & 0x30303030u);
                        // min term: sum over the 8 sub-blocks of m * S as one k16 MMA per
                        // byte of S (k = sub-block; k 8..15 zero)
                        int I2[4];
                        {
                            const uint32_t amA = q == 0 ? mA0 : q == 1 ? mA1 : 0u;
                            const uint32_t amB = q == 0 ? mB0 : q == 1 ? mB1 : 0u;
                            const uint32_t so = sb_g + 128u * (uint32_t)ch;
                            const uint32_t blo = q < 2 ? i_lds32(so) : 0u, bhi = q < 2 ? i_lds32(so + 64u) : 0u;
                            int ml[4], mh[4];
                            imma16z(ml, amA, amB, blo);
                            imma16z(mh, amA, amB, bhi);
#pragma unroll
                            for (int i = 0; i < 4; ++i) I2[i] = mh[i] * 128 + ml[i];
                        }
                        uint2 qhA = make_uint2(0u, 0u), qhB = make_uint2(0u, 0u);
                        if constexpr (T == QT_Q5_K) {
                            qhA = i_lds64(sA + 16u + 8u * q);
                            qhB = i_lds64(sB + 16u + 8u * q);
                        }
                        int I1[4] = {0, 0, 0, 0};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const uint2 wA = i_lds64(sA + QS + 32u * j + 8u * q);
                            const uint2 wB = i_lds64(sB + QS + 32u * j + 8u * q);
                            uint32_t lA0 = wA.x & 0x0F0F0F0Fu, lA2 = wA.y & 0x0F0F0F0Fu;
                            uint32_t lB0 = wB.x & 0x0F0F0F0Fu, lB2 = wB.y & 0x0F0F0F0Fu;
                            uint32_t hA0 = (wA.x >> 4) & 0x0F0F0F0Fu, hA2 = (wA.y >> 4) & 0x0F0F0F0Fu;
                            uint32_t hB0 = (wB.x >> 4) & 0x0F0F0F0Fu, hB2 = (wB.y >> 4) & 0x0F0F0F0Fu;
                            if constexpr (T == QT_Q5_K) {
                                lA0 |= ((qhA.x >> (2 * j)) & 0x01010101u) << 4;
                                lA2 |= ((qhA.y >> (2 * j)) & 0x01010101u) << 4;
                                lB0 |= ((qhB.x >> (2 * j)) & 0x01010101u) << 4;
                                lB2 |= ((qhB.y >> (2 * j)) & 0x01010101u) << 4;
                                hA0 |= ((qhA.x >> (2 * j + 1)) & 0x01010101u) << 4;
                                hA2 |= ((qhA.y >> (2 * j + 1)) & 0x01010101u) << 4;
                                hB0 |= ((qhB.x >> (2 * j + 1)) & 0x01010101u) << 4;
                                hB2 |= ((qhB.y >> (2 * j + 1)) & 0x01010101u) << 4;
                            }
                            const uint32_t xo = (uint32_t)(e0 + 64 * j) + 8u * q;
                            const uint2 xl = i_lds64(xq_b + xo), xh = i_lds64(xq_b + xo + 32u);
                            int cl[4], chh[4];
                            imma32z(cl, lA0, lB0, lA2, lB2, xl.x, xl.y);
                            imma32z(chh, hA0, hB0, hA2, hB2, xh.x, xh.y);
                            const int sAl = ubyte(j < 2 ? scA0 : scA1, (2 * j) & 3);
                            const int sAh = ubyte(j < 2 ? scA0 : scA1, (2 * j + 1) & 3);
                            const int sBl = ubyte(j < 2 ? scB0 : scB1, (2 * j) & 3);
                            const int sBh = ubyte(j < 2 ? scB0 : scB1, (2 * j + 1) & 3);
                            I1[0] += sAl * cl[0] + sAh * chh[0];
                            I1[1] += sAl * cl[1] + sAh * chh[1];
                            I1[2] += sBl * cl[2] + sBh * chh[2];
                            I1[3] += sBl * cl[3] + sBh * chh[3];
                        }
                        const float dA = h2f_lo(hA.x), dmA = h2f_hi(hA.x);
                        const float dB = h2f_lo(hB.x), dmB = h2f_hi(hB.x);
                        const float2 sc = i_lds64f(cs_q + 32u * (uint32_t)ch);
                        acc[0] = fmaf(sc.x, fmaf(dA, __int2float_rn(I1[0]), -dmA * __int2float_rn(I2[0])), acc[0]);
                        acc[1] = fmaf(sc.y, fmaf(dA, __int2float_rn(I1[1]), -dmA * __int2float_rn(I2[1])), acc[1]);
                        acc[2] = fmaf(sc.x, fmaf(dB, __int2float_rn(I1[2]), -dmB * __int2float_rn(I2[2])), acc[2]);
                        acc[3] = fmaf(sc.y, fmaf(dB, __int2float_rn(I1[3]), -dmB * __int2float_rn(I2[3])), acc[3]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
        }
        // ---- planes -> tokens: token 0 is columns 0, 1, 2 (lanes q = 0, 1),
        //      token 1 columns 3, 4, 5 (lanes q = 1, 2) ----
        const float n0 = __shfl_down_sync(0xffffffffu, acc[0], 1), n2 = __shfl_down_sync(0xffffffffu, acc[2], 1);
        const float p1 = __shfl_up_sync(0xffffffffu, acc[1], 1), p3 = __shfl_up_sync(0xffffffffu, acc[3], 1);
        float* pb = part + ((size_t)team * 2 + ((grp / nteams) & 1)) * TWn * 128;
        if (q == 0) {
            pb[tw * 128 + g * 8] = (acc[0] + acc[1]) + n0;
            pb[tw * 128 + (g + 8) * 8] = (acc[2] + acc[3]) + n2;
        } else if (q == 2) {
            pb[tw * 128 + g * 8 + 1] = (p1 + acc[0]) + acc[1];
            pb[tw * 128 + (g + 8) * 8 + 1] = (p3 + acc[2]) + acc[3];
        }
        // ---- sum the team's partials in a fixed order ----
        asm volatile("bar.sync %0, %1;" ::"r"(2 + team), "r"(TWn * 32) : "memory");
        const int tt = threadIdx.x - team * TWn * 32;
        if (ok && tt < 16 * a.M) {
            const int r = tt & 15, m = tt >> 4;
            const int row = r_begin + grp * 16 + (a.CS ? 4 * (r & 3) + (r >> 2) : r);
            if (row < r_end) {
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < TWn; ++w) sum += pb[w * 128 + r * 8 + m];
                if (a.nseg > 1) {
                    int lr;
                    const int sg = gi_seg(a, row, lr);
                    a.ys[sg][(size_t)m * a.ldys[sg] + lr] = sum;
                } else {
                    a.y[(size_t)m * a.ldy + row] = sum;
                }
            }
        }
        // the team's next group writes the other partial buffer; the team
        // barrier of the group after orders these reads before its reuse
    }
}

// ---- host side ----
struct GiPlan {
    int KC, nchunks, nslots, teams, XQ;
    uint32_t kcb, RS, CS;
    size_t smem;
};

static uint32_t gi_block_bytes(int t) { return t == QT_Q8_0 ? 34u : t == QT_Q4_K ? 144u : t == QT_Q5_K ? 176u : 210u; }
static int gi_block_elems(int t) { return t == QT_Q8_0 ? 32 : 256; }

// Plan for a given team count and number of K-chunks: false if the x planes
// and two slots per team ring (one if `one_ok`) do not fit.
// `whole`: a group's 16 rows are contiguous in one weight (one matrix, not
// segments), so a whole-row slot can be four 4-row copies.
static bool gi_plan_for(int t, int N, int K, size_t rb, int M, int grid, int teams, int nc, bool one_ok, bool whole,
                        GiPlan& p) {
    if (K % 256 || M < 1 || M > 2 || (K / 256) % nc) return false;
    const int rows_blk = (N + grid - 1) / grid;
    const int ngroups = (rows_blk + 15) / 16;
    p.XQ = K + 32;                                // 32 mod 128: conflict-free 64-bit x loads
    const int nc256 = K / 256;
    const size_t fixed = 128 + (size_t)3 * M * p.XQ + (size_t)nc256 * 32 + (size_t)nc256 * 128 +
                         2 * GI_CW * 16 * 8 * 4 + 2 * GI_MAXSLOTS * 8 + 64;
    if (fixed >= GI_SMEM_MAX) return false;
    const int KC = K / nc;
    const uint32_t kcb = (uint32_t)((size_t)KC / gi_block_elems(t) * gi_block_bytes(t));
    if (kcb % 16u) return false;                  // bulk copies: 16-byte sizes and source offsets
    const uint32_t rs_mod = t == QT_Q6_K ? 16u : 32u;     // 32-bit (Q6_K) or 64-bit fragment loads
    uint32_t RS = (kcb + 15u) & ~15u;
    while (RS % 128u != rs_mod) RS += 16u;
    // whole rows with no gap between them: four copies of 4 rows per slot
    const uint32_t CS = (whole && nc == 1 && rb == kcb) ? ((4u * kcb + 127u) & ~127u) + 32u : 0u;
    const size_t slot = CS ? 4u * (size_t)CS : 16u * (size_t)RS;
    int nsl = (int)((GI_SMEM_MAX - fixed) / slot) / teams;
    if (nsl > GI_MAXSLOTS / teams) nsl = GI_MAXSLOTS / teams;
    if (nsl < (one_ok ? 1 : 2) || teams * nsl < 2) return false;
    // a team needs no more slots than its groups' chunks
    const int need = ((ngroups + teams - 1) / teams) * nc;
    if (nsl > need) nsl = need;
    p.KC = KC;
    p.nchunks = nc;
    p.kcb = kcb;
    p.RS = RS;
    p.CS = CS;
    p.teams = teams;
    p.nslots = nsl;
    p.smem = fixed + (size_t)teams * nsl * slot;
    return p.smem <= GI_SMEM_MAX + 1024;
}

// Whole rows (one K-chunk) when they fit, with two consumer teams and two
// slots per team, else one; otherwise one team and the fewest K-chunks that
// give two slots.  Fewer, larger bulk copies stream faster.
static bool gi_plan(int t, int N, int K, size_t rb, int M, int grid, GiPlan& p, bool whole = true) {
    if (gi_plan_for(t, N, K, rb, M, grid, 2, 1, false, whole, p)) return true;
    if (gi_plan_for(t, N, K, rb, M, grid, 2, 1, true, whole, p)) return true;
    const int units = K / 256;
    for (int nc = 2; nc <= units; ++nc)
        if (gi_plan_for(t, N, K, rb, M, grid, 1, nc, false, whole, p)) return true;
    return false;
}

bool gemv_imma_ok(int t, size_t rb, int K, int M) {
    if (t != QT_Q8_0 && t != QT_Q4_K && t != QT_Q5_K && t != QT_Q6_K) return false;
    if (M < 1 || M > 2 || rb % 16 || K % 256) return false;
    GiPlan p;
    return gi_plan(t, 148 * 64, K, rb, M, 148, p);
}

struct GiSegs {
    int n;
    const void* const* W;
    const int* rows;
    float* const* y;
    const int* ldy;
};

template <int T>
static tk_status go_imma(tk_ctx* ctx, const uint8_t* W, size_t rb, int N, int K, int M, const float* x, int ldx,
                         float* y, int ldy, bool frozen, cudaStream_t s, const GiSegs* seg = nullptr) {
    const int grid = ctx->num_sms < N ? ctx->num_sms : N;
    GiPlan p;
    if (!gi_plan(T, N, K, rb, M, grid, p, seg == nullptr))
        return fail(TK_ERR_UNSUPPORTED, "gemv imma: shape does not fit shared memory");
    auto kern = gemv_imma_kernel<T>;
    static std::atomic<uint64_t> attr_done{0};   // per instantiation, one bit per device
    {
        const cudaError_t e = smem_attr_once(kern, (int)GI_SMEM_MAX + 1024, ctx->device, attr_done);
        if (e != cudaSuccess) return cuda_fail(e, "gemv imma smem attribute");
    }
    GiArgs a;
    a.W = W; a.rb = rb; a.N = N; a.K = K; a.M = M; a.x = x; a.ldx = ldx; a.y = y; a.ldy = ldy;
    a.KC = p.KC; a.nchunks = p.nchunks; a.kcb = p.kcb; a.RS = p.RS; a.CS = p.CS; a.nslots = p.nslots; a.teams = p.teams; a.XQ = p.XQ;
    a.frozen = frozen;
    a.status = ctx->status;
    a.nseg = 1;
    if (seg) {
        a.nseg = seg->n;
        int end = 0;
        for (int i = 0; i < seg->n; ++i) {
            end += seg->rows[i];
            a.seg_end[i] = end;
            a.Ws[i] = static_cast<const uint8_t*>(seg->W[i]);
            a.ys[i] = seg->y[i];
            a.ldys[i] = seg->ldy[i];
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(GI_THREADS, 1, 1);
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
    if (e != cudaSuccess) return cuda_fail(e, "gemv imma launch");
    return cuda_fail(cudaGetLastError(), "gemv imma launch");
}

tk_status launch_gemv_imma(tk_ctx* ctx, int t, const void* Wv, size_t rb, int N, int K, const float* x, int ldx, int M,
                           float* y, int ldy, bool frozen, cudaStream_t s) {
    const uint8_t* W = static_cast<const uint8_t*>(Wv);
    if (t == QT_Q8_0) return go_imma<QT_Q8_0>(ctx, W, rb, N, K, M, x, ldx, y, ldy, frozen, s);
    if (t == QT_Q4_K) return go_imma<QT_Q4_K>(ctx, W, rb, N, K, M, x, ldx, y, ldy, frozen, s);
    if (t == QT_Q5_K) return go_imma<QT_Q5_K>(ctx, W, rb, N, K, M, x, ldx, y, ldy, frozen, s);
    if (t == QT_Q6_K) return go_imma<QT_Q6_K>(ctx, W, rb, N, K, M, x, ldx, y, ldy, frozen, s);
    return fail(TK_ERR_UNSUPPORTED, "gemv imma: type");
}

bool gemv_imma_multi_ok(int t, size_t rb, int K, int M) {
    if (t != QT_Q8_0 && t != QT_Q4_K && t != QT_Q5_K && t != QT_Q6_K) return false;
    if (M < 1 || M > 2 || rb % 16 || K % 256) return false;
    GiPlan p;
    return gi_plan(t, 148 * 64, K, rb, M, 148, p, false);
}

tk_status launch_gemv_imma_multi(tk_ctx* ctx, int t, int nseg, const void* const* W, const int* rows, float* const* y,
                                 const int* ldy, size_t rb, int K, const float* x, int ldx, int M, bool frozen,
                                 cudaStream_t s) {
    int N = 0;
    for (int i = 0; i < nseg; ++i) N += rows[i];
    const GiSegs seg{nseg, W, rows, y, ldy};
    const uint8_t* W0 = static_cast<const uint8_t*>(W[0]);
    if (t == QT_Q8_0) return go_imma<QT_Q8_0>(ctx, W0, rb, N, K, M, x, ldx, y[0], ldy[0], frozen, s, &seg);
    if (t == QT_Q4_K) return go_imma<QT_Q4_K>(ctx, W0, rb, N, K, M, x, ldx, y[0], ldy[0], frozen, s, &seg);
    if (t == QT_Q5_K) return go_imma<QT_Q5_K>(ctx, W0, rb, N, K, M, x, ldx, y[0], ldy[0], frozen, s, &seg);
    if (t == QT_Q6_K) return go_imma<QT_Q6_K>(ctx, W0, rb, N, K, M, x, ldx, y[0], ldy[0], frozen, s, &seg);
    return fail(TK_ERR_UNSUPPORTED, "gemv imma: type");
}

}  // namespace tk
