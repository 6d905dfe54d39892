// tk_gemv5.cu -- decode GEMV on the tensor cores (mma.sync m16n8k16, fp16 in,
// fp32 accumulate) for Q8_0 / Q4_K / Q5_K / Q6_K rows and M <= 8 tokens with x
// resident in shared memory.  The dispatcher (tk_gemv.cu) sends 1-2 tokens to
// the integer kernel (tk_gemv6.cu) and most 5..16-token cases to the one that
// streams x with the weight (tk_gemv7.cu); this one takes 3-4 tokens whose x
// fits and the shapes those kernels do not plan for.
//
// y[m, n] = sum_k W(n, k) x[m, k].  The path is HBM-bound; the point of the
// tensor cores here is to take the multiply-adds off the issue slots, which
// the scalar kernel (tk_gemv4.cu) fills before HBM does.
//
//  * One block per SM, owning a contiguous range of rows (any count, so the
//    bytes per SM differ by at most one row); rows are processed in groups of
//    16 (one MMA A tile; rows past the range are never loaded and their
//    results are dropped).  A producer warp streams (group, K-chunk) slots
//    through a shared-memory ring: one cp.async.bulk per row, into rows
//    padded to a stride of 32 mod 128 bytes so the 64-bit fragment loads
//    below are bank-conflict-free.
//  * Sixteen consumer warps split every slot's K range (Q8_0: block pairs,
//    K-quants: super-blocks) and keep fp32 partial sums in registers; at the
//    end of a group they are summed over the warps in a fixed order
//    (deterministic), one named barrier per group.
//  * W fragment: the MMA's k index is permuted the same way for A and B.
//    Q8_0 / Q4_K / Q5_K: thread q takes the quants 8q .. 8q+7 of each
//    32-element block: 8q .. 8q+3 are k 2q, 2q+1, 2q+8, 2q+9 of the block's
//    first 16-element window, and 8q+4 .. 8q+7 those of the second.  Q6_K has
//    a scale per 16 elements, so each window is one 16-element sub-block and
//    thread q takes its elements 4q .. 4q+3.  A row's A operand per window is
//    one 32-bit word of quants: a byte permute with the fp16 magic 0x64 gives
//    1024 + u, an exact f16x2 subtraction gives the quant.  Quants of every
//    type here are integers of at most 8 bits: exact in fp16.
//  * x: each 32-element block of each token is scaled by a power of two (its
//    max into [2^14, 2^15)) and split into fp16 hi + lo (x = hi + lo to about
//    2^-22 relative); two MMAs (hi, lo) per window, and the window's fp32
//    result is multiplied by the block scale and by d (Q8_0), d*sc with
//    -dmin*m times the fp32 block sum of x (Q4_K, Q5_K) or d*sc (Q6_K).
//    Agreement with fp64 is ~1e-6 relative; the decode tolerance is 2e-3.
//  * Programmatic dependent launch as in tk_gemv4.cu.
#include "tk_device.cuh"
#include "tk_internal.h"

#include <cmath>

namespace tk {

constexpr int GM_CW = 16;                        // consumer warps
constexpr int GM_THREADS = (GM_CW + 1) * 32;     // + one producer warp
constexpr int GM_MAXSLOTS = 8;
constexpr size_t GM_SMEM_MAX = 220 * 1024;

struct GmArgs {
    const uint8_t* W;
    size_t rb;
    int N, K, M;
    const float* x;
    int ldx;
    float* y;
    int ldy;
    int KP;           // K-parts per 16-row group (one warp item each)
    int KC;           // elements per K-chunk (slot)
    int nchunks;
    uint32_t kcb;     // bytes per row per chunk
    uint32_t RS;      // shared-memory row stride in a slot
    int nslots;
    int XS;           // x row stride in halves
    int frozen;
    int* status;
};

__device__ __forceinline__ uint32_t g_lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 g_lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float2 g_lds64f(uint32_t a) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float4 g_lds128f(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 g_lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
// 32-bit shared load at an address that is 4-byte aligned (odd == false) or
// 2 mod 4 (odd == true: two aligned loads and a funnel shift).  Q6_K
// super-blocks are 210 bytes, so every other one starts at 2 mod 4.
__device__ __forceinline__ uint32_t g_lds32_a(uint32_t a, bool odd) {
    if (!odd) return g_lds32(a);
    return __funnelshift_r(g_lds32(a - 2u), g_lds32(a + 2u), 16);
}
__device__ __forceinline__ uint32_t g_lds16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
// Quant bytes u (< 256) of w -> two f16x2 registers (u0, u1) and (u2, u3)
// minus off, exactly: 0x64 above each byte is the fp16 of 1024 + u.
__device__ __forceinline__ void bytes_h2(uint32_t w, uint32_t off2, uint32_t& lo, uint32_t& hi) {
    lo = hsub2(__byte_perm(w, 0x64646464u, 0x4140), off2);
    hi = hsub2(__byte_perm(w, 0x64646464u, 0x4342), off2);
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void gm_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void gm_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void cp16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int T>
__global__ void __launch_bounds__(GM_THREADS, 1) gemv_mma_kernel(const __grid_constant__ GmArgs a) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int nblk = a.K / 32;
    const uint32_t slot_bytes = 16u * a.RS;
    uint8_t* ring = sm;
    uint16_t* xh = reinterpret_cast<uint16_t*>(ring + (size_t)a.nslots * slot_bytes);
    uint16_t* xl = xh + (size_t)a.M * a.XS;
    float* xsc = reinterpret_cast<float*>(xl + (size_t)a.M * a.XS);   // [nblk][8]: 2^-e per block and token
    float* xsum = xsc + (size_t)nblk * 8;                                // [nblk][8]: fp32 block sums (K-quants)
    float* part = xsum + (size_t)nblk * 8;                               // [2][CW][16][8]
    float* tab = part + 2 * GM_CW * 16 * 8;   // per warp [16 rows][8 sub][2] (Q4_K, Q5_K) or [16 rows][16] (Q6_K)
    uint64_t* full = reinterpret_cast<uint64_t*>(tab + GM_CW * 256);
    uint64_t* empty = full + a.nslots;

    const int r_begin = (int)((long long)a.N * blockIdx.x / gridDim.x);
    const int r_end = (int)((long long)a.N * (blockIdx.x + 1) / gridDim.x);
    const int nrows = r_end - r_begin;
    const int ngroups = (nrows + 15) / 16;
    const int nslot_total = ngroups * a.nchunks;

    gm_launch_dependents();
    if (threadIdx.x == 0) {
        for (int i = 0; i < a.nslots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], GM_CW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (!(a.frozen && warp == GM_CW)) gm_wait_prior();

    if (warp == GM_CW) {
        // ---------------- producer: one bulk copy per row of each slot ----------------
        bool ok = true;
        int slot = 0, issued = 0;
        for (int s = 0; s < nslot_total; ++s) {
            const int grp = s / a.nchunks, c = s - grp * a.nchunks;
            const int row0 = r_begin + grp * 16;
            const int nv = r_end - row0 < 16 ? r_end - row0 : 16;
            if (lane == 0) {
                if (ok && s >= a.nslots)
                    ok = mbar_wait(&empty[slot], (uint32_t)((s / a.nslots) - 1) & 1u, a.status);
                if (ok) mbar_arrive_expect_tx(&full[slot], (uint32_t)nv * a.kcb);
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            if (lane < nv)
                bulk_load(ring + (size_t)slot * slot_bytes + (size_t)lane * a.RS,
                          a.W + (size_t)(row0 + lane) * a.rb + (size_t)c * a.kcb, a.kcb, &full[slot]);
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

    // ---------------- consumers: stage x (per token and 32-block: scale, hi + lo) ----------------
    // four threads per (token, block), eight elements each; max and sum over
    // the four by shuffles (the four are consecutive lanes of one warp)
    for (int it = threadIdx.x; it < 4 * a.M * nblk; it += GM_CW * 32) {
        const int item = it >> 2, sub = it & 3;
        const int m = item / nblk, b = item - m * nblk;
        const float4* src = reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx + b * 32 + 8 * sub);
        const float4 v0 = __ldg(src), v1 = __ldg(src + 1);
        float mx = fmaxf(fmaxf(fmaxf(fabsf(v0.x), fabsf(v0.y)), fmaxf(fabsf(v0.z), fabsf(v0.w))),
                         fmaxf(fmaxf(fabsf(v1.x), fabsf(v1.y)), fmaxf(fabsf(v1.z), fabsf(v1.w))));
        float sum = ((v0.x + v0.y) + (v0.z + v0.w)) + ((v1.x + v1.y) + (v1.z + v1.w));
        // the loop trip count is the same for the 4 lanes of an item (4 * M * nblk is a multiple of 4)
        const unsigned grp_mask = __activemask();
        mx = fmaxf(mx, __shfl_xor_sync(grp_mask, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(grp_mask, mx, 2));
        const float s1 = sum + __shfl_xor_sync(grp_mask, sum, 1);
        sum = s1 + __shfl_xor_sync(grp_mask, s1, 2);
        int e = 0;
        if (mx > 0.0f) {
            int ex;
            (void)frexpf(mx, &ex);        // mx = f * 2^ex, f in [0.5, 1)
            e = 15 - ex;                   // mx * 2^e in [2^14, 2^15)
            if (e > 100) e = 100;
            if (e < -100) e = -100;
        }
        const float up = ldexpf(1.0f, e);
        const float f[8] = {v0.x * up, v0.y * up, v0.z * up, v0.w * up, v1.x * up, v1.y * up, v1.z * up, v1.w * up};
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half h0 = __float2half_rn(f[2 * i]), h1 = __float2half_rn(f[2 * i + 1]);
            const __half l0 = __float2half_rn(f[2 * i] - __half2float(h0));
            const __half l1 = __float2half_rn(f[2 * i + 1] - __half2float(h1));
            hw[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            lw[i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        *reinterpret_cast<uint4*>(xh + (size_t)m * a.XS + b * 32 + 8 * sub) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(xl + (size_t)m * a.XS + b * 32 + 8 * sub) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        if (sub == 0) {
            xsc[b * 8 + m] = ldexpf(1.0f, -e);
            xsum[b * 8 + m] = sum;
        }
    }
    // tokens m >= M: zero scale and sum, so their (unused) columns stay finite
    for (int it = threadIdx.x; it < (8 - a.M) * nblk; it += GM_CW * 32) {
        const int m = a.M + it / nblk, b = it % nblk;
        xsc[b * 8 + m] = 0.0f;
        xsum[b * 8 + m] = 0.0f;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(GM_CW * 32) : "memory");

    // this lane's B-operand token (any valid token for columns >= M: dropped)
    const int tok = g < a.M ? g : 0;
    const uint32_t xh_t = smem_u32(xh + (size_t)tok * a.XS) + 16u * q;   // x[8q .. 8q+7] of each block
    const uint32_t xl_t = smem_u32(xl + (size_t)tok * a.XS) + 16u * q;
    const uint32_t xh6_t = smem_u32(xh + (size_t)tok * a.XS) + 8u * q;   // Q6_K: x[4q .. 4q+3] of each window
    const uint32_t xl6_t = smem_u32(xl + (size_t)tok * a.XS) + 8u * q;
    const uint32_t xsc_q = smem_u32(xsc) + 8u * q;      // + blk * 32: tokens 2q, 2q+1
    const uint32_t xsum_q = smem_u32(xsum) + 8u * q;
    const uint32_t ring_u = smem_u32(ring);
    const uint32_t tab_w = smem_u32(tab + warp * 256);
    const uint32_t h1024 = 0x64006400u, h1152 = 0x64806480u;   // f16x2 (1024, 1024), (1152, 1152)

    int slot = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int grp = 0; grp < ngroups; ++grp) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};     // rows g, g+8 x tokens 2q, 2q+1
        for (int c = 0; c < a.nchunks; ++c) {
            if (ok) {
                const bool w = mbar_wait(&full[slot], ph, a.status);
                ok = __all_sync(0xffffffffu, w);
            }
            if (ok) {
                const uint32_t rA = ring_u + (uint32_t)slot * slot_bytes + (uint32_t)g * a.RS;
                const uint32_t rB = rA + 8u * a.RS;
                const int kc0 = c * a.KC;                 // first element of the chunk
                if constexpr (T == QT_Q8_0) {
                    const int npairs = a.KC / 64;
                    for (int p = warp; p < npairs; p += GM_CW) {
                        const uint32_t pA = rA + 68u * p, pB = rB + 68u * p;
                        const int blk0 = (kc0 >> 5) + 2 * p;
#pragma unroll
                        for (int hb = 0; hb < 2; ++hb) {          // block of the pair
                            uint32_t vA0, vA1, vB0, vB1;
                            if (hb == 0) {                        // quants at +2: 2 mod 4
                                const uint32_t o = 8u * q;
                                const uint32_t a0w = g_lds32(pA + o), a1w = g_lds32(pA + o + 4), a2w = g_lds32(pA + o + 8);
                                const uint32_t b0w = g_lds32(pB + o), b1w = g_lds32(pB + o + 4), b2w = g_lds32(pB + o + 8);
                                vA0 = __funnelshift_r(a0w, a1w, 16);
                                vA1 = __funnelshift_r(a1w, a2w, 16);
                                vB0 = __funnelshift_r(b0w, b1w, 16);
                                vB1 = __funnelshift_r(b1w, b2w, 16);
                            } else {                              // quants at 36: 4-byte aligned
                                const uint32_t o = 36u + 8u * q;
                                vA0 = g_lds32(pA + o);
                                vA1 = g_lds32(pA + o + 4);
                                vB0 = g_lds32(pB + o);
                                vB1 = g_lds32(pB + o + 4);
                            }
                            const uint32_t xo = 64u * (uint32_t)(blk0 + hb);
                            const uint4 bh = g_lds128(xh_t + xo), bl = g_lds128(xl_t + xo);
                            float cb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                            uint32_t a0, a2, a1, a3;
                            bytes_h2(vA0 ^ 0x80808080u, h1152, a0, a2);   // u = q + 128 -> q
                            bytes_h2(vB0 ^ 0x80808080u, h1152, a1, a3);
                            mma16816(cb, a0, a1, a2, a3, bh.x, bh.y);
                            mma16816(cb, a0, a1, a2, a3, bl.x, bl.y);
                            bytes_h2(vA1 ^ 0x80808080u, h1152, a0, a2);
                            bytes_h2(vB1 ^ 0x80808080u, h1152, a1, a3);
                            mma16816(cb, a0, a1, a2, a3, bh.z, bh.w);
                            mma16816(cb, a0, a1, a2, a3, bl.z, bl.w);
                            const uint32_t dA = g_lds32(pA + (hb ? 32u : 0u)), dB = g_lds32(pB + (hb ? 32u : 0u));
                            const float d0 = __half2float(__ushort_as_half((uint16_t)(hb ? dA >> 16 : dA & 0xffff)));
                            const float d1 = __half2float(__ushort_as_half((uint16_t)(hb ? dB >> 16 : dB & 0xffff)));
                            const float2 sc = g_lds64f(xsc_q + 32u * (uint32_t)(blk0 + hb));
                            acc[0] = fmaf(d0 * sc.x, cb[0], acc[0]);
                            acc[1] = fmaf(d0 * sc.y, cb[1], acc[1]);
                            acc[2] = fmaf(d1 * sc.x, cb[2], acc[2]);
                            acc[3] = fmaf(d1 * sc.y, cb[3], acc[3]);
                        }
                    }
                } else if constexpr (T == QT_Q6_K) {
                    // super-block (tier/quant.h:88-90): ql[128] low nibbles, qh[64]
                    // 2-bit high parts, sc[16] int8 per 16 elements, d fp16 at 208.
                    // Element e of half a (e < 128): ql byte 64a + (e & 63), nibble
                    // e >> 6; qh byte 128 + 32a + (e & 31), bits 2 (e >> 5).
                    const int nsb = a.KC / 256;
                    for (int sbi = warp; sbi < nsb; sbi += GM_CW) {
                        const uint32_t sA = rA + 210u * sbi, sB = rB + 210u * sbi;
                        const bool odd = (sbi & 1) != 0;
                        // d * sc of sub-blocks 4q .. 4q+3 for rows g and g+8 -> per-warp table [16 rows][16]
                        {
                            const uint32_t wA = g_lds32_a(sA + 192u + 4u * q, odd);
                            const uint32_t wB = g_lds32_a(sB + 192u + 4u * q, odd);
                            const float dA = __half2float(__ushort_as_half((uint16_t)g_lds16(sA + 208u)));
                            const float dB = __half2float(__ushort_as_half((uint16_t)g_lds16(sB + 208u)));
                            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(tab_w + 64u * g + 16u * q),
                                         "f"(dA * (float)(int8_t)(wA & 0xff)), "f"(dA * (float)(int8_t)((wA >> 8) & 0xff)),
                                         "f"(dA * (float)(int8_t)((wA >> 16) & 0xff)), "f"(dA * (float)(int8_t)(wA >> 24))
                                         : "memory");
                            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(tab_w + 64u * (g + 8) + 16u * q),
                                         "f"(dB * (float)(int8_t)(wB & 0xff)), "f"(dB * (float)(int8_t)((wB >> 8) & 0xff)),
                                         "f"(dB * (float)(int8_t)((wB >> 16) & 0xff)), "f"(dB * (float)(int8_t)(wB >> 24))
                                         : "memory");
                            __syncwarp();
                        }
                        const int sb_elem = kc0 + 256 * sbi;
                        const uint32_t h1056 = 0x64206420u;          // f16x2 (1056, 1056): 1024 + u - 1056 = q - 32
#pragma unroll 1
                        for (int ha = 0; ha < 2; ++ha) {              // 128-element half
                            // d * sc of this half's sub-blocks 8ha .. 8ha+7 (index 2 gq + w)
                            const float4 tA0 = g_lds128f(tab_w + 64u * g + 32u * ha);
                            const float4 tA1 = g_lds128f(tab_w + 64u * g + 32u * ha + 16u);
                            const float4 tB0 = g_lds128f(tab_w + 64u * (g + 8) + 32u * ha);
                            const float4 tB1 = g_lds128f(tab_w + 64u * (g + 8) + 32u * ha + 16u);
                            const float scA[8] = {tA0.x, tA0.y, tA0.z, tA0.w, tA1.x, tA1.y, tA1.z, tA1.w};
                            const float scB[8] = {tB0.x, tB0.y, tB0.z, tB0.w, tB1.x, tB1.y, tB1.z, tB1.w};
#pragma unroll
                            for (int w = 0; w < 2; ++w) {             // 16-element window of each 32-block
                                const uint32_t o = 64u * ha + 16u * w + 4u * q;
                                const uint32_t ho = 128u + 32u * ha + 16u * w + 4u * q;
                                const uint32_t l0A = g_lds32_a(sA + o, odd), l1A = g_lds32_a(sA + o + 32u, odd);
                                const uint32_t l0B = g_lds32_a(sB + o, odd), l1B = g_lds32_a(sB + o + 32u, odd);
                                const uint32_t hA = g_lds32_a(sA + ho, odd), hB = g_lds32_a(sB + ho, odd);
#pragma unroll
                                for (int gq = 0; gq < 4; ++gq) {      // 32-block gq of the half
                                    const uint32_t lA = gq & 1 ? l1A : l0A, lB = gq & 1 ? l1B : l0B;
                                    const uint32_t qA = ((lA >> (4 * (gq >> 1))) & 0x0F0F0F0Fu) |
                                                        (((hA >> (2 * gq)) & 0x03030303u) << 4);
                                    const uint32_t qB = ((lB >> (4 * (gq >> 1))) & 0x0F0F0F0Fu) |
                                                        (((hB >> (2 * gq)) & 0x03030303u) << 4);
                                    uint32_t a0, a1, a2, a3;
                                    bytes_h2(qA, h1056, a0, a2);
                                    bytes_h2(qB, h1056, a1, a3);
                                    const int e0 = sb_elem + 128 * ha + 32 * gq + 16 * w;
                                    const uint2 bh = g_lds64(xh6_t + 2u * (uint32_t)e0);
                                    const uint2 bl = g_lds64(xl6_t + 2u * (uint32_t)e0);
                                    float cb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                                    mma16816(cb, a0, a1, a2, a3, bh.x, bh.y);
                                    mma16816(cb, a0, a1, a2, a3, bl.x, bl.y);
                                    const float2 xs = g_lds64f(xsc_q + 32u * (uint32_t)(e0 >> 5));
                                    const float sa = scA[2 * gq + w], sb = scB[2 * gq + w];
                                    acc[0] = fmaf(sa * xs.x, cb[0], acc[0]);
                                    acc[1] = fmaf(sa * xs.y, cb[1], acc[1]);
                                    acc[2] = fmaf(sb * xs.x, cb[2], acc[2]);
                                    acc[3] = fmaf(sb * xs.y, cb[3], acc[3]);
                                }
                            }
                        }
                        __syncwarp();     // table reads done before the next super-block overwrites it
                    }
                } else {
                    constexpr uint32_t SB = T == QT_Q4_K ? 144u : 176u;
                    constexpr uint32_t QS = T == QT_Q4_K ? 16u : 48u;
                    const int nsb = a.KC / 256;
                    for (int sbi = warp; sbi < nsb; sbi += GM_CW) {
                        const uint32_t sA = rA + SB * sbi, sB = rB + SB * sbi;
                        // scales of sub-blocks 2q, 2q+1 for rows g and g+8 -> per-warp table
                        {
                            const uint4 hA = g_lds128(sA), hB = g_lds128(sB);
                            int sc0, mn0, sc1, mn1;
                            kq_scale_min_reg(2 * q, hA, sc0, mn0);
                            kq_scale_min_reg(2 * q + 1, hA, sc1, mn1);
                            float d = __half2float(__ushort_as_half((uint16_t)(hA.x & 0xffff)));
                            float dm = __half2float(__ushort_as_half((uint16_t)(hA.x >> 16)));
                            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(tab_w + 64u * g + 16u * q),
                                         "f"(d * small_u2f(sc0)), "f"(dm * small_u2f(mn0)), "f"(d * small_u2f(sc1)),
                                         "f"(dm * small_u2f(mn1))
                                         : "memory");
                            kq_scale_min_reg(2 * q, hB, sc0, mn0);
                            kq_scale_min_reg(2 * q + 1, hB, sc1, mn1);
                            d = __half2float(__ushort_as_half((uint16_t)(hB.x & 0xffff)));
                            dm = __half2float(__ushort_as_half((uint16_t)(hB.x >> 16)));
                            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(tab_w + 64u * (g + 8) + 16u * q),
                                         "f"(d * small_u2f(sc0)), "f"(dm * small_u2f(mn0)), "f"(d * small_u2f(sc1)),
                                         "f"(dm * small_u2f(mn1))
                                         : "memory");
                            __syncwarp();
                        }
                        const int sb_elem = kc0 + 256 * sbi;
#pragma unroll 1
                        for (int j = 0; j < 4; ++j) {             // sub-block pair 2j (low), 2j+1 (high)
                            float cl[4] = {0.0f, 0.0f, 0.0f, 0.0f}, chh[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                            const uint32_t o = QS + 32u * j + 8u * q;
                            const uint2 wA = g_lds64(sA + o), wB = g_lds64(sB + o);
                            uint2 qhA = make_uint2(0u, 0u), qhB = make_uint2(0u, 0u);
                            if constexpr (T == QT_Q5_K) {
                                qhA = g_lds64(sA + 16u + 8u * q);
                                qhB = g_lds64(sB + 16u + 8u * q);
                            }
                            const uint32_t xo = 2u * (uint32_t)(sb_elem + 64 * j);
                            const uint4 blo_h = g_lds128(xh_t + xo), blo_l = g_lds128(xl_t + xo);
                            const uint4 bhi_h = g_lds128(xh_t + xo + 64u), bhi_l = g_lds128(xl_t + xo + 64u);
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const uint32_t vA = h ? wA.y : wA.x, vB = h ? wB.y : wB.x;
                                uint32_t loA = vA & 0x0F0F0F0Fu, hiA = (vA >> 4) & 0x0F0F0F0Fu;
                                uint32_t loB = vB & 0x0F0F0F0Fu, hiB = (vB >> 4) & 0x0F0F0F0Fu;
                                if constexpr (T == QT_Q5_K) {
                                    const uint32_t hA5 = h ? qhA.y : qhA.x, hB5 = h ? qhB.y : qhB.x;
                                    loA |= ((hA5 >> (2 * j)) & 0x01010101u) << 4;
                                    hiA |= ((hA5 >> (2 * j + 1)) & 0x01010101u) << 4;
                                    loB |= ((hB5 >> (2 * j)) & 0x01010101u) << 4;
                                    hiB |= ((hB5 >> (2 * j + 1)) & 0x01010101u) << 4;
                                }
                                uint32_t a0, a1, a2, a3;
                                bytes_h2(loA, h1024, a0, a2);
                                bytes_h2(loB, h1024, a1, a3);
                                mma16816(cl, a0, a1, a2, a3, h ? blo_h.z : blo_h.x, h ? blo_h.w : blo_h.y);
                                mma16816(cl, a0, a1, a2, a3, h ? blo_l.z : blo_l.x, h ? blo_l.w : blo_l.y);
                                bytes_h2(hiA, h1024, a0, a2);
                                bytes_h2(hiB, h1024, a1, a3);
                                mma16816(chh, a0, a1, a2, a3, h ? bhi_h.z : bhi_h.x, h ? bhi_h.w : bhi_h.y);
                                mma16816(chh, a0, a1, a2, a3, h ? bhi_l.z : bhi_l.x, h ? bhi_l.w : bhi_l.y);
                            }
                            const float4 tA = g_lds128f(tab_w + 64u * g + 16u * j);        // a, m of 2j; a, m of 2j+1
                            const float4 tB = g_lds128f(tab_w + 64u * (g + 8) + 16u * j);
                            const int blk = (sb_elem >> 5) + 2 * j;
                            const float2 s0 = g_lds64f(xsc_q + 32u * blk), s1 = g_lds64f(xsc_q + 32u * (blk + 1));
                            const float2 x0 = g_lds64f(xsum_q + 32u * blk), x1 = g_lds64f(xsum_q + 32u * (blk + 1));
                            acc[0] = fmaf(tA.x * s0.x, cl[0], acc[0]);
                            acc[1] = fmaf(tA.x * s0.y, cl[1], acc[1]);
                            acc[2] = fmaf(tB.x * s0.x, cl[2], acc[2]);
                            acc[3] = fmaf(tB.x * s0.y, cl[3], acc[3]);
                            acc[0] = fmaf(-tA.y, x0.x, acc[0]);
                            acc[1] = fmaf(-tA.y, x0.y, acc[1]);
                            acc[2] = fmaf(-tB.y, x0.x, acc[2]);
                            acc[3] = fmaf(-tB.y, x0.y, acc[3]);
                            acc[0] = fmaf(tA.z * s1.x, chh[0], acc[0]);
                            acc[1] = fmaf(tA.z * s1.y, chh[1], acc[1]);
                            acc[2] = fmaf(tB.z * s1.x, chh[2], acc[2]);
                            acc[3] = fmaf(tB.z * s1.y, chh[3], acc[3]);
                            acc[0] = fmaf(-tA.w, x1.x, acc[0]);
                            acc[1] = fmaf(-tA.w, x1.y, acc[1]);
                            acc[2] = fmaf(-tB.w, x1.x, acc[2]);
                            acc[3] = fmaf(-tB.w, x1.y, acc[3]);
                        }
                        __syncwarp();     // table reads done before the next super-block overwrites it
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            if (++slot == a.nslots) { slot = 0; ph ^= 1u; }
        }
        // ---- sum the warps' partials in a fixed order ----
        float* pb = part + (size_t)(grp & 1) * GM_CW * 128;
        *reinterpret_cast<float2*>(pb + warp * 128 + g * 8 + 2 * q) = make_float2(acc[0], acc[1]);
        *reinterpret_cast<float2*>(pb + warp * 128 + (g + 8) * 8 + 2 * q) = make_float2(acc[2], acc[3]);
        asm volatile("bar.sync 1, %0;" ::"r"(GM_CW * 32) : "memory");
        if (ok && threadIdx.x < 16 * a.M) {
            const int r = threadIdx.x & 15, m = threadIdx.x >> 4;
            const int row = r_begin + grp * 16 + r;
            if (row < r_end) {
                float sum = 0.0f;
#pragma unroll 4
                for (int w = 0; w < GM_CW; ++w) sum += pb[w * 128 + r * 8 + m];
                a.y[(size_t)m * a.ldy + row] = sum;
            }
        }
        // the next group writes the other partial buffer; the barrier of the
        // following group orders these reads before that buffer's reuse
    }
}

// ---- host side ----
struct GmPlan {
    int KP, KC, nchunks, nslots, XS;
    uint32_t kcb, RS;
    size_t smem;
};


static uint32_t gm_block_bytes(int t) { return t == QT_Q8_0 ? 34u : t == QT_Q4_K ? 144u : t == QT_Q5_K ? 176u : 210u; }
static int gm_block_elems(int t) { return t == QT_Q8_0 ? 32 : 256; }

static bool gm_plan(int t, int N, int K, int M, int grid, GmPlan& p) {
    if (K % 256) return false;
    const int rows_blk = (N + grid - 1) / grid;
    const int ngroups = (rows_blk + 15) / 16;
    p.XS = K + 16;                               // x row: 2K + 32 bytes
    const int nblk = K / 32;
    const size_t fixed = 128 + 2 * (size_t)M * p.XS * 2 + 2 * (size_t)nblk * 8 * 4 + 2 * GM_CW * 16 * 8 * 4 +
                         GM_CW * 256 * 4 + 2 * GM_MAXSLOTS * 8 + 64;
    if (fixed >= GM_SMEM_MAX) return false;
    // K-chunks: the fewest (largest row copies: bulk copies stream faster the
    // larger they are) such that two 16-row slots fit
    const size_t slot_max = (GM_SMEM_MAX - fixed) / 2;
    const int units = K / 256;
    bool found = false;
    for (int nc = 1; nc <= units && !found; ++nc) {
        if (units % nc) continue;
        const int KC = K / nc;
        const uint32_t kcb = (uint32_t)((size_t)KC / gm_block_elems(t) * gm_block_bytes(t));
        if (kcb % 16u) continue;                 // bulk copies: 16-byte sizes and source offsets (Q6_K)
        uint32_t RS = (kcb + 15u) & ~15u;
        while (RS % 128u != 32u) RS += 16u;
        if (16u * (size_t)RS > slot_max) continue;
        p.KC = KC;
        p.nchunks = nc;
        p.kcb = kcb;
        p.RS = RS;
        found = true;
    }
    if (!found) return false;
    const size_t slot = 16u * (size_t)p.RS;
    int ns = (int)((GM_SMEM_MAX - fixed) / slot);
    if (ns > GM_MAXSLOTS) ns = GM_MAXSLOTS;
    const int need = ngroups * p.nchunks;
    if (ns > need) ns = need;
    if (ns < (need < 2 ? need : 2)) return false;
    p.nslots = ns;
    p.KP = 1;
    p.smem = fixed + (size_t)ns * slot;
    return p.smem <= GM_SMEM_MAX + 1024;
}

bool gemv_mma_ok(int t, size_t rb, int K, int M) {
    if (t != QT_Q8_0 && t != QT_Q4_K && t != QT_Q5_K && t != QT_Q6_K) return false;
    if (M < 1 || M > 8 || rb % 16 || K % 256) return false;
    GmPlan p;
    return gm_plan(t, 148 * 64, K, M, 148, p);
}

template <int T>
static tk_status go_mma(tk_ctx* ctx, const uint8_t* W, size_t rb, int N, int K, int M, const float* x, int ldx,
                        float* y, int ldy, bool frozen, cudaStream_t s) {
    const int grid = ctx->num_sms < N ? ctx->num_sms : N;
    GmPlan p;
    if (!gm_plan(T, N, K, M, grid, p)) return fail(TK_ERR_UNSUPPORTED, "gemv mma: shape does not fit shared memory");
    (void)rb;
    auto kern = gemv_mma_kernel<T>;
    static std::atomic<uint64_t> attr_done{0};   // per instantiation, one bit per device
    {
        const cudaError_t e = smem_attr_once(kern, (int)GM_SMEM_MAX + 1024, ctx->device, attr_done);
        if (e != cudaSuccess) return cuda_fail(e, "gemv mma smem attribute");
    }
    GmArgs a;
    a.W = W; a.rb = rb; a.N = N; a.K = K; a.M = M; a.x = x; a.ldx = ldx; a.y = y; a.ldy = ldy;
    a.KP = p.KP; a.KC = p.KC; a.nchunks = p.nchunks; a.kcb = p.kcb; a.RS = p.RS; a.nslots = p.nslots; a.XS = p.XS;
    a.frozen = frozen;
    a.status = ctx->status;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(GM_THREADS, 1, 1);
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
    if (e != cudaSuccess) return cuda_fail(e, "gemv mma launch");
    return cuda_fail(cudaGetLastError(), "gemv mma launch");
}

tk_status launch_gemv_mma(tk_ctx* ctx, int t, const void* Wv, size_t rb, int N, int K, const float* x, int ldx, int M,
                          float* y, int ldy, bool frozen, cudaStream_t s) {
    const uint8_t* W = static_cast<const uint8_t*>(Wv);
    if (t == QT_Q8_0) return go_mma<QT_Q8_0>(ctx, W, rb, N, K, M, x, ldx, y, ldy, frozen, s);
    if (t == QT_Q4_K) return go_mma<QT_Q4_K>(ctx, W, rb, N, K, M, x, ldx, y, ldy, frozen, s);
    if (t == QT_Q5_K) return go_mma<QT_Q5_K>(ctx, W, rb, N, K, M, x, ldx, y, ldy, frozen, s);
    if (t == QT_Q6_K) return go_mma<QT_Q6_K>(ctx, W, rb, N, K, M, x, ldx, y, ldy, frozen, s);
    return fail(TK_ERR_UNSUPPORTED, "gemv mma: type");
}

}  // namespace tk
