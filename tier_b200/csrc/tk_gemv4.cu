// tk_gemv4.cu -- streaming decode GEMV for Q8_0 / Q4_K / Q5_K rows, M <= 4.
//
// y[m, n] = sum_k W(n, k) x[m, k].  HBM-bound: every weight byte is read once.
//
//  * One block per SM owns a contiguous range of rows (N / grid, any count, so
//    the per-SM byte counts differ by at most one row).  A producer warp
//    streams the rows through a ring of shared-memory slots with
//    cp.async.bulk (a slot holds R whole rows, one copy, completion on an
//    mbarrier); with the C1 shape every byte of the block is in flight from
//    the first microsecond.
//  * Sixteen consumer warps take (row, K-part) items round-robin, with no
//    block-wide barrier: each item's partial dot product goes to shared
//    memory, and the warp that finishes a row's last part (a shared-memory
//    counter) sums the parts in a fixed order and writes y.  Results are
//    deterministic.  A slot is handed back to the producer when every item
//    of it has arrived on the slot's "empty" mbarrier.
//  * x (fp32) is staged in shared memory once per block, permuted so that
//    each lane's two float4 reads per 256-element chunk are conflict-free.
//  * Integer quants become floats exactly with the 2^23 magic number: a
//    byte permute places the quant in the mantissa of 2^23 (one PRMT per
//    element), then a packed f32x2 subtraction removes the offset.  Dot
//    products use packed f32x2 FMA (sm_100).
//  * Per lane and sub-block the dot product is factored as
//      sum_j (a q_j - m) x_j = a * sum_j q_j x_j - m * sum_j x_j
//    (Q8_0: m = 0).  The reference (tier/tier.cpp:300-306) forms every
//    weight with q_val and accumulates weight*x; the results agree to fp32
//    rounding (the decode tolerance is 2e-3 relative).
//  * Programmatic dependent launch: the kernel lets the next kernel in the
//    stream start launching at once, and waits (griddepcontrol.wait) for the
//    previous one before it reads any global memory, so back-to-back decode
//    GEMVs do not pay the launch gap.
#include "tk_device.cuh"
#include "tk_internal.h"

#include <cmath>

namespace tk {

constexpr int GV_CW = 12;                       // consumer warps
constexpr int GV_THREADS = (GV_CW + 1) * 32;    // + one producer warp
constexpr int GV_MAXSLOTS = 24;
// Two blocks fit on one SM (registers and shared memory), so the next
// kernel's block can start streaming its weights while this one finishes.
constexpr size_t GV_SMEM_SMALL = 100 * 1024;
constexpr size_t GV_SMEM_MAX = 220 * 1024;      // one block per SM (large x)

struct GvArgs {
    const uint8_t* W;
    size_t rb;
    int N, K;
    const float* x;
    int ldx;
    float* y;
    int ldy;
    int R;            // rows per slot
    int nslots;
    int kp;           // parts per row
    int cpp;          // 256-element chunks per part
    uint32_t slot_bytes;
    int x_vec;        // x 16-byte aligned with ldx % 4 == 0
    int frozen;       // W is not written by earlier kernels: fetch it before griddepcontrol.wait
    int* status;
};

// ---- packed f32x2 arithmetic (sm_100) ----
typedef unsigned long long f2;
__device__ __forceinline__ f2 pk(float a, float b) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float2 upk(f2 v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
    f2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ void lds_f2x2(const float* p, f2& lo, f2& hi) {   // 16-byte shared load
    asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(lo), "=l"(hi) : "r"(smem_u32(p)));
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint16_t lds16(uint32_t addr) {
    uint16_t v;
    asm volatile("ld.shared.b16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

// Exact floats (2^23 + byte) of the four bytes of w, as two packed pairs
// with 2^23 + off subtracted: the values (byte - off).
__device__ __forceinline__ void bytes_to_f2(uint32_t w, float off, f2& p01, f2& p23) {
    const uint32_t m = 0x4B000000u;
    const float f0 = __uint_as_float(__byte_perm(w, m, 0x7440));
    const float f1 = __uint_as_float(__byte_perm(w, m, 0x7441));
    const float f2v = __uint_as_float(__byte_perm(w, m, 0x7442));
    const float f3 = __uint_as_float(__byte_perm(w, m, 0x7443));
    const f2 c = pk(-(8388608.0f + off), -(8388608.0f + off));
    p01 = add2(pk(f0, f1), c);
    p23 = add2(pk(f2v, f3), c);
}

// Element of row chunk c held at permuted position (h, lane, i):
// lane's first four (h = 0) or second four (h = 1) elements.
template <int T>
__device__ __forceinline__ int perm_src(int lane, int h, int i) {
    if constexpr (T == QT_Q8_0) return 8 * lane + 4 * h + i;                       // 8 consecutive
    else return 64 * (lane >> 3) + 32 * h + 4 * (lane & 7) + i;                    // lo / hi nibble groups
}

// One 256-element chunk of one row: acc[m] += this lane's 8 products.
template <int T, int M>
__device__ __forceinline__ void chunk_dot(uint32_t rowp, int c, const float* xs, int K, int lane, f2 (&acc)[M]) {
    const float* xc = xs + c * 256 + 4 * lane;
    if constexpr (T == QT_Q8_0) {
        const uint32_t bp = rowp + (uint32_t)(c * 8 + (lane >> 2)) * 34u;   // block of this lane
        const float d = __half2float(__ushort_as_half(lds16(bp)));
        const uint32_t qa = bp + 2 + 8 * (lane & 3);                       // 2-byte aligned
        const uint32_t al = qa & ~3u, sh = (qa & 2u) * 8u;
        const uint32_t w0 = lds32(al), w1 = lds32(al + 4), w2 = lds32(al + 8);
        const uint32_t lo = __funnelshift_r(w0, w1, sh) ^ 0x80808080u;
        const uint32_t hi = __funnelshift_r(w1, w2, sh) ^ 0x80808080u;
        f2 q01, q23, q45, q67;
        bytes_to_f2(lo, 128.0f, q01, q23);
        bytes_to_f2(hi, 128.0f, q45, q67);
        const f2 d2 = pk(d, d);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            f2 xa0, xa1, xb0, xb1;
            lds_f2x2(xc + (size_t)m * K, xa0, xa1);
            lds_f2x2(xc + (size_t)m * K + 128, xb0, xb1);
            f2 s = mul2(q01, xa0);
            s = fma2(q23, xa1, s);
            s = fma2(q45, xb0, s);
            s = fma2(q67, xb1, s);
            acc[m] = fma2(d2, s, acc[m]);
        }
    } else {
        constexpr int SB = T == QT_Q4_K ? 144 : 176;
        constexpr int QS = T == QT_Q4_K ? 16 : 48;
        const uint32_t sbp = rowp + (uint32_t)c * SB;
        const uint4 hdr = lds128(sbp);
        const int j = lane >> 3, lam = lane & 7;
        const uint32_t w = lds32(sbp + QS + 32 * j + 4 * lam);
        uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
        if constexpr (T == QT_Q5_K) {
            const uint32_t hb = lds32(sbp + 16 + 4 * lam);
            lo |= ((hb >> (2 * j)) & 0x01010101u) << 4;
            hi |= ((hb >> (2 * j + 1)) & 0x01010101u) << 4;
        }
        f2 l01, l23, h01, h23;
        bytes_to_f2(lo, 0.0f, l01, l23);
        bytes_to_f2(hi, 0.0f, h01, h23);
        int sc0, mn0, sc1, mn1;
        kq_scale_min_reg(2 * j, hdr, sc0, mn0);
        kq_scale_min_reg(2 * j + 1, hdr, sc1, mn1);
        const float d = __half2float(__ushort_as_half((uint16_t)(hdr.x & 0xffff)));
        const float dm = __half2float(__ushort_as_half((uint16_t)(hdr.x >> 16)));
        // (d * sc) and (dmin * m) are exact in fp32, as in the reference
        const float a0 = d * small_u2f(sc0), a1 = d * small_u2f(sc1);
        const float m0 = dm * small_u2f(mn0), m1 = dm * small_u2f(mn1);
        const f2 a02 = pk(a0, a0), a12 = pk(a1, a1), nm02 = pk(-m0, -m0), nm12 = pk(-m1, -m1);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            f2 xa0, xa1, xb0, xb1;
            lds_f2x2(xc + (size_t)m * K, xa0, xa1);
            lds_f2x2(xc + (size_t)m * K + 128, xb0, xb1);
            f2 s0 = mul2(l01, xa0);
            s0 = fma2(l23, xa1, s0);
            f2 s1 = mul2(h01, xb0);
            s1 = fma2(h23, xb1, s1);
            const f2 x0 = add2(xa0, xa1), x1 = add2(xb0, xb1);
            acc[m] = fma2(a02, s0, acc[m]);
            acc[m] = fma2(nm02, x0, acc[m]);
            acc[m] = fma2(a12, s1, acc[m]);
            acc[m] = fma2(nm12, x1, acc[m]);
        }
    }
}

__device__ __forceinline__ void gdc_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void gdc_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <int T, int M>
__global__ void __launch_bounds__(GV_THREADS, 2) gemv_sk_kernel(const __grid_constant__ GvArgs a) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* ring = sm;
    float* xs = reinterpret_cast<float*>(ring + (size_t)a.nslots * a.slot_bytes + 128);   // +128: tail over-read pad
    float* part = xs + (size_t)M * a.K;                        // [nslots][R][kp][M]
    int* cnt = reinterpret_cast<int*>(part + (size_t)a.nslots * a.R * a.kp * M);   // [nslots][R]
    uint64_t* full = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(cnt + a.nslots * a.R) + 7) & ~uintptr_t(7));
    uint64_t* empty = full + a.nslots;

    const int r_begin = (int)((long long)a.N * blockIdx.x / gridDim.x);
    const int r_end = (int)((long long)a.N * (blockIdx.x + 1) / gridDim.x);
    const int nrows = r_end - r_begin;
    const int nst = (nrows + a.R - 1) / a.R;

    gdc_launch_dependents();
    if (threadIdx.x == 0) {
        for (int i = 0; i < a.nslots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], a.R * a.kp);
        }
        fence_mbar_init();
    }
    for (int i = threadIdx.x; i < a.nslots * a.R; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    // Nothing global is touched before the previous kernel in the stream is
    // done, except a frozen weight, which no kernel writes.
    if (!(a.frozen && warp == GV_CW)) gdc_wait();

    if (warp == GV_CW) {
        // ---------------- producer ----------------
        if (lane == 0) {
            bool ok = true;
            int issued = 0;
            for (int st = 0; st < nst && ok; ++st) {
                const int slot = st % a.nslots;
                if (st >= a.nslots && !mbar_wait(&empty[slot], (uint32_t)((st / a.nslots) - 1) & 1u, a.status)) {
                    ok = false;
                    break;
                }
                const int r0 = r_begin + st * a.R;
                const int nr = r_end - r0 < a.R ? r_end - r0 : a.R;
                const uint32_t bytes = (uint32_t)((size_t)nr * a.rb);
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_load(ring + (size_t)slot * a.slot_bytes, a.W + (size_t)r0 * a.rb, bytes, &full[slot]);
                issued = st + 1;
            }
            if (!ok) {
                // copies still in flight land before the block exits (bounded): the
                // last nslots uses issued (earlier ones were consumed before reuse)
                const int first = issued > a.nslots ? issued - a.nslots : 0;
                for (int st = first; st < issued; ++st)
                    (void)mbar_wait(&full[st % a.nslots], (uint32_t)(st / a.nslots) & 1u, a.status);
            }
        }
        return;
    }

    // ---------------- consumers: stage x (permuted) ----------------
    // Both permutations move whole float4s: source float4 (c, s4) -> the
    // destination float4 of lane l, half h.  All loads are issued before any
    // store so they overlap.
    {
        const int total4 = M * a.K / 4;
        constexpr int PER = 4;   // float4 loads in flight per thread
        if (a.x_vec) {
            for (int base = 0; base < total4; base += PER * GV_CW * 32) {
                float4 v[PER];
#pragma unroll
                for (int u = 0; u < PER; ++u) {
                    const int f = base + threadIdx.x + u * GV_CW * 32;
                    if (f < total4) {
                        const int m = f / (a.K / 4), e = (f - m * (a.K / 4)) * 4;
                        v[u] = __ldg(reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx + e));
                    }
                }
#pragma unroll
                for (int u = 0; u < PER; ++u) {
                    const int f = base + threadIdx.x + u * GV_CW * 32;
                    if (f < total4) {
                        const int m = f / (a.K / 4), e = (f - m * (a.K / 4)) * 4;
                        const int c = e >> 8, r = e & 255;
                        int l, h;
                        if constexpr (T == QT_Q8_0) { l = r >> 3; h = (r >> 2) & 1; }
                        else { l = 8 * (r >> 6) + ((r & 31) >> 2); h = (r >> 5) & 1; }
                        *reinterpret_cast<float4*>(xs + (size_t)m * a.K + c * 256 + 128 * h + 4 * l) = v[u];
                    }
                }
            }
        } else {
            const int total = M * a.K;
            for (int idx = threadIdx.x; idx < total; idx += GV_CW * 32) {
                const int m = idx / a.K, e = idx - m * a.K;
                const int c = e >> 8, r = e & 255, h = r >> 7, l = (r & 127) >> 2, i = r & 3;
                xs[idx] = a.x[(size_t)m * a.ldx + c * 256 + perm_src<T>(l, h, i)];
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(GV_CW * 32) : "memory");
    }

    const int items = nrows * a.kp;
    bool ok = true;
    // item it = (row rl, part p); rows rl sit in stage rl / R, slot stage % nslots
    int rl = warp / a.kp, p = warp - rl * a.kp;
    int st = rl / a.R, ri = rl - st * a.R, slot = st % a.nslots;
    uint32_t ph = (uint32_t)(st / a.nslots) & 1u;
    const int drl = GV_CW / a.kp, dp = GV_CW - drl * a.kp;   // step of 16 items
    for (int it = warp; it < items && ok; it += GV_CW) {
        const bool w = mbar_wait(&full[slot], ph, a.status);
        if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
        const uint32_t rowp = smem_u32(ring + (size_t)slot * a.slot_bytes + (size_t)ri * a.rb);
        f2 acc[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = 0ull;
        const int c0 = p * a.cpp, c1 = c0 + a.cpp;
#pragma unroll 2
        for (int c = c0; c < c1; ++c) chunk_dot<T, M>(rowp, c, xs, a.K, lane, acc);
        float v[M];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float2 t = upk(acc[m]);
            float s = t.x + t.y;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            v[m] = s;
        }
        float* pp = part + ((size_t)(slot * a.R + ri) * a.kp + p) * M;
        int last = 0;
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < M; ++m) pp[m] = v[m];
            __threadfence_block();
            last = atomicAdd(&cnt[slot * a.R + ri], 1) == a.kp - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            if (lane < M) {
                const float* pr = part + (size_t)(slot * a.R + ri) * a.kp * M + lane;
                float s = 0.0f;
                for (int q = 0; q < a.kp; ++q) s += pr[q * M];
                a.y[(size_t)lane * a.ldy + r_begin + rl] = s;
            }
            if (lane == 0) cnt[slot * a.R + ri] = 0;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        // advance by GV_CW items
        p += dp;
        rl += drl;
        if (p >= a.kp) { p -= a.kp; ++rl; }
        ri = rl - st * a.R;
        while (ri >= a.R) {
            ri -= a.R;
            ++st;
            if (++slot == a.nslots) { slot = 0; ph ^= 1u; }
        }
    }
}

// ---- host side ----
struct GvPlan {
    int R, nslots, kp, cpp;
    uint32_t slot_bytes;
    size_t smem;
};

static size_t gv_smem(const GvPlan& p, int M, int K) {
    return 128 + (size_t)p.nslots * p.slot_bytes + 128 + (size_t)M * K * 4 + (size_t)p.nslots * p.R * p.kp * M * 4 +
           (size_t)p.nslots * p.R * 4 + 8 + 2 * (size_t)p.nslots * 8;
}

static bool gv_plan_budget(size_t rb, int N, int K, int M, int grid, size_t budget, GvPlan& p) {
    const int chunks = K / 256;
    const int rows_blk = (N + grid - 1) / grid;
    // parts per row: the split of (row, part) items over the consumer warps
    // with the least imbalance (ceil(items / warps) / (items / warps)), at
    // least 2 chunks per part; ties go to fewer parts
    int kp = 1;
    double best = 1e30;
    for (int c = 1; c <= 16 && chunks / c >= 2; c *= 2) {
        if (chunks % c) continue;
        const double items = (double)rows_blk * c;
        const double imb = std::ceil(items / GV_CW) / (items / GV_CW);
        if (imb < best - 0.02) { best = imb; kp = c; }
    }
    p.kp = kp;
    p.cpp = chunks / kp;
    // rows per slot: about 16 KB per copy
    int R = (int)(16384 / rb);
    if (R < 1) R = 1;
    if (R > 8) R = 8;
    if (R > rows_blk) R = rows_blk;
    p.R = R;
    p.slot_bytes = (uint32_t)(((size_t)R * rb + 127) & ~size_t(127));
    const size_t fixed = 128 + 128 + (size_t)M * K * 4 + 64;
    if (fixed >= budget) return false;
    const size_t per_slot = p.slot_bytes + (size_t)R * kp * M * 4 + (size_t)R * 4 + 16;
    int ns = (int)((budget - fixed) / per_slot);
    if (ns > GV_MAXSLOTS) ns = GV_MAXSLOTS;
    const int need = (rows_blk + R - 1) / R;
    if (ns > need) ns = need;
    // at least two slots (one when a single slot holds every row), and at
    // least 32 KB in flight unless that is everything
    if (ns < (need < 2 ? need : 2)) return false;
    if (ns < need && (size_t)ns * p.slot_bytes < 32 * 1024) return false;
    p.nslots = ns;
    p.smem = gv_smem(p, M, K);
    return p.smem <= budget + 1024;
}

static bool gv_plan(size_t rb, int N, int K, int M, int grid, GvPlan& p) {
    return gv_plan_budget(rb, N, K, M, grid, GV_SMEM_SMALL, p) || gv_plan_budget(rb, N, K, M, grid, GV_SMEM_MAX, p);
}

bool gemv_stream_ok(int t, size_t rb, int K, int M) {
    if (t != QT_Q8_0 && t != QT_Q4_K && t != QT_Q5_K) return false;
    if (M > 4 || M == 3 || rb % 16 || K % 256) return false;
    GvPlan p;
    return gv_plan(rb, 148 * 64, K, M, 148, p);   // shape-independent part of the plan fits
}

template <int T, int M>
static tk_status go_sk(tk_ctx* ctx, const uint8_t* W, size_t rb, int N, int K, const float* x, int ldx, float* y,
                       int ldy, bool frozen, cudaStream_t s) {
    int grid = ctx->num_sms;
    if (grid > N) grid = N;
    GvPlan p;
    if (!gv_plan(rb, N, K, M, grid, p)) return fail(TK_ERR_UNSUPPORTED, "gemv stream: shape does not fit shared memory");
    auto kern = gemv_sk_kernel<T, M>;
    static std::atomic<uint64_t> attr_done{0};   // per instantiation, one bit per device
    {
        const cudaError_t e = smem_attr_once(kern, (int)GV_SMEM_MAX + 1024, ctx->device, attr_done);
        if (e != cudaSuccess) return cuda_fail(e, "gemv smem attribute");
    }
    GvArgs a;
    a.W = W; a.rb = rb; a.N = N; a.K = K; a.x = x; a.ldx = ldx; a.y = y; a.ldy = ldy;
    a.R = p.R; a.nslots = p.nslots; a.kp = p.kp; a.cpp = p.cpp; a.slot_bytes = p.slot_bytes;
    a.x_vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && ldx % 4 == 0;
    a.frozen = frozen;
    a.status = ctx->status;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(GV_THREADS, 1, 1);
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
    if (e != cudaSuccess) return cuda_fail(e, "gemv stream launch");
    return cuda_fail(cudaGetLastError(), "gemv stream launch");
}

tk_status launch_gemv_stream(tk_ctx* ctx, int t, const void* Wv, size_t rb, int N, int K, const float* x, int ldx,
                             int M, float* y, int ldy, bool frozen, cudaStream_t s) {
    const uint8_t* W = static_cast<const uint8_t*>(Wv);
#define TK_G4(TT)                                                                   \
    if (t == TT) {                                                                  \
        if (M == 1) return go_sk<TT, 1>(ctx, W, rb, N, K, x, ldx, y, ldy, frozen, s);       \
        if (M == 2) return go_sk<TT, 2>(ctx, W, rb, N, K, x, ldx, y, ldy, frozen, s);       \
        return go_sk<TT, 4>(ctx, W, rb, N, K, x, ldx, y, ldy, frozen, s);                   \
    }
    TK_G4(QT_Q8_0)
    TK_G4(QT_Q4_K)
    TK_G4(QT_Q5_K)
#undef TK_G4
    return fail(TK_ERR_UNSUPPORTED, "gemv stream: type");
}

}  // namespace tk
