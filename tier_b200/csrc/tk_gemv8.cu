// tk_gemv8.cu -- decode GEMV for one token on Q8_0 rows with the integer
// dot-product instruction (dp4a), x held in registers.
//
// y[n] = sum_k W(n, k) x[k] (the reference's gemv_q, tier/tier.cpp:300-306,
// for M = 1).  At one token the GEMV only has to stream the weight once; the
// tensor-core designs (tk_gemv5/6.cu) spend their issue slots on fragment
// loads and per-tile bookkeeping for an MMA whose B operand is 1 of 8
// columns.  Here each lane owns a fixed run of K and keeps its part of x
// resident in registers for every row it sees, so the per-weight work is one
// byte-lane of a dp4a per x plane:
//
//  * x (once per CTA, into shared memory, then registers): per 32-element
//    block a power-of-two scale puts the block's max into [2^21, 2^22); the
//    scaled integer xi splits exactly into three signed bytes
//    xi = p0 * 2^16 + p1 * 2^8 + p2, packed four elements to a word per
//    plane.  Relative to the block's max x is kept to 2^-22.
//  * W: a row's blocks are split evenly over the 32 lanes (lane l takes JS
//    consecutive 34-byte blocks, JS <= 4, a compile-time count so a row's
//    blocks interleave freely); longer K is cut into segments owned by teams
//    of warps, whose partial sums meet in shared memory in a fixed order.  A
//    block's quants are realigned with one funnel shift per word (its start
//    is 0 or 2 mod 4) and enter dp4a as the int8 values they are; the three
//    plane sums are exact in int32 and combine in fp32:
//    acc += d * 2^-s * (I0 * 2^16 + (I1 * 2^8 + I2)).
//  * Rows: each CTA owns a contiguous row range and each warp a contiguous
//    part of it, which it streams through its own ring of row slots with one
//    bulk copy per (row, segment) -- no producer warp and no cross-warp
//    handshake: the warp that reads a slot refills it.  Programmatic
//    dependent launch: with TK_WFROZEN the weight copies start before the
//    preceding kernel has finished.
// A non-finite x element makes y non-finite (its block's scale is NaN).
// All waits are bounded (tk_device.cuh); a timeout records a status code.
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

constexpr int GD_CW = 8;                         // warps, each its own ring
constexpr int GD_THREADS = GD_CW * 32;
constexpr int GD_JMAX = 4;                       // blocks per lane held in registers (25 words each)
constexpr int GD_NSLOT = 4;                      // row slots per warp
constexpr size_t GD_SMEM_MAX = 220 * 1024;
constexpr uint32_t GD_XSEG = GD_JMAX * 6 * 32 * 16;   // x plane bytes per segment
constexpr uint32_t GD_SSEG = GD_JMAX * 32 * 4;        // x scale bytes per segment

struct GdArgs {
    const uint8_t* W;
    size_t rb;             // bytes per row (>= 34 K / 32, multiple of 16)
    int N, K;
    const float* x;
    float* y;
    int nseg;              // K segments; a team of GD_CW / nseg warps per segment
    int jseg;              // blocks per lane in a segment (the last may hold fewer)
    uint32_t slot_bytes;   // one row's segment: 34 * 32 * jseg, a multiple of 16
    uint32_t x_off, xs_off, part_off, bar_off;   // shared-memory offsets after the rings
    int frozen;
    int* status;
};

__device__ __forceinline__ uint32_t d_lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 d_lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ int dp4(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ void gd_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void gd_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Blocks per lane of segment s (segments cover K in order, 32 * jseg blocks each).
__device__ __forceinline__ int gd_js(const GdArgs& a, int s) {
    const int J = a.K >> 10;
    const int rest = J - s * a.jseg;
    return rest < a.jseg ? rest : a.jseg;
}

// One row: this lane's JS blocks at shared address rbase.
template <int JS>
__device__ __forceinline__ float gd_row(uint32_t rbase, const uint32_t (&xr)[GD_JMAX][24], const float (&xs)[GD_JMAX]) {
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < JS; ++j) {
        const uint32_t ab = rbase + 34u * j;
        const uint32_t a4 = ab & ~3u, o = ab & 3u;     // o is 0 or 2
        uint32_t w[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) w[i] = d_lds32(a4 + 4u * i);
        const uint32_t sh = 8u * (o + 2u);             // 16, or 32: the next word whole
        // two accumulators per plane: shorter dependent chains
        int I0 = 0, I1 = 0, I2 = 0, K0 = 0, K1 = 0, K2 = 0;
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            const uint32_t q = __funnelshift_rc(w[i], w[i + 1], sh);
            const uint32_t r = __funnelshift_rc(w[i + 1], w[i + 2], sh);
            I0 = dp4(q, xr[j][i], I0);
            I1 = dp4(q, xr[j][8 + i], I1);
            I2 = dp4(q, xr[j][16 + i], I2);
            K0 = dp4(r, xr[j][i + 1], K0);
            K1 = dp4(r, xr[j][9 + i], K1);
            K2 = dp4(r, xr[j][17 + i], K2);
        }
        const float d = __half2float(__ushort_as_half((uint16_t)(__funnelshift_r(w[0], w[1], 8u * o) & 0xffffu)));
        const float t = fmaf((float)(I0 + K0), 65536.0f, (float)((I1 + K1) * 256 + (I2 + K2)));
        acc = fmaf(d * xs[j], t, acc);
    }
    return acc;
}

template <int JS>
__global__ void __launch_bounds__(GD_THREADS, 1) gemv_dp_kernel(const __grid_constant__ GdArgs a) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* ring = sm + (size_t)warp * GD_NSLOT * a.slot_bytes;         // this warp's slots
    uint8_t* xq = sm + a.x_off;                                          // [seg][j][6 chunks][32 lanes][16 B]
    float* xsc = reinterpret_cast<float*>(sm + a.xs_off);                // [seg][j][32 lanes]
    float* part = reinterpret_cast<float*>(sm + a.part_off);             // [row][seg] (nseg > 1)
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + a.bar_off) + warp * GD_NSLOT;

    const int T = GD_CW / a.nseg;                // warps per segment team
    const int seg = warp / T, tw = warp - seg * T;
    const int js = gd_js(a, seg);
    const int r_begin = (int)((long long)a.N * blockIdx.x / gridDim.x);
    const int r_end = (int)((long long)a.N * (blockIdx.x + 1) / gridDim.x);
    const int nrows = r_end - r_begin;
    // this warp's rows: [w0, w0 + nw) of the CTA's rows
    const int w0 = nrows * tw / T, nw = nrows * (tw + 1) / T - w0;
    const uint32_t seg_off = (uint32_t)(seg * 32 * a.jseg) * 34u;       // the segment's bytes in a row
    const uint32_t seg_bytes = (uint32_t)(32 * js) * 34u;               // a multiple of 16

    gd_launch_dependents();
    if (lane == 0) {
        for (int i = 0; i < GD_NSLOT; ++i) mbar_init(&full[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    // the weight copies start first; they overlap the conversion of x
    if (lane == 0 && js > 0) {
        if (!a.frozen) gd_wait_prior();        // the weight may come from the preceding kernel
        for (int u = 0; u < nw && u < GD_NSLOT; ++u) {
            mbar_arrive_expect_tx(&full[u], seg_bytes);
            bulk_load(ring + (size_t)u * a.slot_bytes, a.W + (size_t)(r_begin + w0 + u) * a.rb + seg_off, seg_bytes,
                      &full[u]);
        }
    }

    // ---------------- x -> three int8 planes per 32-element block ----------------
    gd_wait_prior();                          // x may come from the preceding kernel
    const int tid = threadIdx.x;
    const int nb = a.K >> 5;
    const int ntask = nb * 8;                 // a multiple of GD_THREADS (K % 1024 == 0)
    for (int t0 = 0; t0 < ntask; t0 += 4 * GD_THREADS) {
        // up to four float4 loads in flight per thread before any is used
        float4 vv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int task = t0 + u * GD_THREADS + tid;
            if (task < ntask)
                vv[u] = __ldg(reinterpret_cast<const float4*>(a.x + (size_t)(task >> 3) * 32 + 4 * (task & 7)));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int task = t0 + u * GD_THREADS + tid;
            if (t0 + u * GD_THREADS >= ntask) break;   // uniform over the block
            const int n = task >> 3, w = task & 7;      // block n, elements 4w .. 4w+3
            const float4 v = vv[u];
            float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
            int bad = !(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w));
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                bad |= __shfl_xor_sync(0xffffffffu, bad, o);
            }
            int s = 0;
            if (mx > 0.0f && !bad) {
                // mx in [2^(E-127), 2^(E-126)): mx * 2^s in [2^21, 2^22)
                s = 148 - (int)((__float_as_uint(mx) >> 23) & 0xffu);
                if (s > 127) s = 127;
            }
            const float up = bad ? 0.0f : __uint_as_float((uint32_t)(127 + s) << 23);
            const float f[4] = {v.x, v.y, v.z, v.w};
            uint32_t p0 = 0, p1 = 0, p2 = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int xi = __float2int_rn(f[k] * up);      // |xi| <= 2^22
                const int b2 = (int)((uint32_t)xi << 24) >> 24;
                const int r1 = (xi - b2) >> 8;
                const int b1 = (int)((uint32_t)r1 << 24) >> 24;
                const int b0 = (r1 - b1) >> 8;                 // |b0| <= 64
                p0 |= ((uint32_t)b0 & 0xffu) << (8 * k);
                p1 |= ((uint32_t)b1 & 0xffu) << (8 * k);
                p2 |= ((uint32_t)b2 & 0xffu) << (8 * k);
            }
            // block n -> (segment, lane, j)
            const int sg = n / (32 * a.jseg);
            const int b0n = sg * 32 * a.jseg;
            const int jss = gd_js(a, sg);
            const int l = (n - b0n) / jss, j = (n - b0n) - l * jss;
            uint8_t* base = xq + (size_t)sg * GD_XSEG + (size_t)j * (6 * 32 * 16) + (size_t)l * 16 + (w & 3) * 4;
            const int c = w >> 2;                                          // word half of each plane
            *reinterpret_cast<uint32_t*>(base + (size_t)(0 + c) * 512) = p0;
            *reinterpret_cast<uint32_t*>(base + (size_t)(2 + c) * 512) = p1;
            *reinterpret_cast<uint32_t*>(base + (size_t)(4 + c) * 512) = p2;
            if (w == 0)
                xsc[(sg * GD_JMAX + j) * 32 + l] = bad ? __int_as_float(0x7fc00000) : ldexpf(1.0f, -s);
        }
    }
    __syncthreads();

    uint32_t xr[GD_JMAX][24];
    float xs[GD_JMAX];
#pragma unroll
    for (int j = 0; j < GD_JMAX; ++j) {
        if (j < js) {
            const uint32_t b = smem_u32(xq + (size_t)seg * GD_XSEG + (size_t)j * (6 * 32 * 16) + (size_t)lane * 16);
#pragma unroll
            for (int c = 0; c < 6; ++c) {
                const uint4 u = d_lds128(b + c * 512);
                xr[j][4 * c + 0] = u.x;
                xr[j][4 * c + 1] = u.y;
                xr[j][4 * c + 2] = u.z;
                xr[j][4 * c + 3] = u.w;
            }
            xs[j] = xsc[(seg * GD_JMAX + j) * 32 + lane];
        } else {
#pragma unroll
            for (int i = 0; i < 24; ++i) xr[j][i] = 0u;
            xs[j] = 0.0f;
        }
    }
    const uint32_t lane_off = (uint32_t)(lane * js) * 34u;   // this lane's blocks within the segment

    bool ok = js > 0;
    int u = 0;
    for (; u < nw && ok; ++u) {
        const int slot = u % GD_NSLOT;
        ok = mbar_wait(&full[slot], (uint32_t)(u / GD_NSLOT) & 1u, a.status);
        if (!ok) break;
        const uint32_t rbase = smem_u32(ring + (size_t)slot * a.slot_bytes) + lane_off;
        float acc;
        if (js == JS) acc = gd_row<JS>(rbase, xr, xs);        // every segment but a shorter last one
        else if (js == 1) acc = gd_row<1>(rbase, xr, xs);
        else if (js == 2) acc = gd_row<2>(rbase, xr, xs);
        else acc = gd_row<3>(rbase, xr, xs);
        // the slot's words are in registers and consumed: refill it
        __syncwarp();
        if (lane == 0 && u + GD_NSLOT < nw) {
            mbar_arrive_expect_tx(&full[slot], seg_bytes);
            bulk_load(ring + (size_t)slot * a.slot_bytes,
                      a.W + (size_t)(r_begin + w0 + u + GD_NSLOT) * a.rb + seg_off, seg_bytes, &full[slot]);
        }
#pragma unroll
        for (int o2 = 16; o2; o2 >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o2);
        if (lane == 0) {
            if (a.nseg == 1) a.y[r_begin + w0 + u] = acc;
            else part[(w0 + u) * a.nseg + seg] = acc;
        }
    }
    if (!ok && lane == 0 && js > 0) {
        // the copies in flight land before the block exits (bounded waits)
        for (int v = u; v < nw && v < u + GD_NSLOT; ++v)
            (void)mbar_wait(&full[v % GD_NSLOT], (uint32_t)(v / GD_NSLOT) & 1u, a.status);
    }
    if (a.nseg > 1) {
        __syncthreads();
        const int nused = ((a.K >> 10) + a.jseg - 1) / a.jseg;   // segments that hold blocks
        for (int r = tid; r < nrows; r += GD_THREADS) {
            float v = part[r * a.nseg];
            for (int s = 1; s < nused; ++s) v += part[r * a.nseg + s];
            a.y[r_begin + r] = v;
        }
    }
}

// ---------------------------------------------------------------------------
struct GdPlan {
    int nseg, jseg;
    uint32_t slot_bytes, x_off, xs_off, part_off, bar_off;
    size_t smem;
};

static bool gd_plan(int N, int K, size_t rb, int grid, GdPlan& p) {
    if (K % 1024 || K <= 0 || rb % 16 || rb < (size_t)K / 32 * 34) return false;
    const int J = K >> 10;
    p.nseg = 0;
    for (int ns : {1, 2, 4, 8}) {
        if ((J + ns - 1) / ns <= GD_JMAX) { p.nseg = ns; break; }
    }
    if (!p.nseg) return false;
    p.jseg = (J + p.nseg - 1) / p.nseg;
    const int rows_cta = (N + grid - 1) / grid;
    p.slot_bytes = (uint32_t)(34 * 32 * p.jseg);                  // 1088 * jseg: a multiple of 16
    const size_t rings = (size_t)GD_CW * GD_NSLOT * p.slot_bytes;
    p.x_off = (uint32_t)rings;
    p.xs_off = p.x_off + (uint32_t)(p.nseg * GD_XSEG);
    p.part_off = p.xs_off + (uint32_t)(p.nseg * GD_SSEG);
    p.bar_off = (p.part_off + (uint32_t)(p.nseg > 1 ? rows_cta * p.nseg * 4 : 0) + 15u) & ~15u;
    p.smem = (size_t)p.bar_off + (size_t)GD_CW * GD_NSLOT * 8 + 128;   // + alignment slack
    return p.smem <= GD_SMEM_MAX;
}

// Chosen over the tensor-core kernel (tk_gemv6.cu) from 32 MB of weight on:
// measured on B200 (graph replay, weight from HBM), q8_0 14336x4096 runs in
// 14.3 us here against 17.4 us there, while at 4096x4096 the fixed cost of a
// launch (first bytes, x staging) dominates and tk_gemv6.cu's 7.0 us beats
// 8.2 us here.
constexpr size_t GD_MIN_BYTES = 32u << 20;

bool gemv_dp_ok(int t, size_t rb, int N, int K, int M, int num_sms) {
    if (t != QT_Q8_0 || M != 1 || N <= 0 || (size_t)N * rb < GD_MIN_BYTES) return false;
    GdPlan p;
    return gd_plan(N, K, rb, num_sms < N ? num_sms : N, p);
}

template <int JS>
static tk_status go_dp(tk_ctx* ctx, const GdArgs& a, const GdPlan& p, int grid, cudaStream_t s) {
    static std::atomic<uint64_t> attr_done{0};   // per instantiation, one bit per device
    {
        const cudaError_t e = smem_attr_once(gemv_dp_kernel<JS>, (int)GD_SMEM_MAX, ctx->device, attr_done);
        if (e != cudaSuccess) return cuda_fail(e, "gemv dp4a smem attribute");
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(GD_THREADS, 1, 1);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ProfScope ps(ctx, s, PK_GEMV);
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_dp_kernel<JS>, a);
    ctx->launches++;
    if (e != cudaSuccess) return cuda_fail(e, "gemv dp4a launch");
    return cuda_fail(cudaGetLastError(), "gemv dp4a launch");
}

tk_status launch_gemv_dp(tk_ctx* ctx, const void* W, size_t rb, int N, int K, const float* x, float* y, bool frozen,
                         cudaStream_t s) {
    const int grid = ctx->num_sms < N ? ctx->num_sms : N;
    GdPlan p;
    if (!gd_plan(N, K, rb, grid, p)) return fail(TK_ERR_UNSUPPORTED, "gemv dp4a: shape does not fit shared memory");
    GdArgs a;
    a.W = static_cast<const uint8_t*>(W);
    a.rb = rb;
    a.N = N;
    a.K = K;
    a.x = x;
    a.y = y;
    a.nseg = p.nseg;
    a.jseg = p.jseg;
    a.slot_bytes = p.slot_bytes;
    a.x_off = p.x_off;
    a.xs_off = p.xs_off;
    a.part_off = p.part_off;
    a.bar_off = p.bar_off;
    a.frozen = frozen;
    a.status = ctx->status;
    switch (p.jseg) {
        case 1: return go_dp<1>(ctx, a, p, grid, s);
        case 2: return go_dp<2>(ctx, a, p, grid, s);
        case 3: return go_dp<3>(ctx, a, p, grid, s);
        default: return go_dp<4>(ctx, a, p, grid, s);
    }
}

}  // namespace tk
