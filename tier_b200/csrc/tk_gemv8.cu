// tk_gemv8.cu -- decode GEMV for one token on Q8_0 rows with the integer
// dot-product instruction (dp4a), x held in registers.
//
// y[n] = sum_k W(n, k) x[k] (the reference's gemv_q, tier/tier.cpp:300-306,
// for M = 1).  At one token the GEMV only has to stream the weight once; the
// tensor-core designs (tk_gemv5/6.cu) spend their issue slots on fragment
// loads and per-tile bookkeeping for an MMA whose B operand is 1 of 8
// columns.  Here each lane owns a fixed run of K and keeps its part of x
// resident in registers for every row of the CTA, so the per-weight work is
// one byte-lane of a dp4a per x plane:
//
//  * x (once per CTA, into shared memory, then registers): per 32-element
//    block a power-of-two scale puts the block's max into [2^21, 2^22); the
//    scaled integer xi splits exactly into three signed bytes
//    xi = p0 * 2^16 + p1 * 2^8 + p2, packed four elements to a word per
//    plane.  Relative to the block's max x is kept to 2^-22.
//  * W: a row's blocks are split evenly over the 32 lanes (lane l takes J
//    consecutive 34-byte blocks); K beyond 4 blocks per lane is cut into
//    segments owned by teams of warps, whose partial sums meet in shared
//    memory in a fixed order.  A block's quants are realigned with one funnel
//    shift per word (its start is 0 or 2 mod 4) and enter dp4a as the int8
//    values they are; the three plane sums are exact in int32 and combine
//    in fp32: acc += d * 2^-s * (I0 * 2^16 + (I1 * 2^8 + I2)).
//  * Rows: each CTA owns a contiguous row range; a producer warp streams it
//    through a ring of slots, R whole rows per slot in one bulk copy (the
//    rows are contiguous in W), and the consumer warps take the rows of a
//    slot in turn.  Programmatic dependent launch: with TK_WFROZEN the
//    weight copies start before the preceding kernel has finished.
// A non-finite x element makes y non-finite (its block's scale is NaN).
// All waits are bounded (tk_device.cuh); a timeout records a status code.
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

constexpr int GD_CW = 8;                         // consumer warps
constexpr int GD_THREADS = (GD_CW + 1) * 32;     // + one producer warp
constexpr int GD_JMAX = 4;                       // blocks per lane held in registers (25 words each)
constexpr int GD_MAXSLOTS = 8;
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
    int R;                 // rows per slot
    int nslots;
    uint32_t xs_off, part_off, bar_off;   // shared-memory offsets after the ring
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
__device__ __forceinline__ void gd_bar_consumers() { asm volatile("bar.sync 1, %0;" ::"n"(GD_CW * 32) : "memory"); }
__device__ __forceinline__ void gd_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void gd_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Blocks per lane of segment s (segments cover K in order, 32 * jseg blocks each).
__device__ __forceinline__ int gd_js(const GdArgs& a, int s) {
    const int J = a.K >> 10;
    const int rest = J - s * a.jseg;
    return rest < a.jseg ? rest : a.jseg;
}

__global__ void __launch_bounds__(GD_THREADS, 1) gemv_dp_kernel(const __grid_constant__ GdArgs a) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t slot_bytes = (uint32_t)a.R * (uint32_t)a.rb;
    uint8_t* ring = sm;
    uint8_t* xq = sm + (size_t)a.nslots * slot_bytes;                 // [seg][j][6 chunks][32 lanes][16 B]
    float* xsc = reinterpret_cast<float*>(sm + a.xs_off);              // [seg][j][32 lanes]
    float* part = reinterpret_cast<float*>(sm + a.part_off);           // [row][seg] (nseg > 1)
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + a.bar_off);
    uint64_t* empty = full + a.nslots;

    const int r_begin = (int)((long long)a.N * blockIdx.x / gridDim.x);
    const int r_end = (int)((long long)a.N * (blockIdx.x + 1) / gridDim.x);
    const int nrows = r_end - r_begin;
    const int nst = (nrows + a.R - 1) / a.R;

    gd_launch_dependents();
    if (threadIdx.x == 0) {
        for (int i = 0; i < a.nslots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], GD_CW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == GD_CW) {
        // ---------------- producer: R whole rows per slot, one bulk copy ----------------
        if (lane != 0) return;
        if (!a.frozen) gd_wait_prior();       // the weight may come from the preceding kernel
        bool ok = true;
        int issued = 0;
        for (int st = 0; st < nst && ok; ++st) {
            const int slot = st % a.nslots;
            if (st >= a.nslots) ok = mbar_wait(&empty[slot], (uint32_t)((st / a.nslots) - 1) & 1u, a.status);
            if (!ok) break;
            const int rows = nrows - st * a.R < a.R ? nrows - st * a.R : a.R;
            const uint32_t bytes = (uint32_t)rows * (uint32_t)a.rb;
            mbar_arrive_expect_tx(&full[slot], bytes);
            bulk_load(ring + (size_t)slot * slot_bytes, a.W + (size_t)(r_begin + st * a.R) * a.rb, bytes, &full[slot]);
            issued = st + 1;
        }
        if (!ok) {
            // the copies in flight land before the block exits (bounded waits)
            for (int st = issued - a.nslots < 0 ? 0 : issued - a.nslots; st < issued; ++st)
                (void)mbar_wait(&full[st % a.nslots], (uint32_t)(st / a.nslots) & 1u, a.status);
        }
        return;
    }

    // ---------------- consumers: x -> three int8 planes per 32-element block ----------------
    gd_wait_prior();                          // x may come from the preceding kernel
    const int tid = threadIdx.x;              // 0 .. GD_CW*32-1
    const int nb = a.K >> 5;
    for (int task = tid; task < nb * 8; task += GD_CW * 32) {
        const int n = task >> 3, w = task & 7;                        // block n, elements 4w .. 4w+3
        const float4 v = __ldg(reinterpret_cast<const float4*>(a.x + (size_t)n * 32 + 4 * w));
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
        const int seg = n / (32 * a.jseg);
        const int b0n = seg * 32 * a.jseg;
        const int js = gd_js(a, seg);
        const int l = (n - b0n) / js, j = (n - b0n) - l * js;
        uint8_t* base = xq + (size_t)seg * GD_XSEG + (size_t)j * (6 * 32 * 16) + (size_t)l * 16 + (w & 3) * 4;
        const int c = w >> 2;                                          // word half of each plane
        *reinterpret_cast<uint32_t*>(base + (size_t)(0 + c) * 512) = p0;
        *reinterpret_cast<uint32_t*>(base + (size_t)(2 + c) * 512) = p1;
        *reinterpret_cast<uint32_t*>(base + (size_t)(4 + c) * 512) = p2;
        if (w == 0)
            xsc[(seg * GD_JMAX + j) * 32 + l] = bad ? __int_as_float(0x7fc00000) : ldexpf(1.0f, -s);
    }
    gd_bar_consumers();

    const int T = GD_CW / a.nseg;                // warps per segment team
    const int seg = warp / T, tw = warp - seg * T;
    const int js = gd_js(a, seg);
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
    // this lane's bytes of a row: blocks [seg*32*jseg + lane*js, + js)
    const uint32_t lane_off = (uint32_t)(seg * 32 * a.jseg + lane * js) * 34u;

    bool ok = true;
    for (int st = 0; st < nst; ++st) {
        const int slot = st % a.nslots;
        if (ok) ok = mbar_wait(&full[slot], (uint32_t)(st / a.nslots) & 1u, a.status);
        if (ok) {
            const int rows = nrows - st * a.R < a.R ? nrows - st * a.R : a.R;
            const uint32_t sbase = smem_u32(ring + (size_t)slot * slot_bytes) + lane_off;
            for (int rho = tw; rho < rows; rho += T) {
                const uint32_t rbase = sbase + (uint32_t)rho * (uint32_t)a.rb;
                float acc = 0.0f;
#pragma unroll
                for (int j = 0; j < GD_JMAX; ++j) {
                    if (j < js) {
                        const uint32_t ab = rbase + 34u * j;
                        const uint32_t a4 = ab & ~3u, o = ab & 3u;     // o is 0 or 2
                        uint32_t wv[9];
#pragma unroll
                        for (int i = 0; i < 9; ++i) wv[i] = d_lds32(a4 + 4u * i);
                        const uint32_t dbits = __funnelshift_r(wv[0], wv[1], 8u * o) & 0xffffu;
                        const uint32_t sh = 8u * (o + 2u);             // 16, or 32: the next word whole
                        int I0 = 0, I1 = 0, I2 = 0;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const uint32_t q = __funnelshift_rc(wv[i], wv[i + 1], sh);
                            I0 = dp4(q, xr[j][i], I0);
                            I1 = dp4(q, xr[j][8 + i], I1);
                            I2 = dp4(q, xr[j][16 + i], I2);
                        }
                        const float t = fmaf((float)I0, 65536.0f, (float)(I1 * 256 + I2));
                        acc = fmaf(__half2float(__ushort_as_half((uint16_t)dbits)) * xs[j], t, acc);
                    }
                }
#pragma unroll
                for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if (lane == 0) {
                    const int r = st * a.R + rho;
                    if (a.nseg == 1) a.y[r_begin + r] = acc;
                    else part[r * a.nseg + seg] = acc;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (a.nseg > 1) {
        gd_bar_consumers();
        if (ok) {
            for (int r = tid; r < nrows; r += GD_CW * 32) {
                float v = part[r * a.nseg];
                for (int s = 1; s < a.nseg; ++s) v += part[r * a.nseg + s];
                a.y[r_begin + r] = v;
            }
        }
    }
}

// ---------------------------------------------------------------------------
struct GdPlan {
    int nseg, jseg, R, nslots;
    uint32_t xs_off, part_off, bar_off;
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
    const int T = GD_CW / p.nseg;
    const int rows_cta = (N + grid - 1) / grid;
    const size_t fixed = (size_t)p.nseg * (GD_XSEG + GD_SSEG) + (p.nseg > 1 ? (size_t)rows_cta * p.nseg * 4 : 0) +
                         2 * GD_MAXSLOTS * 8 + 128 + 256;
    if (fixed >= GD_SMEM_MAX) return false;
    const size_t ring = GD_SMEM_MAX - fixed;
    // rows per slot: a multiple of the team size, slots of at most ~48 KB,
    // at least two slots
    int R = T;
    while ((size_t)(R + T) * rb <= 48 * 1024 && 2 * (size_t)(R + T) * rb <= ring && R + T <= rows_cta) R += T;
    if (2 * (size_t)R * rb > ring) return false;
    p.R = R;
    const int nst = (rows_cta + R - 1) / R;
    int slots = (int)(ring / ((size_t)R * rb));
    if (slots > GD_MAXSLOTS) slots = GD_MAXSLOTS;
    if (slots > nst) slots = nst < 2 ? 2 : nst;
    p.nslots = slots;
    const size_t ring_bytes = (size_t)slots * R * rb;
    p.xs_off = (uint32_t)(ring_bytes + (size_t)p.nseg * GD_XSEG);
    p.part_off = p.xs_off + (uint32_t)(p.nseg * GD_SSEG);
    p.bar_off = (p.part_off + (uint32_t)(p.nseg > 1 ? rows_cta * p.nseg * 4 : 0) + 15u) & ~15u;
    p.smem = (size_t)p.bar_off + 2 * (size_t)slots * 8 + 128;   // + alignment slack
    return p.smem <= GD_SMEM_MAX + 1024;
}

bool gemv_dp_ok(int t, size_t rb, int N, int K, int M, int num_sms) {
    if (t != QT_Q8_0 || M != 1 || N <= 0) return false;
    GdPlan p;
    return gd_plan(N, K, rb, num_sms < N ? num_sms : N, p);
}

tk_status launch_gemv_dp(tk_ctx* ctx, const void* W, size_t rb, int N, int K, const float* x, float* y, bool frozen,
                         cudaStream_t s) {
    const int grid = ctx->num_sms < N ? ctx->num_sms : N;
    GdPlan p;
    if (!gd_plan(N, K, rb, grid, p)) return fail(TK_ERR_UNSUPPORTED, "gemv dp4a: shape does not fit shared memory");
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemv_dp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)GD_SMEM_MAX + 1024);
        if (e != cudaSuccess) return cuda_fail(e, "gemv dp4a smem attribute");
        attr_set = true;
    }
    GdArgs a;
    a.W = static_cast<const uint8_t*>(W);
    a.rb = rb;
    a.N = N;
    a.K = K;
    a.x = x;
    a.y = y;
    a.nseg = p.nseg;
    a.jseg = p.jseg;
    a.R = p.R;
    a.nslots = p.nslots;
    a.xs_off = p.xs_off;
    a.part_off = p.part_off;
    a.bar_off = p.bar_off;
    a.frozen = frozen;
    a.status = ctx->status;
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
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_dp_kernel, a);
    ctx->launches++;
    if (e != cudaSuccess) return cuda_fail(e, "gemv dp4a launch");
    return cuda_fail(cudaGetLastError(), "gemv dp4a launch");
}

}  // namespace tk
