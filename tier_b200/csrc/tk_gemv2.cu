// tk_gemv2.cu -- streaming decode GEMV for Q8_0 / Q4_K / Q5_K rows, M <= 4.
//
// y[m, n] = sum_k W(n, k) x[m, k].  HBM-bound: every weight byte is read once.
//
//  * One block of 16 warps per SM owns a contiguous range of rows and streams
//    them through a 4-stage shared-memory ring with cp.async.bulk (a stage is
//    up to 4 consecutive rows, one copy, completion on an mbarrier), so tens
//    of KB per SM are in flight while the previous stage is reduced.
//  * x (fp32, M x K) lives in shared memory, loaded once per block; lanes are
//    contiguous over elements so every x read is a conflict-free 16-byte load.
//  * Integer quants become floats exactly with the 2^23 magic-number trick
//    (integer OR into the mantissa of 2^23, then one subtraction), keeping the
//    slow int->float conversion pipe out of the loop.
//  * Per four elements of one sub-block the dot product is factored as
//      sum_j (a q_j - m) x_j = a * sum_j q_j x_j - m * sum_j x_j
//    (Q8_0: m = 0), so each weight costs one conversion and M fused
//    multiply-adds.  The reference (tier/tier.cpp:300-306) forms every
//    weight with q_val and accumulates weight*x; the results agree to fp32
//    rounding (the decode tolerance is 2e-3 relative).
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {


__device__ __forceinline__ float magic_u8(uint32_t b) {        // exact float of 0..255
    return __uint_as_float(0x4B000000u | b) - 8388608.0f;
}

// One row's partial dot products for this lane.  Lanes are contiguous over
// elements: in every 128-element chunk lane l takes elements 4l .. 4l+3, so
// the x reads are conflict-free 16-byte shared-memory loads and the four
// quants of a lane sit in one sub-block (one scale, one min).
template <int T, int M>
__device__ __forceinline__ void row_dot(const uint8_t* __restrict__ row, const float* __restrict__ xs, int K,
                                        int lane, float (&acc)[M], int p, int wpr, int nchunk) {
#pragma unroll 2
    for (int c = p; c < nchunk; c += wpr) {
        const int e = c * 128 + 4 * lane;            // first of this lane's four elements
        float q[4], a = 1.0f, mm = 0.0f;
        if constexpr (T == QT_Q8_0) {
            const uint8_t* blk = row + (e >> 5) * 34;
            a = h2f_bits(*reinterpret_cast<const uint16_t*>(blk));
            const uint16_t* qp = reinterpret_cast<const uint16_t*>(blk + 2 + (e & 31));   // 2-byte aligned
            const uint32_t w0 = qp[0] ^ 0x8080u, w1 = qp[1] ^ 0x8080u;
            q[0] = __uint_as_float(0x4B000000u | (w0 & 0xffu)) - 8388736.0f;   // (2^23 + q + 128) - (2^23 + 128)
            q[1] = __uint_as_float(0x4B000000u | (w0 >> 8)) - 8388736.0f;
            q[2] = __uint_as_float(0x4B000000u | (w1 & 0xffu)) - 8388736.0f;
            q[3] = __uint_as_float(0x4B000000u | (w1 >> 8)) - 8388736.0f;
        } else {
            constexpr int SB = T == QT_Q4_K ? 144 : 176;
            constexpr int QS = T == QT_Q4_K ? 16 : 48;
            const int i = e & 255, g = i >> 6, hi = (i & 63) >= 32;
            const uint8_t* blk = row + (e >> 8) * SB;
            const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
            int sc, mn;
            kq_scale_min_reg(2 * g + hi, hdr, sc, mn);
            a = __fmul_rn(h2f_bits((uint16_t)(hdr.x & 0xffff)), (float)sc);
            mm = __fmul_rn(h2f_bits((uint16_t)(hdr.x >> 16)), (float)mn);
            const uint32_t w = *reinterpret_cast<const uint32_t*>(blk + QS + g * 32 + (i & 31));
            uint32_t hb = 0;
            if constexpr (T == QT_Q5_K) hb = *reinterpret_cast<const uint32_t*>(blk + 16 + (i & 31));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t v = (w >> (8 * j + 4 * hi)) & 15u;
                if constexpr (T == QT_Q5_K) v |= ((hb >> (8 * j + (i >> 5))) & 1u) << 4;
                q[j] = magic_u8(v);
            }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float4 xv = *reinterpret_cast<const float4*>(xs + (size_t)m * K + e);
            float s = q[0] * xv.x;
            s = fmaf(q[1], xv.y, s);
            s = fmaf(q[2], xv.z, s);
            s = fmaf(q[3], xv.w, s);
            acc[m] = fmaf(a, s, acc[m]);
            if constexpr (T != QT_Q8_0) acc[m] = fmaf(-mm, (xv.x + xv.y) + (xv.z + xv.w), acc[m]);
        }
    }
}

// Block = 16 warps on one SM, owning a contiguous range of rows.  A stage is
// RPS consecutive rows (one bulk copy); the 16 warps split the stage's rows
// (16/RPS warps per row, each taking every (16/RPS)-th 128-element chunk);
// per-warp partials are summed in a fixed order, so results are deterministic.
constexpr int G3_WARPS = 16, G3_STAGES = 4;

template <int T, int M>
__global__ void __launch_bounds__(G3_WARPS * 32, 1)
    gemv_stream_kernel(const uint8_t* __restrict__ W, size_t rb, int N, int K, const float* __restrict__ x, int ldx,
                       float* __restrict__ y, int ldy, int rps, int* status) {
    extern __shared__ uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t stage_bytes = ((size_t)rps * rb + 127) & ~size_t(127);
    uint8_t* ring = sm;
    float* xs = reinterpret_cast<float*>(sm + G3_STAGES * stage_bytes);
    float* part = xs + (size_t)M * K;                                   // [G3_WARPS][M]
    uint64_t* bars = reinterpret_cast<uint64_t*>(part + G3_WARPS * M);

    const int r_begin = (int)((long long)N * blockIdx.x / gridDim.x);
    const int r_end = (int)((long long)N * (blockIdx.x + 1) / gridDim.x);
    const int nst = (r_end - r_begin + rps - 1) / rps;
    auto issue = [&](int st) {
        const int r0 = r_begin + st * rps;
        const int nr = r_end - r0 < rps ? r_end - r0 : rps;
        uint64_t* b = &bars[st % G3_STAGES];
        mbar_arrive_expect_tx(b, (uint32_t)(nr * rb));
        bulk_load(ring + (size_t)(st % G3_STAGES) * stage_bytes, W + (size_t)r0 * rb, (uint32_t)(nr * rb), b);
    };
    if (threadIdx.x == 0) {
        for (int i = 0; i < G3_STAGES; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
        for (int i = 0; i < G3_STAGES && i < nst; ++i) issue(i);
    }
    for (int m = 0; m < M; ++m)
        for (int k = threadIdx.x * 4; k < K; k += blockDim.x * 4)
            *reinterpret_cast<float4*>(xs + (size_t)m * K + k) =
                __ldg(reinterpret_cast<const float4*>(x + (size_t)m * ldx + k));
    __syncthreads();

    const int wpr = G3_WARPS / rps;               // warps per row
    const int rloc = warp / wpr, p = warp % wpr;
    const int nchunk = K >> 7;
    bool ok = true;
    for (int st = 0; st < nst; ++st) {
        const int slot = st % G3_STAGES;
        if (ok && !mbar_wait(&bars[slot], (uint32_t)(st / G3_STAGES) & 1u, status)) ok = false;
        const int r0 = r_begin + st * rps;
        const int nr = r_end - r0 < rps ? r_end - r0 : rps;
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = 0.0f;
        if (ok && rloc < nr) {
            const uint8_t* row = ring + (size_t)slot * stage_bytes + (size_t)rloc * rb;
            row_dot<T, M>(row, xs, K, lane, acc, p, wpr, nchunk);
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float a = acc[m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            if (lane == 0) part[warp * M + m] = a;
        }
        __syncthreads();
        if (threadIdx.x < nr * M) {
            const int rr = threadIdx.x / M, m = threadIdx.x % M;
            float sum = 0.0f;
            for (int q = 0; q < wpr; ++q) sum += part[(rr * wpr + q) * M + m];
            y[(size_t)m * ldy + r0 + rr] = sum;
        }
        if (threadIdx.x == 0 && ok && st + G3_STAGES < nst) {
            fence_async_shared();     // this stage's generic reads precede the async overwrite
            issue(st + G3_STAGES);
        }
        __syncthreads();              // partials consumed before the next stage writes them
    }
}

// Rows per stage: as many as fit 48 KB (<= 4, a power of two dividing 16).
static int pick_rps(size_t rb) {
    int r = 4;
    while (r > 1 && (size_t)r * rb > 48 * 1024) r >>= 1;
    return r;
}

static size_t stream_smem(size_t rb, int K, int M) {
    const size_t stage = ((size_t)pick_rps(rb) * rb + 127) & ~size_t(127);
    return 128 + G3_STAGES * stage + (size_t)M * K * 4 + (size_t)G3_WARPS * M * 4 + G3_STAGES * 8 + 64;
}

constexpr size_t kStreamSmemMax = 200 * 1024;

bool gemv_stream_ok(int t, size_t rb, int K, int M) {
    if (t != QT_Q8_0 && t != QT_Q4_K && t != QT_Q5_K) return false;
    if (M > 4 || M == 3 || rb % 16 || K % 128) return false;
    return stream_smem(rb, K, M) <= kStreamSmemMax;
}

template <int T, int M>
static tk_status go_stream(tk_ctx* ctx, const uint8_t* W, size_t rb, int N, int K, const float* x, int ldx, float* y,
                           int ldy, cudaStream_t s) {
    const int rps = pick_rps(rb);
    const size_t smem = stream_smem(rb, K, M);
    auto kern = gemv_stream_kernel<T, M>;
    static bool attr_set = false;   // per instantiation: one limit for every launch
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStreamSmemMax + 256);
        if (e != cudaSuccess) return cuda_fail(e, "gemv smem attribute");
        attr_set = true;
    }
    int grid = (N + rps - 1) / rps;
    if (grid > ctx->num_sms) grid = ctx->num_sms;
    ProfScope ps(ctx, s, PK_GEMV);
    kern<<<grid, G3_WARPS * 32, smem, s>>>(W, rb, N, K, x, ldx, y, ldy, rps, ctx->status);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "gemv stream launch");
}

tk_status launch_gemv_stream(tk_ctx* ctx, int t, const void* Wv, size_t rb, int N, int K, const float* x, int ldx,
                             int M, float* y, int ldy, cudaStream_t s) {
    const uint8_t* W = static_cast<const uint8_t*>(Wv);
#define TK_G2(TT)                                                                       \
    if (t == TT) {                                                                      \
        if (M == 1) return go_stream<TT, 1>(ctx, W, rb, N, K, x, ldx, y, ldy, s);       \
        if (M == 2) return go_stream<TT, 2>(ctx, W, rb, N, K, x, ldx, y, ldy, s);       \
        return go_stream<TT, 4>(ctx, W, rb, N, K, x, ldx, y, ldy, s);                   \
    }
    TK_G2(QT_Q8_0)
    TK_G2(QT_Q4_K)
    TK_G2(QT_Q5_K)
#undef TK_G2
    return fail(TK_ERR_UNSUPPORTED, "gemv stream: type");
}

}  // namespace tk
