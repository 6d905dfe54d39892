// tk_gemv.cu -- decode GEMV, y[m, n] = sum_k W(n, k) x[m, k] for M = 1..16
// tokens.  Replaces gemv_q (tier/tier.cpp:300-306) and gemv<T>
// (tier/tier.cpp:2261-2268).
//
// HBM-bound: each weight byte is read once.  One warp owns one output row at
// a time.  For block-quantized rows the warp copies a 4096-element slice of
// the row (whole 16-byte aligned blocks) from HBM into its own shared buffer
// with 16-byte loads (all loads of the slice issued before any use), then
// decodes 8-element groups from shared memory with the bit-exact dequant and
// accumulates fp32 dot products for all M tokens.  Lane partial sums are
// reduced with a shuffle tree, as the reference does.  fp16/bf16/fp32 rows
// are read directly with 16-byte vector loads.  Every other block type (the
// legacy and remaining K-quants, the table-level types of tk_qtypes.h, the
// lattice types of tk_qgrid.h) decodes per element straight from global
// memory, as gemv_q does for every type.  The dedicated kernels for Q8_0 /
// Q4_K / Q5_K / Q6_K live in tk_gemv4-7.cu; launch_gemv picks among them.
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

constexpr int GEMV_WARPS = 8;
constexpr int SLICE = 4096;        // elements per staged slice

__host__ __device__ constexpr int slice_bytes(int t) {
    return t == QT_Q8_0 ? SLICE / 32 * 34
         : t == QT_Q4_0 ? SLICE / 32 * 18
         : t == QT_Q4_K ? SLICE / 256 * 144
         : t == QT_Q5_K ? SLICE / 256 * 176
         : 0;
}

template <int T>
__device__ __forceinline__ void dec8(const uint8_t* row, int c, float (&v)[8]) {
    if constexpr (T == QT_Q4_K) {
        q4k_decode8(row, c, v);
    } else if constexpr (T == QT_Q5_K) {
        q5k_decode8(row, c, v);
    } else if constexpr (T == QT_Q8_0) {
        const uint8_t* b = row + (c >> 5) * 34;
        const float d = blk_scale(b);
        const uint16_t* q = reinterpret_cast<const uint16_t*>(b + 2 + (c & 31));   // 2-byte aligned
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint16_t w = q[j];
            v[2 * j] = __fmul_rn(d, (float)(int8_t)(w & 0xff));
            v[2 * j + 1] = __fmul_rn(d, (float)(int8_t)(w >> 8));
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = qval(row, T, c + j);
    }
}

template <int M>
__device__ __forceinline__ void fma8(float (&acc)[M], const float (&v)[8], const float* __restrict__ x, int ldx,
                                     int c) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(x + (size_t)m * ldx + c));
        const float4 b = __ldg(reinterpret_cast<const float4*>(x + (size_t)m * ldx + c + 4));
        float s = acc[m];
        s = fmaf(v[0], a.x, s); s = fmaf(v[1], a.y, s); s = fmaf(v[2], a.z, s); s = fmaf(v[3], a.w, s);
        s = fmaf(v[4], b.x, s); s = fmaf(v[5], b.y, s); s = fmaf(v[6], b.z, s); s = fmaf(v[7], b.w, s);
        acc[m] = s;
    }
}

template <int M>
__device__ __forceinline__ void warp_store(float (&acc)[M], float* y, int ldy, int n, int lane) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
        float a = acc[m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_down_sync(0xffffffffu, a, o);
        if (lane == 0) y[(size_t)m * ldy + n] = a;
    }
}

// Block-quantized rows, staged through shared memory.
template <int T, int M>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_block_kernel(const uint8_t* __restrict__ W, size_t rb, int N,
                                                                     int K, const float* __restrict__ x, int ldx,
                                                                     float* __restrict__ y, int ldy) {
    constexpr int SB = slice_bytes(T);
    __shared__ __align__(16) uint8_t buf[GEMV_WARPS][SB];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* my = buf[warp];
    const int nwarps = gridDim.x * GEMV_WARPS;
    for (int n = blockIdx.x * GEMV_WARPS + warp; n < N; n += nwarps) {
        const uint8_t* row = W + (size_t)n * rb;
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = 0.0f;
        for (int k0 = 0; k0 < K; k0 += SLICE) {
            const int len = K - k0 < SLICE ? K - k0 : SLICE;
            const int bytes = (int)((size_t)len * SB / SLICE);   // len is a multiple of 256: bytes % 16 == 0
            const uint8_t* src = row + (size_t)k0 / SLICE * SB;
            // stage: all 16-byte loads of the slice in flight together
            constexpr int PER_LANE = (SB + 16 * 32 - 1) / (16 * 32);
            uint4 t[PER_LANE];
#pragma unroll
            for (int i = 0; i < PER_LANE; ++i) {
                const int off = (i * 32 + lane) * 16;
                if (off < bytes) t[i] = __ldg(reinterpret_cast<const uint4*>(src + off));
            }
#pragma unroll
            for (int i = 0; i < PER_LANE; ++i) {
                const int off = (i * 32 + lane) * 16;
                if (off < bytes) *reinterpret_cast<uint4*>(my + off) = t[i];
            }
            __syncwarp();
            for (int c = lane * 8; c < len; c += 256) {
                float v[8];
                dec8<T>(my, c, v);
                fma8<M>(acc, v, x, ldx, k0 + c);
            }
            __syncwarp();
        }
        warp_store<M>(acc, y, ldy, n, lane);
    }
}

// fp16 / bf16 / fp32 rows read directly (16-byte loads of 8 or 4 elements).
template <int T, int M>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_dense_kernel(const uint8_t* __restrict__ W, size_t rb, int N,
                                                                     int K, const float* __restrict__ x, int ldx,
                                                                     float* __restrict__ y, int ldy) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = gridDim.x * GEMV_WARPS;
    for (int n = blockIdx.x * GEMV_WARPS + warp; n < N; n += nwarps) {
        const uint8_t* row = W + (size_t)n * rb;
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = 0.0f;
#pragma unroll 4
        for (int c = lane * 8; c < K; c += 256) {
            float v[8];
            if constexpr (T == QT_F32) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(row + (size_t)c * 4));
                const float4 b = __ldg(reinterpret_cast<const float4*>(row + (size_t)c * 4 + 16));
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
                const uint4 w = __ldg(reinterpret_cast<const uint4*>(row + (size_t)c * 2));
                const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint16_t h = (uint16_t)(u[j >> 1] >> (16 * (j & 1)));
                    v[j] = T == QT_F16 ? h2f_bits(h) : __uint_as_float((uint32_t)h << 16);
                }
            }
            fma8<M>(acc, v, x, ldx, c);
        }
        warp_store<M>(acc, y, ldy, n, lane);
    }
}

// Any other block type: per-element q_val straight from global memory.
template <int T, int M>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_direct_kernel(const uint8_t* __restrict__ W, size_t rb, int N,
                                                                      int K, const float* __restrict__ x, int ldx,
                                                                      float* __restrict__ y, int ldy) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = gridDim.x * GEMV_WARPS;
    for (int n = blockIdx.x * GEMV_WARPS + warp; n < N; n += nwarps) {
        const uint8_t* row = W + (size_t)n * rb;
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = 0.0f;
        for (int c = lane * 8; c < K; c += 256) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = qval(row, T, c + j);
            fma8<M>(acc, v, x, ldx, c);
        }
        warp_store<M>(acc, y, ldy, n, lane);
    }
}

// Lattice types (tk_qgrid.h): as gemv_direct_kernel, the registered table
// buffer passed in.
template <int T, int M>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_grid_kernel(const uint8_t* __restrict__ W, size_t rb, int N,
                                                                    int K, const float* __restrict__ x, int ldx,
                                                                    float* __restrict__ y, int ldy,
                                                                    const int8_t* __restrict__ tab) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = gridDim.x * GEMV_WARPS;
    for (int n = blockIdx.x * GEMV_WARPS + warp; n < N; n += nwarps) {
        const uint8_t* row = W + (size_t)n * rb;
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = 0.0f;
        for (int c = lane * 8; c < K; c += 256) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = tkq::grid_value(row, T, c + j, tab);
            fma8<M>(acc, v, x, ldx, c);
        }
        warp_store<M>(acc, y, ldy, n, lane);
    }
}

template <int T>
static void gemv_grid_m(int M, int blocks, cudaStream_t s, const uint8_t* W, size_t rb, int N, int K, const float* x,
                        int ldx, float* y, int ldy, const int8_t* tab) {
    int m0 = 0;
    while (m0 < M) {
        const int r = M - m0;
        const float* xs = x + (size_t)m0 * ldx;
        float* ys = y + (size_t)m0 * ldy;
        const dim3 g(blocks), b(GEMV_WARPS * 32);
        if (r >= 16) { gemv_grid_kernel<T, 16><<<g, b, 0, s>>>(W, rb, N, K, xs, ldx, ys, ldy, tab); m0 += 16; }
        else if (r >= 8) { gemv_grid_kernel<T, 8><<<g, b, 0, s>>>(W, rb, N, K, xs, ldx, ys, ldy, tab); m0 += 8; }
        else if (r >= 4) { gemv_grid_kernel<T, 4><<<g, b, 0, s>>>(W, rb, N, K, xs, ldx, ys, ldy, tab); m0 += 4; }
        else if (r >= 2) { gemv_grid_kernel<T, 2><<<g, b, 0, s>>>(W, rb, N, K, xs, ldx, ys, ldy, tab); m0 += 2; }
        else { gemv_grid_kernel<T, 1><<<g, b, 0, s>>>(W, rb, N, K, xs, ldx, ys, ldy, tab); m0 += 1; }
    }
}

// Every block type of the dequant: the reference's gemv_q decodes any type
// through q_val; the types without a dedicated kernel take gemv_direct_kernel.
bool gemv_supported(int t) { return dequant_supported(t); }

template <int T, int M>
static void gemv_go(int blocks, cudaStream_t s, const uint8_t* W, size_t rb, int N, int K, const float* x, int ldx,
                    float* y, int ldy) {
    if constexpr (T == QT_F16 || T == QT_BF16 || T == QT_F32)
        gemv_dense_kernel<T, M><<<blocks, GEMV_WARPS * 32, 0, s>>>(W, rb, N, K, x, ldx, y, ldy);
    else if constexpr (slice_bytes(T) > 0)
        gemv_block_kernel<T, M><<<blocks, GEMV_WARPS * 32, 0, s>>>(W, rb, N, K, x, ldx, y, ldy);
    else
        gemv_direct_kernel<T, M><<<blocks, GEMV_WARPS * 32, 0, s>>>(W, rb, N, K, x, ldx, y, ldy);
}

template <int T>
static void gemv_m(int M, int blocks, cudaStream_t s, const uint8_t* W, size_t rb, int N, int K, const float* x,
                   int ldx, float* y, int ldy) {
    // Token counts are handled in chunks of 16/8/4/2/1 so every M in 1..16 works.
    int m0 = 0;
    while (m0 < M) {
        const int r = M - m0;
        const float* xs = x + (size_t)m0 * ldx;
        float* ys = y + (size_t)m0 * ldy;
        if (r >= 16) { gemv_go<T, 16>(blocks, s, W, rb, N, K, xs, ldx, ys, ldy); m0 += 16; }
        else if (r >= 8) { gemv_go<T, 8>(blocks, s, W, rb, N, K, xs, ldx, ys, ldy); m0 += 8; }
        else if (r >= 4) { gemv_go<T, 4>(blocks, s, W, rb, N, K, xs, ldx, ys, ldy); m0 += 4; }
        else if (r >= 2) { gemv_go<T, 2>(blocks, s, W, rb, N, K, xs, ldx, ys, ldy); m0 += 2; }
        else { gemv_go<T, 1>(blocks, s, W, rb, N, K, xs, ldx, ys, ldy); m0 += 1; }
    }
}

static int popcount_chunks(int M) {
    int n = 0, m0 = 0;
    while (m0 < M) {
        int r = M - m0;
        m0 += r >= 16 ? 16 : r >= 8 ? 8 : r >= 4 ? 4 : r >= 2 ? 2 : 1;
        ++n;
    }
    return n;
}

tk_status launch_gemv(tk_ctx* ctx, int t, const void* Wv, size_t rb, int N, int K, const float* x, int ldx, int M,
                      float* y, int ldy, cudaStream_t s, bool frozen) {
    if (N == 0 || M == 0) return TK_OK;
    // One Q8_0 token: dp4a with x in registers (tk_gemv8.cu).
    if (M == 1 && (reinterpret_cast<uintptr_t>(Wv) & 15) == 0 && gemv_dp_ok(t, rb, N, K, M, ctx->num_sms))
        return launch_gemv_dp(ctx, Wv, rb, N, K, x, y, frozen, s);
    // Integer tensor-core kernel (tk_gemv6.cu) for one or two tokens.
    if (M <= 2 && gemv_imma_ok(t, rb, K, M) && (reinterpret_cast<uintptr_t>(Wv) & 15) == 0)
        return launch_gemv_imma(ctx, t, Wv, rb, N, K, x, ldx, M, y, ldy, frozen, s);
    // 3..16 tokens reading W once, x records streamed with the weight
    // (tk_gemv7.cu); 3 or 4 tokens whose x fits shared memory stay on the fp16
    // kernel below (one launch, measured faster there).
    const bool aligned = (reinterpret_cast<uintptr_t>(Wv) & 15) == 0;
    if (M >= 3 && aligned && !(M <= 4 && gemv_mma_ok(t, rb, K, M))) {
        if (gemv_wide_ok(t, rb, K, M)) return launch_gemv_wide(ctx, t, Wv, rb, N, K, x, ldx, M, y, ldy, s);
        if (M > 8 && gemv_wide_ok(t, rb, K, 8)) {
            // 16-token records do not fit next to the weight ring (Q6_K): token
            // halves, W read twice; a remainder of 1-2 tokens takes the M <= 2 path
            for (int m0 = 0; m0 < M; m0 += 8) {
                const int c = M - m0 < 8 ? M - m0 : 8;
                tk_status st = c >= 3 ? launch_gemv_wide(ctx, t, Wv, rb, N, K, x + (size_t)m0 * ldx, ldx, c,
                                                         y + (size_t)m0 * ldy, ldy, s)
                                      : launch_gemv(ctx, t, Wv, rb, N, K, x + (size_t)m0 * ldx, ldx, c,
                                                    y + (size_t)m0 * ldy, ldy, s, frozen);
                if (st != TK_OK) return st;
            }
            return TK_OK;
        }
    }
    // fp16 tensor-core kernel (tk_gemv5.cu) for Q8_0 / Q4_K / Q5_K / Q6_K when
    // x fits in shared memory: token chunks of up to 8.
    if (gemv_mma_ok(t, rb, K, 1) && (reinterpret_cast<uintptr_t>(Wv) & 15) == 0) {
        int m0 = 0;
        while (m0 < M) {
            int c = M - m0 < 8 ? M - m0 : 8;
            while (c > 1 && !gemv_mma_ok(t, rb, K, c)) --c;
            tk_status st = launch_gemv_mma(ctx, t, Wv, rb, N, K, x + (size_t)m0 * ldx, ldx, c, y + (size_t)m0 * ldy,
                                           ldy, frozen, s);
            if (st != TK_OK) return st;
            m0 += c;
        }
        return TK_OK;
    }
    // Streaming kernel (tk_gemv4.cu) for Q8_0 / Q4_K / Q5_K when x fits in
    // shared memory: token chunks of 4, 2 and 1.
    if (gemv_stream_ok(t, rb, K, 1) && (reinterpret_cast<uintptr_t>(Wv) & 15) == 0) {
        int m0 = 0;
        while (m0 < M) {
            const int r = M - m0;
            const int c = (r >= 4 && gemv_stream_ok(t, rb, K, 4)) ? 4 : (r >= 2 && gemv_stream_ok(t, rb, K, 2)) ? 2 : 1;
            tk_status st = launch_gemv_stream(ctx, t, Wv, rb, N, K, x + (size_t)m0 * ldx, ldx, c, y + (size_t)m0 * ldy,
                                              ldy, frozen, s);
            if (st != TK_OK) return st;
            m0 += c;
        }
        return TK_OK;
    }
    const uint8_t* W = static_cast<const uint8_t*>(Wv);
    const int rows_per_block = GEMV_WARPS;
    int blocks = (N + rows_per_block - 1) / rows_per_block;
    if (tkq::is_grid(t)) {
        if (!ctx->iq_tab)
            return fail(TK_ERR_UNSUPPORTED, "tk_gemv: type " + std::to_string(t) +
                                                " needs the IQ grid tables (tk_set_iq_grids)");
        const int8_t* tab = ctx->iq_tab;
        ProfScope ps(ctx, s, PK_GEMV);
        switch (t) {
            case tkq::IQ2_XXS: gemv_grid_m<tkq::IQ2_XXS>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy, tab); break;
            case tkq::IQ2_XS: gemv_grid_m<tkq::IQ2_XS>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy, tab); break;
            case tkq::IQ2_S: gemv_grid_m<tkq::IQ2_S>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy, tab); break;
            case tkq::IQ3_XXS: gemv_grid_m<tkq::IQ3_XXS>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy, tab); break;
            case tkq::IQ3_S: gemv_grid_m<tkq::IQ3_S>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy, tab); break;
            case tkq::IQ1_S: gemv_grid_m<tkq::IQ1_S>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy, tab); break;
            default: gemv_grid_m<tkq::IQ1_M>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy, tab); break;
        }
        ctx->launches += popcount_chunks(M);
        return cuda_fail(cudaGetLastError(), "gemv launch");
    }
    ProfScope ps(ctx, s, PK_GEMV);
    switch (t) {
        case QT_Q8_0: gemv_m<QT_Q8_0>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_Q4_0: gemv_m<QT_Q4_0>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_Q4_K: gemv_m<QT_Q4_K>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_Q5_K: gemv_m<QT_Q5_K>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_Q6_K: gemv_m<QT_Q6_K>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_F16: gemv_m<QT_F16>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_BF16: gemv_m<QT_BF16>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_F32: gemv_m<QT_F32>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_Q4_1: gemv_m<QT_Q4_1>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_Q5_0: gemv_m<QT_Q5_0>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_Q5_1: gemv_m<QT_Q5_1>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_Q2_K: gemv_m<QT_Q2_K>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_Q3_K: gemv_m<QT_Q3_K>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_IQ4_NL: gemv_m<QT_IQ4_NL>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_IQ4_XS: gemv_m<QT_IQ4_XS>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_MXFP4: gemv_m<QT_MXFP4>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_NF4: gemv_m<QT_NF4>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_FP4: gemv_m<QT_FP4>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_TQ1_0: gemv_m<QT_TQ1_0>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        case QT_TQ2_0: gemv_m<QT_TQ2_0>(M, blocks, s, W, rb, N, K, x, ldx, y, ldy); break;
        default: return fail(TK_ERR_UNSUPPORTED, "tk_gemv: unsupported weight type " + std::to_string(t));
    }
    ctx->launches += popcount_chunks(M);
    return cuda_fail(cudaGetLastError(), "gemv launch");
}

}  // namespace tk
