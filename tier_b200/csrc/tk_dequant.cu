// tk_dequant.cu -- HBM-bound elementwise kernels of the path:
//   * block dequant to fp32/fp16/bf16, bit-exact with q_val
//     (tier/quant.h:59-121) and dq_k (tier/tier.cpp:294-298);
//   * activation split/convert into fp16 planes for the tensor-core GEMM
//     (the reference's split3_fp_k, tier/tier.cpp:869-870, plus an exact
//     per-row power-of-two scale that keeps the low parts out of the fp16
//     subnormal range);
//   * fp32 weight -> fp16 hi/lo planes with a per-tensor power-of-two scale.
// Every thread produces 8 consecutive outputs so stores are 16-32 B vectors.
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

int block_elems(int t) {
    switch (t) {
        case QT_F32: case QT_F16: case QT_BF16: return 1;
        case QT_Q4_0: case QT_Q4_1: case QT_Q5_0: case QT_Q5_1: case QT_Q8_0: return 32;
        case QT_Q2_K: case QT_Q3_K: case QT_Q4_K: case QT_Q5_K: case QT_Q6_K: return 256;
        default: return 0;
    }
}
int block_bytes(int t) {
    switch (t) {
        case QT_F32: return 4;
        case QT_F16: case QT_BF16: return 2;
        case QT_Q4_0: return 18;
        case QT_Q4_1: return 20;
        case QT_Q5_0: return 22;
        case QT_Q5_1: return 24;
        case QT_Q8_0: return 34;
        case QT_Q2_K: return 84;
        case QT_Q3_K: return 110;
        case QT_Q4_K: return 144;
        case QT_Q5_K: return 176;
        case QT_Q6_K: return 210;
        default: return 0;
    }
}
bool dequant_supported(int t) { return block_elems(t) > 0; }

// Eight consecutive values [c, c+8) of a row.
template <int T>
__device__ __forceinline__ void decode8(const uint8_t* row, int c, float (&v)[8]) {
    if constexpr (T == QT_Q4_K) {
        q4k_decode8(row, c, v);
    } else if constexpr (T == QT_Q5_K) {
        q5k_decode8(row, c, v);
    } else if constexpr (T == QT_Q8_0) {
        const uint8_t* b = row + (size_t)(c >> 5) * 34;
        const float d = blk_scale(b);
        const uint8_t* q = b + 2 + (c & 31);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(d, (float)(int8_t)q[j]);
    } else if constexpr (T == QT_F16) {
        const uint4 w = *reinterpret_cast<const uint4*>(row + (size_t)c * 2);
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = h2f_bits((uint16_t)(u[j >> 1] >> (16 * (j & 1))));
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = qval(row, T, c + j);
    }
}

template <int T, int OUT>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ W, size_t rb, int r0, int nrows,
                                                      int cols, void* __restrict__ out) {
    const int gpr = cols >> 3;                       // 8-element groups per row
    const size_t total = (size_t)nrows * gpr;
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(g / gpr), c = (int)(g % gpr) * 8;
        float v[8];
        decode8<T>(W + (size_t)(r0 + r) * rb, c, v);
        const size_t o = (size_t)r * cols + c;
        if constexpr (OUT == TK_DT_F32) {
            float4* p = reinterpret_cast<float4*>(static_cast<float*>(out) + o);
            p[0] = make_float4(v[0], v[1], v[2], v[3]);
            p[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
            uint32_t u[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint16_t lo = OUT == TK_DT_F16 ? f2h_bits(v[2 * j]) : f2bf_bits(v[2 * j]);
                uint16_t hi = OUT == TK_DT_F16 ? f2h_bits(v[2 * j + 1]) : f2bf_bits(v[2 * j + 1]);
                u[j] = (uint32_t)lo | ((uint32_t)hi << 16);
            }
            *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + o) = make_uint4(u[0], u[1], u[2], u[3]);
        }
    }
}

template <int T>
static void dq_dispatch_out(int out_dtype, dim3 g, dim3 b, cudaStream_t s, const uint8_t* W, size_t rb, int r0,
                            int nrows, int cols, void* out) {
    if (out_dtype == TK_DT_F32) dequant_kernel<T, TK_DT_F32><<<g, b, 0, s>>>(W, rb, r0, nrows, cols, out);
    else if (out_dtype == TK_DT_F16) dequant_kernel<T, TK_DT_F16><<<g, b, 0, s>>>(W, rb, r0, nrows, cols, out);
    else dequant_kernel<T, TK_DT_BF16><<<g, b, 0, s>>>(W, rb, r0, nrows, cols, out);
}

tk_status launch_dequant(tk_ctx* ctx, int t, const void* W, size_t rb, int r0, int nrows, int cols, int out_dtype,
                         void* out, cudaStream_t s) {
    if (nrows == 0) return TK_OK;
    const size_t groups = (size_t)nrows * (cols / 8);
    const int threads = 256;
    size_t want = (groups + threads - 1) / threads;
    size_t cap = (size_t)ctx->num_sms * 16;
    dim3 grid((unsigned)(want < cap ? want : cap)), block(threads);
    const uint8_t* w = static_cast<const uint8_t*>(W);
    ProfScope ps(ctx, s, PK_DEQUANT);
    switch (t) {
        case QT_F32: dq_dispatch_out<QT_F32>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_F16: dq_dispatch_out<QT_F16>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_BF16: dq_dispatch_out<QT_BF16>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_Q4_0: dq_dispatch_out<QT_Q4_0>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_Q4_1: dq_dispatch_out<QT_Q4_1>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_Q5_0: dq_dispatch_out<QT_Q5_0>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_Q5_1: dq_dispatch_out<QT_Q5_1>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_Q8_0: dq_dispatch_out<QT_Q8_0>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_Q2_K: dq_dispatch_out<QT_Q2_K>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_Q3_K: dq_dispatch_out<QT_Q3_K>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_Q4_K: dq_dispatch_out<QT_Q4_K>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_Q5_K: dq_dispatch_out<QT_Q5_K>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_Q6_K: dq_dispatch_out<QT_Q6_K>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        default: return fail(TK_ERR_UNSUPPORTED, "tk_dequant: unsupported block type " + std::to_string(t));
    }
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "dequant launch");
}

// ---------------------------------------------------------------------------
// Activation split.  One 256-thread block per row: pass 1 finds max|x| of the
// row, pass 2 writes the scaled fp16 parts.  Scaling by 2^e is exact.
// ---------------------------------------------------------------------------
template <int XT>
__device__ __forceinline__ float ld_act(const void* X, size_t i) {
    if constexpr (XT == TK_DT_F32) return static_cast<const float*>(X)[i];
    else if constexpr (XT == TK_DT_F16) return h2f_bits(static_cast<const uint16_t*>(X)[i]);
    else return __uint_as_float((uint32_t)static_cast<const uint16_t*>(X)[i] << 16);
}

__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// Exponent e with amax * 2^e in [2^14, 2^15); 0 for zero / non-finite rows.
__device__ __forceinline__ int row_exponent(float amax) {
    if (!(amax > 0.0f) || !(amax < INFINITY)) return 0;
    int e = 14 - ilogbf(amax);
    return e < -100 ? -100 : (e > 100 ? 100 : e);
}

template <int XT, int NP>
__global__ void __launch_bounds__(256) act_split_kernel(const void* __restrict__ X, int M, int K, long ldx,
                                                        long ldp, bool scaled, uint16_t* __restrict__ planes,
                                                        int* __restrict__ row_exp) {
    __shared__ float red[8];
    const int m = blockIdx.x;
    const size_t xrow = (size_t)m * ldx;
    int e = 0;
    if (scaled) {
        float a = 0.0f;
        for (int k = threadIdx.x; k < K; k += blockDim.x) a = fmaxf(a, fabsf(ld_act<XT>(X, xrow + k)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
        __syncthreads();
        if (threadIdx.x < 32) {
            a = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
            if (threadIdx.x == 0) red[0] = a;
        }
        __syncthreads();
        e = row_exponent(red[0]);
    }
    if (threadIdx.x == 0 && row_exp) row_exp[m] = e;
    const float f = pow2f(e);
    const size_t pstride = (size_t)M * ldp, orow = (size_t)m * ldp;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float v = ld_act<XT>(X, xrow + k) * f;
        const uint16_t h = f2h_bits(v);
        planes[orow + k] = h;
        if constexpr (NP >= 2) {
            const float r = v - h2f_bits(h);
            const uint16_t mm = f2h_bits(r);
            if constexpr (NP == 2) {
                planes[pstride + orow + k] = mm;
            } else {
                planes[pstride + orow + k] = mm;
                planes[2 * pstride + orow + k] = f2h_bits(r - h2f_bits(mm));
            }
        }
    }
}

template <int XT>
static void act_split_np(int np, int M, int K, long ldx, long ldp, bool scaled, const void* X, uint16_t* planes,
                         int* re, cudaStream_t s) {
    if (np == 1) act_split_kernel<XT, 1><<<M, 256, 0, s>>>(X, M, K, ldx, ldp, scaled, planes, re);
    else if (np == 2) act_split_kernel<XT, 2><<<M, 256, 0, s>>>(X, M, K, ldx, ldp, scaled, planes, re);
    else act_split_kernel<XT, 3><<<M, 256, 0, s>>>(X, M, K, ldx, ldp, scaled, planes, re);
}

tk_status launch_act_split(tk_ctx* ctx, const void* X, int x_dtype, int M, int K, long ldx, int nplanes, bool scaled,
                           uint16_t* planes, int* row_exp, cudaStream_t s, long ldp) {
    if (M == 0) return TK_OK;
    if (ldp <= 0) ldp = K;
    ProfScope ps(ctx, s, PK_SPLIT);
    if (x_dtype == TK_DT_F32) act_split_np<TK_DT_F32>(nplanes, M, K, ldx, ldp, scaled, X, planes, row_exp, s);
    else if (x_dtype == TK_DT_F16) act_split_np<TK_DT_F16>(nplanes, M, K, ldx, ldp, scaled, X, planes, row_exp, s);
    else if (x_dtype == TK_DT_BF16) act_split_np<TK_DT_BF16>(nplanes, M, K, ldx, ldp, scaled, X, planes, row_exp, s);
    else return fail(TK_ERR_INVALID, "activation dtype " + std::to_string(x_dtype));
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "act_split launch");
}

// split3_fp_k exactly (no scaling): h = f16(x), m = f16(x-h), l = f16(x-h-m).
__global__ void split3_raw_kernel(const float* __restrict__ x, size_t n, uint16_t* __restrict__ h,
                                  uint16_t* __restrict__ m, uint16_t* __restrict__ l) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        const uint16_t a = f2h_bits(v);
        const float r = v - h2f_bits(a);
        const uint16_t b = f2h_bits(r);
        h[i] = a;
        m[i] = b;
        l[i] = f2h_bits(r - h2f_bits(b));
    }
}

tk_status launch_split3_raw(tk_ctx* ctx, const float* x, size_t n, uint16_t* h, uint16_t* m, uint16_t* l,
                            cudaStream_t s) {
    if (n == 0) return TK_OK;
    size_t want = (n + 255) / 256, cap = (size_t)ctx->num_sms * 16;
    ProfScope ps(ctx, s, PK_SPLIT);
    split3_raw_kernel<<<(unsigned)(want < cap ? want : cap), 256, 0, s>>>(x, n, h, m, l);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "split3 launch");
}

// ---------------------------------------------------------------------------
// fp32 weight -> TK_F16X2 planes.  Pass 1: max|W| (as ordered uint bits).
// ---------------------------------------------------------------------------
__global__ void absmax_kernel(const float* __restrict__ W, size_t n, unsigned int* out) {
    float a = 0.0f;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        a = fmaxf(a, fabsf(W[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(a));
}

__global__ void wsplit_kernel(const float* __restrict__ W, size_t n, const unsigned int* amax_bits,
                              uint16_t* __restrict__ hi, uint16_t* __restrict__ lo, int* scale_out) {
    const int e = row_exponent(__uint_as_float(*amax_bits));
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = e;
    const float f = pow2f(e);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = W[i] * f;
        const uint16_t h = f2h_bits(v);
        hi[i] = h;
        lo[i] = f2h_bits(v - h2f_bits(h));
    }
}

tk_status weight_split_f32(tk_ctx* ctx, const float* W, int rows, int cols, uint16_t* planes, int* scale_log2,
                           cudaStream_t s) {
    const size_t n = (size_t)rows * cols;
    tk_status st = ws_ensure(ctx, 256, s);
    if (st != TK_OK) return st;
    unsigned int* amax = static_cast<unsigned int*>(ctx->ws);
    int* sc = reinterpret_cast<int*>(amax + 1);
    cudaError_t e = cudaMemsetAsync(amax, 0, 8, s);
    if (e != cudaSuccess) return cuda_fail(e, "memset");
    const unsigned g = (unsigned)ctx->num_sms * 8;
    absmax_kernel<<<g, 256, 0, s>>>(W, n, amax);
    wsplit_kernel<<<g, 256, 0, s>>>(W, n, amax, planes, planes + n, sc);
    ctx->launches += 2;
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "weight split launch");
    int host_sc = 0;
    e = cudaMemcpyAsync(&host_sc, sc, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "weight split scale readback");
    *scale_log2 = host_sc;
    return TK_OK;
}

}  // namespace tk
