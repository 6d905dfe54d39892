// tk_dequant.cu -- HBM-bound elementwise kernels of the path:
//   * block dequant to fp32/fp16/bf16, bit-exact with q_val
//     (tier/quant.h:59-121) and dq_k (tier/tier.cpp:294-298), for all 27
//     block types (the lattice types read the tables of tk_set_iq_grids);
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
        default: return tkq::is_grid(t) ? 256 : tkq::elems(t);
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
        default: return tkq::is_grid(t) ? tkq::grid_bytes(t) : tkq::bytes(t);
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
        const uint16_t* q = reinterpret_cast<const uint16_t*>(b + 2 + (c & 31));   // 2-byte aligned
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t w = q[j] ^ 0x8080u;                 // int8 pair -> biased uint8 pair
            v[2 * j] = __fmul_rn(d, small_u2f(w & 0xffu) - 128.0f);
            v[2 * j + 1] = __fmul_rn(d, small_u2f(w >> 8) - 128.0f);
        }
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

constexpr int DQ_UNROLL = 4;   // independent 8-element groups in flight per thread

template <int OUT>
__device__ __forceinline__ void store8(void* __restrict__ out, size_t o, const float (&v)[8]) {
    if constexpr (OUT == TK_DT_F32) {
        float4* p = reinterpret_cast<float4*>(static_cast<float*>(out) + o);
        p[0] = make_float4(v[0], v[1], v[2], v[3]);
        p[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else if constexpr (OUT == TK_DT_F16) {
        // packed round-to-nearest-even; NaN needs the reference's bit pattern
        // (sign | 0x7e00), so fall back per element only if one is present.
        const bool nan = (v[0] != v[0]) | (v[1] != v[1]) | (v[2] != v[2]) | (v[3] != v[3]) | (v[4] != v[4]) |
                         (v[5] != v[5]) | (v[6] != v[6]) | (v[7] != v[7]);
        uint32_t u[4];
        if (!nan) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
                u[j] = *reinterpret_cast<const uint32_t*>(&h);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) u[j] = (uint32_t)f2h_bits(v[2 * j]) | ((uint32_t)f2h_bits(v[2 * j + 1]) << 16);
        }
        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + o) = make_uint4(u[0], u[1], u[2], u[3]);
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

// Grid: x = chunks of DQ_THREADS*DQ_UNROLL groups within a row, y = rows
// (strided).  No integer division on the device.
constexpr int DQ_THREADS = 128;

template <int T, int OUT>
__global__ void __launch_bounds__(DQ_THREADS) dequant_kernel(const uint8_t* __restrict__ W, size_t rb, int r0,
                                                             int nrows, int cols, void* __restrict__ out) {
    const int gpr = cols >> 3;                       // 8-element groups per row
    for (int r = blockIdx.y; r < nrows; r += gridDim.y) {
        const uint8_t* row = W + (size_t)(r0 + r) * rb;
        const size_t orow = (size_t)r * cols;
        for (int base = blockIdx.x * DQ_THREADS * DQ_UNROLL + threadIdx.x; base < gpr;
             base += gridDim.x * DQ_THREADS * DQ_UNROLL) {
            float v[DQ_UNROLL][8];
#pragma unroll
            for (int u = 0; u < DQ_UNROLL; ++u) {
                const int g = base + u * DQ_THREADS;
                if (g < gpr) decode8<T>(row, g * 8, v[u]);
            }
#pragma unroll
            for (int u = 0; u < DQ_UNROLL; ++u) {
                const int g = base + u * DQ_THREADS;
                if (g < gpr) store8<OUT>(out, orow + (size_t)g * 8, v[u]);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Sub-block kernel for Q4_K / Q5_K / Q8_0 -> fp16 (the tensor-core path's
// format): one thread per 32-element sub-block (decoder sub32_to_f16 in
// tk_device.cuh), 64 B of output per thread.  A warp's 32 consecutive
// sub-blocks are 2 KB of consecutive output: they are staged in shared memory
// and written as four fully coalesced 512-byte stores instead of each lane
// writing its own 64 bytes (16 bytes per lane per instruction, 64 bytes
// apart).  Threads run flat over (row, sub-block): one 32-bit division per 32
// weights.
template <int T>
__global__ void __launch_bounds__(256) dequant_sub_f16_kernel(const uint8_t* __restrict__ W, size_t rb, int r0,
                                                              int nrows, int cols, uint16_t* __restrict__ out) {
    pdl_trigger();
    __shared__ uint4 stage[8][32 * 4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned spr = (unsigned)cols >> 5;       // sub-blocks per row
    const unsigned total = (unsigned)nrows * spr;
    const unsigned stride = gridDim.x * blockDim.x;
    for (unsigned base = blockIdx.x * blockDim.x + warp * 32; base < total; base += stride) {
        const unsigned g = base + lane;
        if (g < total) {
            const unsigned r = g / spr, sb = g - r * spr;
            uint32_t h[16];
            sub32_to_f16<T>(W + (size_t)(r0 + r) * rb, (int)sb, h);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int q = (c + lane) & 3;        // spreads the lanes of one instruction over the banks
                stage[warp][lane * 4 + q] = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
            }
        }
        __syncwarp();
        // output of sub-blocks base .. base+31 is contiguous (row stride = cols)
        uint4* o = reinterpret_cast<uint4*>(out + (size_t)base * 32);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int idx = c * 32 + lane;           // 16-byte unit of the warp's 2 KB
            if (base + (unsigned)(idx >> 2) < total) o[idx] = stage[warp][idx];
        }
        __syncwarp();
    }
}

// Lattice types (tk_qgrid.h): as dequant_kernel, the table buffer in global
// memory (34 KB, L1/L2-resident after the first touches).
template <int T, int OUT>
__global__ void __launch_bounds__(DQ_THREADS) dequant_grid_kernel(const uint8_t* __restrict__ W, size_t rb, int r0,
                                                                  int nrows, int cols, void* __restrict__ out,
                                                                  const int8_t* __restrict__ tab) {
    const int gpr = cols >> 3;
    for (int r = blockIdx.y; r < nrows; r += gridDim.y) {
        const uint8_t* row = W + (size_t)(r0 + r) * rb;
        const size_t orow = (size_t)r * cols;
        for (int g = blockIdx.x * DQ_THREADS + threadIdx.x; g < gpr; g += gridDim.x * DQ_THREADS) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = tkq::grid_value(row, T, g * 8 + j, tab);
            store8<OUT>(out, orow + (size_t)g * 8, v);
        }
    }
}

template <int T>
static void dq_grid_out(int out_dtype, dim3 g, dim3 b, cudaStream_t s, const uint8_t* W, size_t rb, int r0,
                        int nrows, int cols, void* out, const int8_t* tab) {
    if (out_dtype == TK_DT_F32) dequant_grid_kernel<T, TK_DT_F32><<<g, b, 0, s>>>(W, rb, r0, nrows, cols, out, tab);
    else if (out_dtype == TK_DT_F16) dequant_grid_kernel<T, TK_DT_F16><<<g, b, 0, s>>>(W, rb, r0, nrows, cols, out, tab);
    else dequant_grid_kernel<T, TK_DT_BF16><<<g, b, 0, s>>>(W, rb, r0, nrows, cols, out, tab);
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
    if (out_dtype == TK_DT_F16 && (t == QT_Q4_K || t == QT_Q5_K || t == QT_Q8_0) &&
        (reinterpret_cast<uintptr_t>(W) & 15) == 0 && rb % 16 == 0) {
        if ((size_t)nrows * (cols / 32) >= (1ull << 32))
            return fail(TK_ERR_INVALID, "tk_dequant: more than 2^32 sub-blocks in one call");
        const size_t total = (size_t)nrows * (cols / 32);
        // one sub-block per thread up to 64 blocks per SM: a second, partly
        // empty pass over the grid costs more than the extra blocks
        size_t want = (total + 255) / 256, cap = (size_t)ctx->num_sms * 64;
        const dim3 grid((unsigned)(want < cap ? want : cap));
        ProfScope ps(ctx, s, PK_DEQUANT);
        const uint8_t* w = static_cast<const uint8_t*>(W);
        uint16_t* o = static_cast<uint16_t*>(out);
        if (t == QT_Q4_K) dequant_sub_f16_kernel<QT_Q4_K><<<grid, 256, 0, s>>>(w, rb, r0, nrows, cols, o);
        else if (t == QT_Q5_K) dequant_sub_f16_kernel<QT_Q5_K><<<grid, 256, 0, s>>>(w, rb, r0, nrows, cols, o);
        else dequant_sub_f16_kernel<QT_Q8_0><<<grid, 256, 0, s>>>(w, rb, r0, nrows, cols, o);
        ctx->launches++;
        return cuda_fail(cudaGetLastError(), "dequant launch");
    }
    const int gpr = cols / 8;
    if (tkq::is_grid(t)) {
        if (!ctx->iq_tab)
            return fail(TK_ERR_UNSUPPORTED, "tk_dequant: type " + std::to_string(t) +
                                                " needs the IQ grid tables (tk_set_iq_grids)");
        const int gx = (gpr + DQ_THREADS - 1) / DQ_THREADS;
        const int gy_cap = (ctx->num_sms * 16 + gx - 1) / gx;
        const int gy = nrows < gy_cap ? nrows : (gy_cap < 65535 ? gy_cap : 65535);
        const dim3 grid((unsigned)gx, (unsigned)gy), block(DQ_THREADS);
        const uint8_t* w = static_cast<const uint8_t*>(W);
        const int8_t* tab = ctx->iq_tab;
        ProfScope ps(ctx, s, PK_DEQUANT);
        switch (t) {
            case tkq::IQ2_XXS: dq_grid_out<tkq::IQ2_XXS>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out, tab); break;
            case tkq::IQ2_XS: dq_grid_out<tkq::IQ2_XS>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out, tab); break;
            case tkq::IQ2_S: dq_grid_out<tkq::IQ2_S>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out, tab); break;
            case tkq::IQ3_XXS: dq_grid_out<tkq::IQ3_XXS>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out, tab); break;
            case tkq::IQ3_S: dq_grid_out<tkq::IQ3_S>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out, tab); break;
            case tkq::IQ1_S: dq_grid_out<tkq::IQ1_S>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out, tab); break;
            default: dq_grid_out<tkq::IQ1_M>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out, tab); break;
        }
        ctx->launches++;
        return cuda_fail(cudaGetLastError(), "dequant launch");
    }
    const int gx = (gpr + DQ_THREADS * DQ_UNROLL - 1) / (DQ_THREADS * DQ_UNROLL);
    const int gy_cap = (ctx->num_sms * 16 + gx - 1) / gx;      // ~16 blocks per SM in flight
    const int gy = nrows < gy_cap ? nrows : (gy_cap < 65535 ? gy_cap : 65535);
    dim3 grid((unsigned)gx, (unsigned)gy), block(DQ_THREADS);
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
        case QT_IQ4_NL: dq_dispatch_out<QT_IQ4_NL>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_IQ4_XS: dq_dispatch_out<QT_IQ4_XS>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_MXFP4: dq_dispatch_out<QT_MXFP4>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_NF4: dq_dispatch_out<QT_NF4>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_FP4: dq_dispatch_out<QT_FP4>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_TQ1_0: dq_dispatch_out<QT_TQ1_0>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
        case QT_TQ2_0: dq_dispatch_out<QT_TQ2_0>(out_dtype, grid, block, s, w, rb, r0, nrows, cols, out); break;
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
    pdl_trigger();
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

// Vector variant: K % 8 == 0, 16-byte aligned rows.  The row stays in
// registers between the max pass and the split, so X is read from HBM once;
// loads are 16 B (bf16/fp16) or 2 x 16 B (fp32), plane stores 16 B.
constexpr int AS_THREADS = 256, AS_MAXCH = 8;    // rows up to 256*8*8 = 16384 elements

template <int XT>
__device__ __forceinline__ void ld8(const void* X, size_t i, float (&v)[8]) {
    if constexpr (XT == TK_DT_F32) {
        const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(X) + i);
        const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(X) + i + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(X) + i);
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint16_t h = (uint16_t)(u[j >> 1] >> (16 * (j & 1)));
            v[j] = XT == TK_DT_F16 ? h2f_bits(h) : __uint_as_float((uint32_t)h << 16);
        }
    }
}

__device__ __forceinline__ void st8h(uint16_t* p, const uint16_t (&h)[8]) {
    *reinterpret_cast<uint4*>(p) = make_uint4((uint32_t)h[0] | ((uint32_t)h[1] << 16), (uint32_t)h[2] | ((uint32_t)h[3] << 16),
                                              (uint32_t)h[4] | ((uint32_t)h[5] << 16), (uint32_t)h[6] | ((uint32_t)h[7] << 16));
}

// The raw 16-byte chunks (8 elements of a 16-bit type, or 4 of fp32 in two
// halves) stay in registers between the max and split passes and are decoded
// twice; keeping raw bits instead of floats halves the register footprint.
template <int XT>
struct RawChunk {
    uint4 a, b;   // b unused for 16-bit types
};
template <int XT>
__device__ __forceinline__ void ld_raw(const void* X, size_t i, RawChunk<XT>& r) {
    if constexpr (XT == TK_DT_F32) {
        r.a = *reinterpret_cast<const uint4*>(static_cast<const float*>(X) + i);
        r.b = *reinterpret_cast<const uint4*>(static_cast<const float*>(X) + i + 4);
    } else {
        r.a = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(X) + i);
    }
}
template <int XT>
__device__ __forceinline__ void dec_raw(const RawChunk<XT>& r, float (&v)[8]) {
    if constexpr (XT == TK_DT_F32) {
        v[0] = __uint_as_float(r.a.x); v[1] = __uint_as_float(r.a.y); v[2] = __uint_as_float(r.a.z); v[3] = __uint_as_float(r.a.w);
        v[4] = __uint_as_float(r.b.x); v[5] = __uint_as_float(r.b.y); v[6] = __uint_as_float(r.b.z); v[7] = __uint_as_float(r.b.w);
    } else {
        const uint32_t u[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint16_t h = (uint16_t)(u[j >> 1] >> (16 * (j & 1)));
            v[j] = XT == TK_DT_F16 ? h2f_bits(h) : __uint_as_float((uint32_t)h << 16);
        }
    }
}

template <int XT, int NP, int TH>
__global__ void __launch_bounds__(TH) act_split_vec_kernel(const void* __restrict__ X, int M, int K, long ldx,
                                                                   long ldp, bool scaled, uint16_t* __restrict__ planes,
                                                                   int* __restrict__ row_exp) {
    pdl_trigger();
    __shared__ float red[TH / 32];
    const int m = blockIdx.x;
    const int nch = K >> 3;
    RawChunk<XT> raw[AS_MAXCH];
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < AS_MAXCH; ++i) {
        const int c = threadIdx.x + i * TH;
        if (c < nch) ld_raw<XT>(X, (size_t)m * ldx + (size_t)c * 8, raw[i]);
    }
#pragma unroll
    for (int i = 0; i < AS_MAXCH; ++i) {
        const int c = threadIdx.x + i * TH;
        if (c < nch) {
            float v[8];
            dec_raw<XT>(raw[i], v);
#pragma unroll
            for (int j = 0; j < 8; ++j) a = fmaxf(a, fabsf(v[j]));
        }
    }
    int e = 0;
    if (scaled) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
        __syncthreads();
        a = red[0];
#pragma unroll
        for (int w = 1; w < TH / 32; ++w) a = fmaxf(a, red[w]);
        e = row_exponent(a);
    }
    if (threadIdx.x == 0 && row_exp) row_exp[m] = e;
    const float f = pow2f(e);
    const size_t pstride = (size_t)M * ldp;
    uint16_t* orow = planes + (size_t)m * ldp;
#pragma unroll
    for (int i = 0; i < AS_MAXCH; ++i) {
        const int c = threadIdx.x + i * TH;
        if (c >= nch) continue;
        float v[8];
        dec_raw<XT>(raw[i], v);
        if constexpr (NP == 1) {
            // one packed conversion per pair (round to nearest even, as f2h_bits)
            uint32_t hp[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const __half2 p2 = __floats2half2_rn(v[2 * j] * f, v[2 * j + 1] * f);
                hp[j] = *reinterpret_cast<const uint32_t*>(&p2);
            }
            *reinterpret_cast<uint4*>(orow + (size_t)c * 8) = make_uint4(hp[0], hp[1], hp[2], hp[3]);
            continue;
        }
        uint16_t h[8], mm[8], l[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float x = v[j] * f;
            h[j] = f2h_bits(x);
            if constexpr (NP >= 2) {
                const float r = x - h2f_bits(h[j]);
                mm[j] = f2h_bits(r);
                if constexpr (NP == 3) l[j] = f2h_bits(r - h2f_bits(mm[j]));
            }
        }
        st8h(orow + (size_t)c * 8, h);
        if constexpr (NP >= 2) st8h(orow + pstride + (size_t)c * 8, mm);
        if constexpr (NP == 3) st8h(orow + 2 * pstride + (size_t)c * 8, l);
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
    const size_t esz = x_dtype == TK_DT_F32 ? 4 : 2;
    const bool vec = K % 8 == 0 && ldx % 8 == 0 && ldp % 8 == 0 && K <= AS_THREADS * AS_MAXCH * 8 &&
                     (reinterpret_cast<uintptr_t>(X) % 16) == 0 && (reinterpret_cast<uintptr_t>(planes) % 16) == 0 &&
                     (ldx * esz) % 16 == 0;
    if (vec) {
        // rows of up to 4096 elements take 128-thread blocks (4 chunks per
        // thread): twice the blocks per SM, so more bytes in flight per SM
        const bool narrow = K <= 128 * 4 * 8;
#define TK_SPLIT_VEC_TH(XT, TH)                                                                                       \
    do {                                                                                                              \
        if (nplanes == 1) act_split_vec_kernel<XT, 1, TH><<<M, TH, 0, s>>>(X, M, K, ldx, ldp, scaled, planes, row_exp); \
        else if (nplanes == 2) act_split_vec_kernel<XT, 2, TH><<<M, TH, 0, s>>>(X, M, K, ldx, ldp, scaled, planes, row_exp); \
        else act_split_vec_kernel<XT, 3, TH><<<M, TH, 0, s>>>(X, M, K, ldx, ldp, scaled, planes, row_exp);          \
    } while (0)
#define TK_SPLIT_VEC(XT)                                                                                              \
    do {                                                                                                              \
        if (narrow) TK_SPLIT_VEC_TH(XT, 128);                                                                         \
        else TK_SPLIT_VEC_TH(XT, AS_THREADS);                                                                         \
    } while (0)
        if (x_dtype == TK_DT_F32) TK_SPLIT_VEC(TK_DT_F32);
        else if (x_dtype == TK_DT_F16) TK_SPLIT_VEC(TK_DT_F16);
        else if (x_dtype == TK_DT_BF16) TK_SPLIT_VEC(TK_DT_BF16);
        else return fail(TK_ERR_INVALID, "activation dtype " + std::to_string(x_dtype));
#undef TK_SPLIT_VEC
#undef TK_SPLIT_VEC_TH
        ctx->launches++;
        return cuda_fail(cudaGetLastError(), "act_split launch");
    }
    if (x_dtype == TK_DT_F32) act_split_np<TK_DT_F32>(nplanes, M, K, ldx, ldp, scaled, X, planes, row_exp, s);
    else if (x_dtype == TK_DT_F16) act_split_np<TK_DT_F16>(nplanes, M, K, ldx, ldp, scaled, X, planes, row_exp, s);
    else if (x_dtype == TK_DT_BF16) act_split_np<TK_DT_BF16>(nplanes, M, K, ldx, ldp, scaled, X, planes, row_exp, s);
    else return fail(TK_ERR_INVALID, "activation dtype " + std::to_string(x_dtype));
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "act_split launch");
}

// fp32 -> fp16 bits as tier_fp16::from_float (tier/gpu_compat.h:151-171):
// round to nearest even, overflow to inf, and every NaN encoded as its sign
// with 0x7e00 (the hardware conversion would keep NaN payload bits).
__device__ __forceinline__ uint16_t f2h_ref(float v) {
    if (isnan(v)) return (uint16_t)(((__float_as_uint(v) >> 16) & 0x8000u) | 0x7e00u);
    return f2h_bits(v);
}

// split3_fp_k exactly (no scaling): h = f16(x), m = f16(x-h), l = f16(x-h-m).
__global__ void split3_raw_kernel(const float* __restrict__ x, size_t n, uint16_t* __restrict__ h,
                                  uint16_t* __restrict__ m, uint16_t* __restrict__ l) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        const uint16_t a = f2h_ref(v);
        const float r = v - h2f_bits(a);
        const uint16_t b = f2h_ref(r);
        h[i] = a;
        m[i] = b;
        l[i] = f2h_ref(r - h2f_bits(b));
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
