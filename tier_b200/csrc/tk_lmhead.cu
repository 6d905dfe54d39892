// tk_lmhead.cu -- small kernels around the LM-head GEMMs:
//   * merge of per-(row, 256-column tile) partial statistics produced by the
//     logits GEMM epilogue into the running fp64 state, with the semantics of
//     lse_chunk_kernel (tier/tier.cpp:750-759): chunk max with its lowest
//     index, fp64 sum of exp(logit - chunk max), running merge
//     rsum = rsum*e^(om-nm) + s*e^(bm-nm), target logit of labels[t+1];
//   * the loss / hit count of tier/tier.cpp:3227-3228;
//   * the max-rescale used between all-reduces when the vocab is sharded;
//   * the single-pass head's probability planes and final dX scaling.
//
// Single pass (one logits GEMM per chunk instead of two): the logits GEMM
// stores the chunk's logits, the merge records alpha[t] = exp(m_old - m_new),
// lm_prob writes P = exp(l - m_new) * (1 - (l/cap)^2) (<= 1) as fp16 hi + lo,
// and the dX GEMM computes dXacc = alpha * dXacc + P . W_chunk.  At the end
// dXacc = sum_v exp(l_v - m) g_v W_v with m the final max, so
//   dX = (exp(l - lse) - onehot) g W / n = dXacc / (n S) - g_t W_t / n,
// S = sum_v exp(l_v - m): the reference's dlogit (tier/tier.cpp:736-748)
// summed against W without a second logits GEMM.
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

// One warp per predicted row.
__global__ void lse_merge_kernel(const float* __restrict__ pmax, const int32_t* __restrict__ parg,
                                 const double* __restrict__ psum, const float* __restrict__ ptgt, int ld_part,
                                 int ntiles, int n_pred, int vc, int v0, const int32_t* __restrict__ labels,
                                 const uint8_t* __restrict__ mask, double* rmax, double* rsum, int32_t* amax,
                                 float* tgt, float* alpha) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= n_pred) return;
    if (!mask[t]) {
        if (alpha && lane == 0) alpha[t] = 1.0f;   // row stays zero; any finite factor
        return;
    }
    const size_t base = (size_t)t * ld_part;
    float bm = -1e30f;
    int bi = 0x7fffffff;
    for (int j = lane; j < ntiles; j += 32) {
        const float m = pmax[base + j];
        const int a = parg[base + j];
        if (m > bm || (m == bm && a < bi)) { bm = m; bi = a; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m = __shfl_xor_sync(0xffffffffu, bm, o);
        const int a = __shfl_xor_sync(0xffffffffu, bi, o);
        if (m > bm || (m == bm && a < bi)) { bm = m; bi = a; }
    }
    double s = 0.0;
    for (int j = lane; j < ntiles; j += 32) s += psum[base + j] * exp((double)pmax[base + j] - (double)bm);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
        const double om = rmax[t], nm = fmax(om, (double)bm);
        if ((double)bm > om) amax[t] = v0 + bi;
        rsum[t] = rsum[t] * exp(om - nm) + s * exp((double)bm - nm);
        rmax[t] = nm;
        if (alpha) alpha[t] = (float)exp(om - nm);
        const int g = labels[t + 1] - v0;
        if (g >= 0 && g < vc) tgt[t] = ptgt[base + (g >> 8)];
    }
}

tk_status launch_lse_merge(tk_ctx* ctx, const float* pmax, const int32_t* parg, const double* psum, const float* ptgt,
                           int ld_part, int ntiles, int n_pred, int vc, int v0, const int32_t* labels,
                           const uint8_t* mask, double* rmax, double* rsum, int32_t* amax, float* tgt,
                           cudaStream_t s, float* alpha) {
    if (n_pred <= 0) return TK_OK;
    const int warps = 8;
    ProfScope ps(ctx, s, PK_LMHEAD);
    lse_merge_kernel<<<(n_pred + warps - 1) / warps, warps * 32, 0, s>>>(pmax, parg, psum, ptgt, ld_part, ntiles,
                                                                          n_pred, vc, v0, labels, mask, rmax, rsum,
                                                                          amax, tgt, alpha);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "lse merge launch");
}

// Single block: deterministic fp64 loss sum and hit count.
__global__ void lm_loss_kernel(int T, const int32_t* __restrict__ labels, const uint8_t* __restrict__ mask,
                               const double* __restrict__ rmax, const double* __restrict__ rsum,
                               const int32_t* __restrict__ amax, const float* __restrict__ tgt, double* loss,
                               int32_t* hits) {
    __shared__ double sl[256];
    __shared__ int sh[256];
    double l = 0.0;
    int h = 0;
    for (int t = threadIdx.x; t < T - 1; t += blockDim.x) {
        if (!mask[t]) continue;
        l += rmax[t] + log(rsum[t]) - (double)tgt[t];
        h += amax[t] == labels[t + 1];
    }
    sl[threadIdx.x] = l;
    sh[threadIdx.x] = h;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o) {
            sl[threadIdx.x] += sl[threadIdx.x + o];
            sh[threadIdx.x] += sh[threadIdx.x + o];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        *loss = sl[0];
        *hits = sh[0];
    }
}

tk_status launch_lm_loss(tk_ctx* ctx, int T, const int32_t* labels, const uint8_t* mask, const double* rmax,
                         const double* rsum, const int32_t* amax, const float* tgt, double* loss, int32_t* hits,
                         cudaStream_t s) {
    ProfScope ps(ctx, s, PK_LMHEAD);
    lm_loss_kernel<<<1, 256, 0, s>>>(T, labels, mask, rmax, rsum, amax, tgt, loss, hits);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "lm loss launch");
}

// One block per row: rsum and (optionally) the dX accumulator row scale by
// exp(rmax_local - rmax_global).
__global__ void lm_rescale_kernel(int n, double* rmax_l, double* rsum_l, const double* rmax_g, float* dX, int H) {
    const int t = blockIdx.x;
    if (t >= n) return;
    const double g = rmax_g[t], l = rmax_l[t];
    const double f = exp(l - g);
    if (dX) {
        const float ff = (float)f;
        float* row = dX + (size_t)t * H;
        for (int h = threadIdx.x; h < H; h += blockDim.x) row[h] *= ff;
    }
    __syncthreads();     // every thread read rmax_l before it changes
    if (threadIdx.x == 0) {
        rsum_l[t] *= f;
        rmax_l[t] = g;
    }
}

tk_status launch_lm_rescale(tk_ctx* ctx, int n, double* rmax_l, double* rsum_l, const double* rmax_g,
                            cudaStream_t s, float* dX, int H) {
    if (n <= 0) return TK_OK;
    ProfScope ps(ctx, s, PK_LMHEAD);
    lm_rescale_kernel<<<n, 128, 0, s>>>(n, rmax_l, rsum_l, rmax_g, dX, H);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "lm rescale launch");
}

// P planes: one thread per 8 consecutive columns of one row.
__global__ void lm_prob_kernel(const float* __restrict__ Z, long ldz, int rows, int vc, const double* __restrict__ rmax,
                               const uint8_t* __restrict__ mask, float cap, uint16_t* __restrict__ planes,
                               long plane_stride, int ld) {
    const int per_row = vc / 8;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)rows * per_row) return;
    const int t = (int)(i / per_row), c = (int)(i - (long)t * per_row) * 8;
    uint4 hv = make_uint4(0u, 0u, 0u, 0u), lv = make_uint4(0u, 0u, 0u, 0u);
    if (mask[t]) {
        const float m = (float)rmax[t];
        const float4 z0 = *reinterpret_cast<const float4*>(Z + (size_t)t * ldz + c);
        const float4 z1 = *reinterpret_cast<const float4*>(Z + (size_t)t * ldz + c + 4);
        const float l[8] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w};
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t hh = 0, ll = 0;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float x = l[2 * k + j];
                float pv = expf(x - m);
                if (cap > 0.0f) {
                    const float y = x / cap;
                    pv *= 1.0f - y * y;
                }
                const uint16_t h = f2h_bits(pv);
                const uint16_t lo = f2h_bits(pv - h2f_bits(h));
                hh |= (uint32_t)h << (16 * j);
                ll |= (uint32_t)lo << (16 * j);
            }
            hw[k] = hh;
            lw[k] = ll;
        }
        hv = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        lv = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    *reinterpret_cast<uint4*>(planes + (size_t)t * ld + c) = hv;
    *reinterpret_cast<uint4*>(planes + plane_stride + (size_t)t * ld + c) = lv;
}

tk_status launch_lm_prob(tk_ctx* ctx, const float* Z, long ldz, int rows, int vc, const double* rmax,
                         const uint8_t* mask, float cap, uint16_t* planes, long plane_stride, int ld, cudaStream_t s) {
    if (rows <= 0 || vc <= 0) return TK_OK;
    const long n = (long)rows * (vc / 8);
    ProfScope ps(ctx, s, PK_LMHEAD);
    lm_prob_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(Z, ldz, rows, vc, rmax, mask, cap, planes,
                                                                 plane_stride, ld);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "lm prob launch");
}

// One block per row t < T: live rows scale and subtract the label's W row.
__global__ void lm_finish_kernel(const uint16_t* __restrict__ W, int v0, int V_shard, int H, int T,
                                 const int32_t* __restrict__ labels, const uint8_t* __restrict__ mask, int n_loss,
                                 float cap, const double* __restrict__ rsum, const float* __restrict__ tgt,
                                 float* __restrict__ dX) {
    const int t = blockIdx.x;
    float* row = dX + (size_t)t * H;
    const bool live = t < T - 1 && mask[t] != 0;
    if (!live) {
        for (int h = threadIdx.x; h < H; h += blockDim.x) row[h] = 0.0f;
        return;
    }
    const float inv = (float)(1.0 / ((double)n_loss * rsum[t]));
    const int lab = labels[t + 1] - v0;
    const bool own = lab >= 0 && lab < V_shard;
    float gt = 1.0f / (float)n_loss;
    if (cap > 0.0f) {
        const float y = tgt[t] / cap;
        gt *= 1.0f - y * y;
    }
    const uint16_t* wr = W + (size_t)(own ? lab : 0) * H;
    for (int h = threadIdx.x; h < H; h += blockDim.x) {
        float v = row[h] * inv;
        if (own) v -= gt * h2f_bits(wr[h]);
        row[h] = v;
    }
}

tk_status launch_lm_finish(tk_ctx* ctx, const uint16_t* W, int v0, int V_shard, int H, int T, const int32_t* labels,
                           const uint8_t* mask, int n_loss, float cap, const double* rsum, const float* tgt, float* dX,
                           cudaStream_t s) {
    if (T <= 0) return TK_OK;
    ProfScope ps(ctx, s, PK_LMHEAD);
    lm_finish_kernel<<<T, 256, 0, s>>>(W, v0, V_shard, H, T, labels, mask, n_loss, cap, rsum, tgt, dX);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "lm finish launch");
}

}  // namespace tk
