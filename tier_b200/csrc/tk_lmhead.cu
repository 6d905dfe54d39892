// tk_lmhead.cu -- small kernels around the LM-head GEMMs:
//   * merge of per-(row, 256-column tile) partial statistics produced by the
//     logits GEMM epilogue into the running fp64 state, with the semantics of
//     lse_chunk_kernel (tier/tier.cpp:750-759): chunk max with its lowest
//     index, fp64 sum of exp(logit - chunk max), running merge
//     rsum = rsum*e^(om-nm) + s*e^(bm-nm), target logit of labels[t+1];
//   * the loss / hit count of tier/tier.cpp:3227-3228;
//   * the max-rescale used between all-reduces when the vocab is sharded.
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

// One warp per predicted row.
__global__ void lse_merge_kernel(const float* __restrict__ pmax, const int32_t* __restrict__ parg,
                                 const double* __restrict__ psum, const float* __restrict__ ptgt, int ld_part,
                                 int ntiles, int n_pred, int vc, int v0, const int32_t* __restrict__ labels,
                                 const uint8_t* __restrict__ mask, double* rmax, double* rsum, int32_t* amax,
                                 float* tgt) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= n_pred || !mask[t]) return;
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
        const int g = labels[t + 1] - v0;
        if (g >= 0 && g < vc) tgt[t] = ptgt[base + (g >> 8)];
    }
}

tk_status launch_lse_merge(tk_ctx* ctx, const float* pmax, const int32_t* parg, const double* psum, const float* ptgt,
                           int ld_part, int ntiles, int n_pred, int vc, int v0, const int32_t* labels,
                           const uint8_t* mask, double* rmax, double* rsum, int32_t* amax, float* tgt,
                           cudaStream_t s) {
    if (n_pred <= 0) return TK_OK;
    const int warps = 8;
    ProfScope ps(ctx, s, PK_LMHEAD);
    lse_merge_kernel<<<(n_pred + warps - 1) / warps, warps * 32, 0, s>>>(pmax, parg, psum, ptgt, ld_part, ntiles,
                                                                          n_pred, vc, v0, labels, mask, rmax, rsum,
                                                                          amax, tgt);
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

__global__ void lm_rescale_kernel(int n, double* rmax_l, double* rsum_l, const double* rmax_g) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    const double g = rmax_g[t];
    rsum_l[t] *= exp(rmax_l[t] - g);
    rmax_l[t] = g;
}

tk_status launch_lm_rescale(tk_ctx* ctx, int n, double* rmax_l, double* rsum_l, const double* rmax_g,
                            cudaStream_t s) {
    if (n <= 0) return TK_OK;
    ProfScope ps(ctx, s, PK_LMHEAD);
    lm_rescale_kernel<<<(n + 255) / 256, 256, 0, s>>>(n, rmax_l, rsum_l, rmax_g);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "lm rescale launch");
}

}  // namespace tk
