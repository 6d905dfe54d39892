// ref_harness.cpp -- thin C-ABI shim over the REFERENCE's own code, for tests
// and the timed CPU baseline only (never linked into the product).
//
// It is compiled (oracle/Makefile) against the reference's quant.h where it
// lies (tier/quant.h, tier/quant_tables.h) and against kernel bodies that
// oracle/extract_ref.py copies out of tier/tier.cpp into oracle/_ref/ at build
// time -- the same extraction the reference's own test tier/cpu_gpu_sim.py:13-27
// performs.  Nothing from the reference is stored in this repository; the
// built .so lives in oracle/_ref/ (git-ignored).
//
// Exports:
//   ref_q_val / ref_dequant      tier/quant.h:59-121 (q_val), tier/tier.cpp:294-296 (dq_k)
//   ref_q_row                    tier/quant.h:201-204 (CPU quantizers)
//   ref_split3_fp16              tier/tier.cpp:869-870 (split3_fp_k, extracted)
//   ref_dlogit                   tier/tier.cpp:736-748 (dlogit_kernel, extracted)
//   ref_softcap                  tier/tier.cpp:728 (softcap_kernel, extracted)
//   ref_lse_chunk                tier/tier.cpp:750-759 (lse_chunk_kernel, extracted;
//                                each block runs as 256 host threads with a
//                                barrier for __syncthreads, as launched at 3219)
//   ref_cpu_qgemm_fwd / _dx      a restatement (not the reference's code):
//                                q_val row expansion + the cpu_gemm_fwd /
//                                cpu_gemm_dx loop structure over fp32 rows
//   ref_cpu_pool, ref_cpu_gemm_fwd / _dx, ref_dequant_bf16
//                                the engine's own CPU GEMMs, extracted
//                                (cpu_gemm_fwd / cpu_gemm_dx with pool_run and
//                                its workers, tier/tier.cpp:1015-1099): AVX2 FMA
//                                over bf16 weight rows; ref_dequant_bf16 feeds
//                                them q_val rounded to bf16 (nearest even).
#include "quant.h"
#include <cstdint>
#include <cstring>
#include <cmath>
#include <thread>
#include <vector>
#include <algorithm>
#include <functional>
#include <mutex>
#include <condition_variable>

// ---- emulated CUDA launch environment for the extracted kernel bodies ----
namespace refsim {
struct dim { unsigned x = 0, y = 0, z = 0; };
static thread_local dim threadIdx, blockIdx, blockDim;
// __syncthreads for one block run as blockDim.x host threads (one block at a
// time, so a kernel's __shared__ arrays can be function statics)
struct Barrier {
    std::mutex m;
    std::condition_variable cv;
    unsigned n = 0, waiting = 0, gen = 0;
    void wait() {
        std::unique_lock<std::mutex> lk(m);
        const unsigned g = gen;
        if (++waiting == n) { waiting = 0; ++gen; cv.notify_all(); return; }
        cv.wait(lk, [&] { return gen != g; });
    }
};
static Barrier block_barrier;
}
using refsim::threadIdx;
using refsim::blockIdx;
using refsim::blockDim;
#define __host__
#define __device__
#define __global__
#define __shared__ static
#define __syncthreads() refsim::block_barrier.wait()
typedef unsigned short ref_u16;
#include "ref_kernels.inc"   // generated: tier_fp16 + split3_fp_k + dlogit_kernel + softcap_kernel

extern "C" {

float ref_q_val(const uint8_t* row, int type, int col) { return q_val(row, type, col); }

size_t ref_row_bytes(int type, int cols) { return q_row_bytes(type, cols); }

// out_dtype: 0 fp32, 1 fp16 (tier_fp16 RNE, the training storage path)
void ref_dequant(const uint8_t* W, size_t rb, int type, int r0, int nrows, int cols, int out_dtype, void* out)
{
    for (int r = 0; r < nrows; ++r) {
        const uint8_t* row = W + (size_t)(r0 + r) * rb;
        for (int c = 0; c < cols; ++c) {
            float v = q_val(row, type, c);
            size_t o = (size_t)r * cols + c;
            if (out_dtype == 0) ((float*)out)[o] = v;
            else ((uint16_t*)out)[o] = tier_fp16(v).bits;
        }
    }
}

int ref_q_row(int type, const float* x, uint8_t* o, int k) { return q_row(type, x, o, k) ? 1 : 0; }

void ref_split3_fp16(const float* x, uint16_t* h, uint16_t* m, uint16_t* l, size_t n)
{
    blockDim.x = 256;
    for (size_t i = 0; i < n; ++i) {
        blockIdx.x = (unsigned)(i / 256); threadIdx.x = (unsigned)(i % 256);
        split3_fp_k(x, (tier_fp16*)h, (tier_fp16*)m, (tier_fp16*)l, n);
    }
}

void ref_dlogit(const float* lg, const double* rmax, const double* rsum, const int32_t* tokens, float* dl,
                int seq_len, int vc, int v0, int n_loss, const unsigned char* mask, float cap)
{
    blockDim.x = 256;
    size_t n = (size_t)seq_len * vc;
    for (size_t i = 0; i < n; ++i) {
        blockIdx.x = (unsigned)(i / 256); threadIdx.x = (unsigned)(i % 256);
        dlogit_kernel(lg, rmax, rsum, tokens, dl, seq_len, vc, v0, n_loss, mask, cap);
    }
}

// lse_chunk_kernel<<<n_pred, 256>>> (tier/tier.cpp:3219): blocks one after
// another, each as 256 threads.
void ref_lse_chunk(const float* lg, double* rmax, double* rsum, int* amax, float* tgt, const int32_t* tokens,
                   const unsigned char* mask, int n_pred, int vc, int v0)
{
    const unsigned nt = 256;
    refsim::block_barrier.n = nt;
    for (int b = 0; b < n_pred; ++b) {
        std::vector<std::thread> th;
        for (unsigned i = 0; i < nt; ++i)
            th.emplace_back([=] {
                blockDim.x = nt; blockIdx.x = (unsigned)b; threadIdx.x = i;
                lse_chunk_kernel(lg, rmax, rsum, amax, tgt, tokens, mask, vc, v0);
            });
        for (auto& t : th) t.join();
    }
}

void ref_softcap(float* lg, float cap, size_t n)
{
    blockDim.x = 256;
    for (size_t i = 0; i < n; ++i) {
        blockIdx.x = (unsigned)(i / 256); threadIdx.x = (unsigned)(i % 256);
        softcap_kernel(lg, cap, n);
    }
}

// ---- CPU baseline ----------------------------------------------------------
static void run_rows(int n_items, int threads, const std::function<void(int, int)>& f)
{
    if (threads < 2) { f(0, n_items); return; }
    std::vector<std::thread> th;
    for (int t = 0; t < threads; ++t) {
        int a = (int)((long long)n_items * t / threads), b = (int)((long long)n_items * (t + 1) / threads);
        if (b > a) th.emplace_back(f, a, b);
    }
    for (auto& x : th) x.join();
}

// Y[m, n0+i] = sum_k X[m,k] * q_val(W[n0+i], k) for i < nrows.  ldy = row
// stride of Y.  Each worker expands one weight row to fp32 with q_val and
// dots it against 4 token rows at a time (cpu_gemm_fwd's blocking).
void ref_cpu_qgemm_fwd(const uint8_t* W, size_t rb, int type, int n0, int nrows, int K,
                       const float* X, int M, float* Y, int ldy, int threads)
{
    run_rows(nrows, threads, [&](int a, int b) {
        std::vector<float> w(K);
        for (int i = a; i < b; ++i) {
            const uint8_t* row = W + (size_t)(n0 + i) * rb;
            for (int k = 0; k < K; ++k) w[k] = q_val(row, type, k);
            for (int m = 0; m < M; m += 4) {
                int mm = std::min(4, M - m);
                float r[4] = {0, 0, 0, 0};
                for (int j = 0; j < mm; ++j) {
                    const float* x = X + (size_t)(m + j) * K;
                    float acc = 0;
#pragma omp simd reduction(+ : acc)
                    for (int k = 0; k < K; ++k) acc += w[k] * x[k];
                    r[j] = acc;
                }
                for (int j = 0; j < mm; ++j) Y[(size_t)(m + j) * ldy + i] = r[j];
            }
        }
    });
}

// dX[m,k] = sum_{i<nrows} dY[m, i] * q_val(W[n0+i], k); per-thread partial
// [M,K] accumulators summed at the end (cpu_gemm_dx's structure).
void ref_cpu_qgemm_dx(const uint8_t* W, size_t rb, int type, int n0, int nrows, int K,
                      const float* dY, int lddy, int M, float* dX, int threads)
{
    int T = threads < 1 ? 1 : threads;
    std::vector<std::vector<float>> part(T);
    std::vector<std::thread> th;
    auto job = [&](int id, int a, int b) {
        auto& acc = part[id];
        acc.assign((size_t)M * K, 0.0f);
        std::vector<float> w(K);
        for (int i = a; i < b; ++i) {
            const uint8_t* row = W + (size_t)(n0 + i) * rb;
            for (int k = 0; k < K; ++k) w[k] = q_val(row, type, k);
            for (int m = 0; m < M; ++m) {
                float c = dY[(size_t)m * lddy + i];
                if (c == 0.0f) continue;
                float* o = acc.data() + (size_t)m * K;
#pragma omp simd
                for (int k = 0; k < K; ++k) o[k] += c * w[k];
            }
        }
    };
    for (int t = 0; t < T; ++t) {
        int a = (int)((long long)nrows * t / T), b = (int)((long long)nrows * (t + 1) / T);
        th.emplace_back(job, t, a, b);
    }
    for (auto& x : th) x.join();
    std::memset(dX, 0, (size_t)M * K * sizeof(float));
    for (int t = 0; t < T; ++t) {
        if (part[t].size() != (size_t)M * K) continue;
        const float* a = part[t].data();
        for (size_t i = 0, n = (size_t)M * K; i < n; ++i) dX[i] += a[i];
    }
}

}  // extern "C"

// ---- the engine's CPU GEMMs (tier/tier.cpp:1015-1099), extracted ----
#include <immintrin.h>
#include <atomic>
#include <chrono>
static int g_cpu_thr = 1;   // the engine's CPU thread count (pool_init starts that many workers)
#include "ref_cpu_gemm.inc"

extern "C" {

// Start the reference's thread pool with `threads` workers (once; later
// calls with another count restart it, as pool_init does).
void ref_cpu_pool(int threads)
{
    g_cpu_thr = threads;
    pool_init();
}

void ref_cpu_gemm_fwd(const float* X, const uint16_t* Wbf16, float* out, int M, int K, int N)
{
    cpu_gemm_fwd(X, Wbf16, out, M, K, N);
}

void ref_cpu_gemm_dx(const float* dY, const uint16_t* Wbf16, float* dX, int M, int K, int N)
{
    cpu_gemm_dx(dY, Wbf16, dX, M, K, N);
}

// rows n0 .. n0+nrows of a block-quantized W as bf16 (q_val, then nearest
// even), the weight form the engine's CPU GEMMs read; rows split over
// the pool like the GEMMs themselves.
void ref_dequant_bf16(const uint8_t* W, size_t rb, int type, int n0, int nrows, int K, uint16_t* out)
{
    pool_run(nrows, [&](int a, int b) {
        for (int i = a; i < b; ++i) {
            const uint8_t* row = W + (size_t)(n0 + i) * rb;
            uint16_t* o = out + (size_t)i * K;
            for (int k = 0; k < K; ++k) {
                float f = q_val(row, type, k);
                uint32_t u;
                std::memcpy(&u, &f, 4);
                u += 0x7FFFu + ((u >> 16) & 1u);
                o[k] = (uint16_t)(u >> 16);
            }
        }
    });
}

}  // extern "C"

