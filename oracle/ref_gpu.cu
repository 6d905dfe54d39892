// ref_gpu.cu -- the REFERENCE engine's own GPU linear path, compiled from its
// sources, for timing beside libtierk in bench.py's reference arm (and for
// tests).  Test infrastructure: never linked into the product.
//
// tier/tier.cpp is compiled whole, as its own build compiles it
// (tier/build.sh:89: nvcc -x cu -DTIER_CUDA, cuBLAS / cuBLASLt), with its
// main renamed, so that these entry points run the engine's functions
// unchanged:
//   refgpu_fp3gemm_fwd   linear -> low3_linear -> fp3gemm (tier/tier.cpp:1186-1209,
//                        922-943): split3_fp_k of X, then three cuBLASLt GEMMs
//                        W.xl, W.xm, W.xh accumulating into Y (fp16 in, fp32 out)
//   refgpu_fp3gemm_dx    linear_dx's fp3gemm (tier/tier.cpp:1217-1231)
//   refgpu_dequant_f16   dq_launch / dq_k to fp16 (tier/tier.cpp:294-298), the
//                        training path's per-pass expansion of a quantized W
//   refgpu_gemv_q        gemv_q as chat_lin launches it for one token
//                        (tier/tier.cpp:300-306, 2357): 8 warps per block
// The built library lives in oracle/_ref/ (git-ignored); nothing from the
// reference is stored in this repository.
#define main tier_ref_main
#include "tier.cpp"
#undef main

extern "C" {

int refgpu_fp3gemm_fwd(const void* W16, const float* X, float* Y, int M, int K, int N)
{
    fp3gemm(nullptr, HIPBLAS_OP_T, N, M, K, (const tier_fp16*)W16, K, X, 0.0f, Y, N);
    return (int)hipGetLastError();
}

int refgpu_fp3gemm_dx(const void* W16, const float* dY, float* dX, int M, int K, int N)
{
    fp3gemm(nullptr, HIPBLAS_OP_N, K, M, N, (const tier_fp16*)W16, K, dY, 0.0f, dX, K);
    return (int)hipGetLastError();
}

int refgpu_dequant_f16(const void* W, int type, size_t rb, int rows, int cols, void* out)
{
    QRef Q{};
    Q.type = type;
    Q.rows = rows;
    Q.cols = cols;
    Q.rb = rb;
    dq_launch(W, Q, 0, (size_t)rows, (tier_fp16*)out);
    return (int)hipGetLastError();
}

int refgpu_gemv_q(const void* W, int type, size_t rb, const float* x, float* y, int N, int K)
{
    const int wpb = 256 / 32;
    gemv_q<<<(N + wpb - 1) / wpb, 256>>>((const uint8_t*)W, type, rb, x, y, N, K);
    return (int)hipGetLastError();
}

int refgpu_sync(void) { return (int)hipDeviceSynchronize(); }

}  // extern "C"
