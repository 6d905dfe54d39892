// tk_noalloc.cu -- tk_linear_fwd_noalloc: the forward linear for callers that
// cannot allocate device memory.
//
// Who needs it: an engine that owns every byte of VRAM through its own arena
// and budget (tierlm's training engine accounts for each allocation and
// relieves memory pressure itself), or host code that must not allocate once
// its steady state has begun.  tk_linear_fwd grows a per-context workspace
// with cudaMalloc on demand; this variant never does.
//
// Its scratch -- the fp16 split planes of X and the per-row scale exponents --
// lives in one file-scope device array of kScratchBytes (24 MiB).  Every GPU
// that loads libtierk.so holds that array until the process exits.  Host code
// cannot use the array's name as a device address, so the first call on each
// device looks the address up with cudaGetSymbolAddress (with that device
// current) and caches it; make that first call before any stream capture.
// All calls on one device share the array: each call rewrites every scratch
// byte it reads, so nothing has to start at zero, but calls whose GPU work
// overlaps (different streams, host threads or contexts on the same device)
// race on the array; the caller must order them.
#include <mutex>
#include <string>
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

constexpr size_t kScratchBytes = 24u << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
static std::mutex g_scratch_mu;
static void* g_scratch_ptr[kMaxDevices];

// Device address of g_noalloc_scratch on `device` (looked up once per device).
static tk_status scratch_address(int device, void** out) {
    if (device < 0 || device >= kMaxDevices) return fail(TK_ERR_UNSUPPORTED, "tk_linear_fwd_noalloc: device index");
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[device]) {
        int cur = -1;
        cudaError_t e = cudaGetDevice(&cur);
        if (e != cudaSuccess) return cuda_fail(e, "tk_linear_fwd_noalloc: cudaGetDevice");
        if (cur != device && (e = cudaSetDevice(device)) != cudaSuccess)
            return cuda_fail(e, "tk_linear_fwd_noalloc: cudaSetDevice");
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (cur != device) cudaSetDevice(cur);
        if (e != cudaSuccess) return cuda_fail(e, "tk_linear_fwd_noalloc: cudaGetSymbolAddress");
        g_scratch_ptr[device] = p;
    }
    *out = g_scratch_ptr[device];
    return TK_OK;
}

static tk_status noalloc_fwd(tk_ctx* ctx, const tk_weight* W, const void* X, int x_dtype, int M, int ldx, float* Y,
                             int ldy, float beta, int products, cudaStream_t s) {
    const char* fn = "tk_linear_fwd_noalloc";
    if (!ctx) return fail(TK_ERR_INVALID, std::string(fn) + ": null context");
    if (!W || !W->data || W->rows <= 0 || W->cols <= 0) return fail(TK_ERR_INVALID, std::string(fn) + ": bad weight");
    if (W->qtype != TK_F16 && W->qtype != TK_F16X2)
        return fail(TK_ERR_UNSUPPORTED, std::string(fn) + ": only TK_F16 / TK_F16X2 weights (a quantized weight needs "
                                                          "a dequant buffer; use tk_linear_fwd)");
    if (W->row_bytes != (size_t)W->cols * 2 || W->cols % 8 || (reinterpret_cast<uintptr_t>(W->data) & 15))
        return fail(TK_ERR_INVALID, std::string(fn) + ": fp16 weight rows must be dense, 16-byte aligned, cols % 8 == 0");
    if (M < 0) return fail(TK_ERR_INVALID, std::string(fn) + ": negative M");
    if (M == 0) return TK_OK;
    if (!X || !Y) return fail(TK_ERR_INVALID, std::string(fn) + ": null activation or output");
    if (beta != 0.0f && beta != 1.0f) return fail(TK_ERR_INVALID, std::string(fn) + ": beta must be 0 or 1");
    if (x_dtype != TK_DT_F32 && x_dtype != TK_DT_F16 && x_dtype != TK_DT_BF16)
        return fail(TK_ERR_INVALID, std::string(fn) + ": activation dtype");
    const int N = W->rows, K = W->cols;
    if (ldx < K || ldy < N) return fail(TK_ERR_INVALID, std::string(fn) + ": leading dimension too small");
    if ((reinterpret_cast<uintptr_t>(Y) & 15) || ldy % 4)
        return fail(TK_ERR_INVALID, std::string(fn) + ": output must be 16-byte aligned, ld % 4 == 0");

    // product set: same meaning as tk_linear_fwd.  TK_QFUSED and TK_WREUSE
    // only concern quantized weights, which this entry point does not take.
    products &= ~(TK_QFUSED | TK_WREUSE);
    const bool wx2 = W->qtype == TK_F16X2;
    int mode = products == TK_X3_AUTO ? (wx2 ? TK_X3_HHL : (x_dtype == TK_DT_F32 ? TK_X3_REF : TK_X1)) : products;
    int planes = 1, nprod = 1, pa[3] = {0, 0, 0}, pb[3] = {0, 0, 0};
    if (mode == TK_X3_REF) { planes = 3; nprod = 3; pa[0] = 2; pa[1] = 1; pa[2] = 0; }
    else if (mode == TK_X3_HHL) {
        if (!wx2) return fail(TK_ERR_INVALID, std::string(fn) + ": TK_X3_HHL needs a TK_F16X2 weight");
        planes = 2; nprod = 3; pa[0] = 1; pb[0] = 0; pa[1] = 0; pb[1] = 1; pa[2] = 0; pb[2] = 0;
    } else if (mode == TK_X2) { planes = 2; nprod = 2; pa[0] = 1; pa[1] = 0; }
    else if (mode != TK_X1) return fail(TK_ERR_INVALID, std::string(fn) + ": unknown product set");

    // scratch: planes [planes][M][ld] fp16, then row exponents [M] int32
    const long ld = (K + 7) / 8 * 8;
    const size_t plane_bytes = align256((size_t)M * ld * 2 * planes);
    const size_t need = plane_bytes + align256((size_t)M * 4);
    if (need > kScratchBytes)
        return fail(TK_ERR_INVALID, std::string(fn) + ": M * K * parts needs " + std::to_string(need) +
                                        " bytes of scratch; the static limit is " + std::to_string(kScratchBytes) +
                                        " (use tk_linear_fwd, or split M)");
    void* base = nullptr;
    tk_status st = scratch_address(ctx->device, &base);
    if (st != TK_OK) return st;
    uint16_t* pl = static_cast<uint16_t*>(base);
    int* row_exp = reinterpret_cast<int*>(static_cast<uint8_t*>(base) + plane_bytes);

    st = launch_act_split(ctx, X, x_dtype, M, K, ldx, planes, true, pl, row_exp, s, ld);
    if (st != TK_OK) return st;
    GemmDesc g;
    for (int i = 0; i < planes; ++i) g.A[i] = pl + (size_t)i * M * ld;
    g.B[0] = static_cast<const uint16_t*>(W->data);
    g.B[1] = wx2 ? g.B[0] + (size_t)N * K : nullptr;
    g.lda = ld;
    g.ldb = K;
    g.b_mn = false;
    g.M = M;
    g.N = N;
    g.K = K;
    g.nprod = nprod;
    for (int i = 0; i < 3; ++i) { g.pa[i] = pa[i]; g.pb[i] = pb[i]; }
    g.D = Y;
    g.ldd = ldy;
    g.beta = beta != 0.0f;
    g.row_exp = row_exp;
    g.col_exp = wx2 ? W->scale_log2 : 0;
    g.seg_kb = nprod > 1 ? kSegKb : 0;   // the accumulation segments tk_linear_fwd uses
    // no split-K workspace (g.split_ws stays null): K is never split here
    return launch_gemm(ctx, g, s);
}

}  // namespace tk

extern "C" tk_status tk_linear_fwd_noalloc(tk_ctx* ctx, const tk_weight* W, const void* X, int x_dtype, int M,
                                           int ldx, float* Y, int ldy, float beta, int products, void* stream) {
    return tk::noalloc_fwd(ctx, W, X, x_dtype, M, ldx, Y, ldy, beta, products, static_cast<cudaStream_t>(stream));
}
