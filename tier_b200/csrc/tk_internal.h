// tk_internal.h -- host-side declarations shared by the tierk .cu files.
#pragma once
#include <atomic>
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>
#include <cuda_runtime.h>
#include "../../include/tierk.h"

// Optional per-kernel timing: CUDA events recorded on the launching stream
// around each kernel (enabled with tk_profile; read with tk_profile_read).
struct tk_prof {
    bool on = false;
    std::vector<cudaEvent_t> ev;   // pairs (start, stop)
    std::vector<int> kind;         // one per pair
    size_t used = 0;               // pairs recorded
};

struct tk_ctx {
    int device = 0;
    int num_sms = 0;
    void* ws = nullptr;          // workspace (device)
    size_t ws_bytes = 0;
    int* status = nullptr;       // device status word (tk::DEV_*)
    uint64_t launches = 0;       // kernels launched through this context
    int* flags = nullptr;        // split-K progress flags (device), flags_len ints
    int flags_len = 0;
    uint32_t epoch = 0;          // stamps split-K flags per launch (no reset needed)
    tk_prof prof;
    struct tk_comm_state* comm = nullptr;   // peer buffers for the reduce-scatter (tk_comm.cu)
    // fp16 expansion of a quantized weight left at the start of ws by the
    // last linear call (TK_WREUSE); any other workspace user clears it
    bool wexp_valid = false;
    const void* wexp_data = nullptr;
    int wexp_qtype = 0, wexp_rows = 0, wexp_cols = 0;
    size_t wexp_rb = 0;
    // IQ1/IQ2/IQ3 lattice tables registered by tk_set_iq_grids (device,
    // tkq::GRID_BYTES, layout in tk_qgrid.h); null until then
    int8_t* iq_tab = nullptr;
    // schedule of the last two-problem GEMM launch (tk_gemm.cu): per CTA pair
    // its units in order, [offsets (pairs + 1) | unit ids], on the device;
    // rebuilt when the key (shapes, tile counts, grid) changes
    int* sched = nullptr;
    size_t sched_cap = 0;            // ints
    std::vector<long> sched_key;
};

namespace tk {

// k-blocks (64 each) per fp32 accumulation segment for the split product sets.
// The error of the tensor-core fp32 accumulation grows with the segment
// length, not with K (measured relative error vs fp64 on B200, x3 REF / HHL:
// 8 -> 1.2e-6 / 1.7e-6, 16 -> 2.4e-6 / 3.5e-6, 32 -> 4.5e-6 / 7.1e-6), while
// each segment costs one fp32 read-modify-write of the tile.  16 keeps a 3x
// margin under the 1e-5 bound.
#ifndef TK_SEG_KB
#define TK_SEG_KB 16
#endif
constexpr int kSegKb = TK_SEG_KB;

// The dynamic shared-memory limit set by cudaFuncSetAttribute holds for the
// device current at the call only: record it per device (bit `device` of
// `done`, one mask per kernel instantiation), so that contexts on several
// devices of one process each get it before their first launch.
template <class K>
inline cudaError_t smem_attr_once(K* kern, int bytes, int device, std::atomic<uint64_t>& done) {
    const uint64_t bit = 1ull << (device & 63);
    if (done.load(std::memory_order_relaxed) & bit) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.fetch_or(bit);
    return e;
}

// Kernel families for tk_profile_read (TK_PROF_* in tierk.h).
enum ProfKind { PK_GEMM = 0, PK_DEQUANT = 1, PK_SPLIT = 2, PK_GEMV = 3, PK_LMHEAD = 4, PK_COMM = 5, PK_COUNT = 6 };
int prof_begin(tk_ctx* ctx, cudaStream_t s);
void prof_end(tk_ctx* ctx, cudaStream_t s, int slot, int kind);
struct ProfScope {
    tk_ctx* c; cudaStream_t s; int slot; int kind;
    ProfScope(tk_ctx* c_, cudaStream_t s_, int k) : c(c_), s(s_), slot(prof_begin(c_, s_)), kind(k) {}
    ~ProfScope() { prof_end(c, s, slot, kind); }
};

// Thread-local last-error text; returns `st` for chaining.
tk_status fail(tk_status st, const std::string& msg);
tk_status cuda_fail(cudaError_t e, const char* what);

// Workspace carving helper: 256-byte aligned sub-buffers of ctx->ws.
tk_status ws_ensure(tk_ctx* ctx, size_t bytes, cudaStream_t stream);
inline size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// ---- tk_dequant.cu ----
bool dequant_supported(int qtype);
int block_elems(int qtype);
int block_bytes(int qtype);
tk_status launch_dequant(tk_ctx* ctx, int qtype, const void* W, size_t rb, int r0, int nrows, int cols,
                         int out_dtype, void* out, cudaStream_t s);
// X[M, K] (x_dtype, row stride ldx) -> nplanes fp16 planes [M, K] (plane p at
// planes + p*M*K) of X * 2^e_m, e_m per row so that max|row|*2^e_m is in
// [2^14, 2^15); row_exp[m] = e_m.  scaled == false uses e_m = 0.
tk_status launch_act_split(tk_ctx* ctx, const void* X, int x_dtype, int M, int K, long ldx, int nplanes,
                           bool scaled, uint16_t* planes, int* row_exp, cudaStream_t s, long ldp = 0);
tk_status launch_split3_raw(tk_ctx* ctx, const float* x, size_t n, uint16_t* h, uint16_t* m, uint16_t* l,
                            cudaStream_t s);
tk_status weight_split_f32(tk_ctx* ctx, const float* W, int rows, int cols, uint16_t* planes, int* scale_log2,
                           cudaStream_t s);

// ---- tk_gemv4.cu (streaming decode GEMV, Q8_0 / Q4_K / Q5_K, M in {1, 2, 4}) ----
bool gemv_stream_ok(int qtype, size_t rb, int K, int M);
tk_status launch_gemv_stream(tk_ctx* ctx, int qtype, const void* W, size_t rb, int N, int K, const float* x, int ldx,
                             int M, float* y, int ldy, bool frozen, cudaStream_t s);
// ---- tk_gemv5.cu (decode GEMV on mma.sync tensor cores, Q8_0 / Q4_K / Q5_K, M <= 8) ----
bool gemv_mma_ok(int qtype, size_t rb, int K, int M);
tk_status launch_gemv_mma(tk_ctx* ctx, int qtype, const void* W, size_t rb, int N, int K, const float* x, int ldx,
                          int M, float* y, int ldy, bool frozen, cudaStream_t s);
bool gemv_imma_ok(int qtype, size_t rb, int K, int M);
bool gemv_imma_multi_ok(int qtype, size_t rb, int K, int M);
tk_status launch_gemv_imma_multi(tk_ctx* ctx, int qtype, int nseg, const void* const* W, const int* rows,
                                 float* const* y, const int* ldy, size_t rb, int K, const float* x, int ldx, int M,
                                 bool frozen, cudaStream_t s);
bool gemv_wide_ok(int qtype, size_t rb, int K, int M);
tk_status launch_gemv_wide(tk_ctx* ctx, int qtype, const void* W, size_t rb, int N, int K, const float* x, int ldx,
                           int M, float* y, int ldy, cudaStream_t s);
tk_status launch_gemv_imma(tk_ctx* ctx, int qtype, const void* W, size_t rb, int N, int K, const float* x, int ldx,
                           int M, float* y, int ldy, bool frozen, cudaStream_t s);

// ---- tk_gemv8.cu (decode GEMV, one token, Q8_0, dp4a with x in registers) ----
bool gemv_dp_ok(int t, size_t rb, int N, int K, int M, int num_sms);
tk_status launch_gemv_dp(tk_ctx* ctx, const void* W, size_t rb, int N, int K, const float* x, float* y, bool frozen,
                         cudaStream_t s);
// ---- tk_gemv.cu ----
bool gemv_supported(int qtype);
tk_status launch_gemv(tk_ctx* ctx, int qtype, const void* W, size_t rb, int N, int K, const float* x, int ldx,
                      int M, float* y, int ldy, cudaStream_t s, bool frozen = false);

// ---- tk_gemm.cu ----
// D[M, N] (fp32, row stride ldd) = sum_p A_{pa[p]}[M, K] . B_{pb[p]}^T, scaled
// per row by 2^-(row_exp[m] + col_exp) and added to D when beta != 0.
//   A planes: fp16 [M, K] K-major, row stride lda elements.
//   B planes: b_mn == false -> fp16 [N, K] K-major (row stride ldb);
//             b_mn == true  -> fp16 [K, N] N-major (row stride ldb).
struct GemmDesc {
    const uint16_t* A[3] = {nullptr, nullptr, nullptr};
    const uint16_t* B[2] = {nullptr, nullptr};
    long lda = 0, ldb = 0;
    bool b_mn = false;
    int M = 0, N = 0, K = 0;
    int nprod = 1;
    int pa[3] = {0, 0, 0}, pb[3] = {0, 0, 0};
    float* D = nullptr;
    long ldd = 0;
    int beta = 0;
    const int* row_exp = nullptr;
    int col_exp = 0;
    int seg_kb = 0;        // k-blocks (of 64) per fp32 accumulation segment; 0 = whole K
    const float* row_alpha = nullptr;   // with beta = 1: D = row_alpha[row] * D + A.B
    const struct RsDesc* rs = nullptr;  // reduce-scatter the result over peer memory (tk_comm.cu)
    float* split_ws = nullptr;   // fp32 [M, split_ld] slab; enables split-K when given
    long split_ld = 0;
};
// Reduce-scatter target of a GEMM (rows split over `world` owners, `rpo` rows
// each): the last segment of row r goes to dst[r / rpo] + (r % rpo) * ldd;
// the launch's last CTA then stores `epoch` into done[o] of every owner.
constexpr int TK_MAX_RANKS = 8;
struct RsDesc {
    float* dst[TK_MAX_RANKS] = {};
    int* done[TK_MAX_RANKS] = {};
    int* counter = nullptr;
    int world = 0, rpo = 0, epoch = 0;
};

// ---- tk_quant.cu: quantizers byte-exact with the reference's CPU ones ----
tk_status launch_quantize(tk_ctx* ctx, int qtype, const float* x, long ldx, int rows, int cols, uint8_t* out,
                          size_t rb, cudaStream_t s);
tk_status launch_bf16_to_f32(tk_ctx* ctx, const uint16_t* src, long lds, int rows, int cols, float* dst,
                             cudaStream_t s);

// ---- tk_comm.cu: peer buffers (CUDA IPC) and the reduce-scatter around a GEMM ----
void comm_destroy(tk_ctx* ctx);
// Before the GEMM: wait (bounded) until every owner has consumed the receive
// buffer this launch will overwrite; fills `rs` for the GEMM and returns the epoch.
tk_status rs_begin(tk_ctx* ctx, int M, int K, RsDesc& rs, cudaStream_t s);
// After the GEMM: wait for every rank's done flag, sum the slots in rank
// order into out[rpo, ldo], then acknowledge to every rank.
tk_status rs_finish(tk_ctx* ctx, const RsDesc& rs, int K, float* out, long ldo, cudaStream_t s);

// K splits launch_gemm would use for g given a split workspace (1 or 2).
int gemm_splits(const tk_ctx* ctx, const GemmDesc& g);
tk_status launch_gemm(tk_ctx* ctx, const GemmDesc& g, cudaStream_t s);
// Two GEMMs in one persistent launch, their tiles interleaved.  Both need CTA
// pairs (M > 128) and no split-K; only g1 may carry a reduce-scatter.  Each
// result equals its own launch_gemm without split-K bit for bit.
bool gemm_pair_ok(const GemmDesc& g0, const GemmDesc& g1);
tk_status launch_gemm_pair(tk_ctx* ctx, const GemmDesc& g0, const GemmDesc& g1, cudaStream_t s);

// Fused-dequant GEMM (tk_gemm_q.cu): B is the raw quantized weight W[w_rows,
// row_bytes]; dx == false: D[M, N] = A . W^T with N = w_rows, K = cols of W;
// dx == true: D[M, N] = A . W with K = w_rows, N = cols of W.  CTA pairs only
// (M > 128).  Every product multiplies an A plane by the same dequantized W.
struct GemmQDesc {
    const uint16_t* A[3] = {nullptr, nullptr, nullptr};
    long lda = 0;
    int nprod = 1;
    int pa[3] = {0, 0, 0};
    int qtype = 0;
    const void* W = nullptr;
    size_t w_row_bytes = 0;
    int w_rows = 0;
    bool dx = false;
    int M = 0, N = 0, K = 0;
    float* D = nullptr;
    long ldd = 0;
    int beta = 0;
    const int* row_exp = nullptr;
    int seg_kb = 0;
};
bool gemm_q_supported(int qtype);
tk_status launch_gemm_q(tk_ctx* ctx, const GemmQDesc& g, cudaStream_t s);

// LM-head epilogue variants (tk_gemm.cu)
struct LseDesc {               // pass 1: per (row, 256-column tile) partial stats
    float* pmax; int32_t* parg; double* psum; float* ptgt;   // [T_rows, ntiles]
    const int32_t* labels; int v0; float cap; int ld_part;
    float* zout = nullptr; long ldz = 0;   // optional: the softcapped logits [T_rows, ldz]
};
struct DlogitDesc {            // pass 2: dlogit planes
    const double* rmax; const double* rsum; const int32_t* labels; const uint8_t* mask;
    int T; int v0; int n_loss; float cap; int dl_exp; int nplanes;
    uint16_t* planes; long plane_stride; int ld;            // planes [nplanes][T, ld]
};
tk_status launch_gemm_lse(tk_ctx* ctx, const GemmDesc& g, const LseDesc& e, cudaStream_t s);
tk_status launch_gemm_dlogit(tk_ctx* ctx, const GemmDesc& g, const DlogitDesc& e, cudaStream_t s);

// ---- tk_lmhead.cu ----
tk_status launch_lse_merge(tk_ctx* ctx, const float* pmax, const int32_t* parg, const double* psum,
                           const float* ptgt, int ld_part, int ntiles, int n_pred, int vc, int v0,
                           const int32_t* labels, const uint8_t* mask, double* rmax, double* rsum,
                           int32_t* amax, float* tgt, cudaStream_t s, float* alpha = nullptr);
// Single-pass head: P[t, v] = exp(l - rmax[t]) * (1 - (l/cap)^2) as fp16 hi/lo planes.
tk_status launch_lm_prob(tk_ctx* ctx, const float* Z, long ldz, int rows, int vc, const double* rmax,
                         const uint8_t* mask, float cap, uint16_t* planes, long plane_stride, int ld, cudaStream_t s);
// dX[t] = dX[t] / (n_loss * rsum[t]) - g_t * W[label - v0] / n_loss (label in this shard), 0 for rows
// without loss; g_t = 1 - (tgt/cap)^2.
tk_status launch_lm_finish(tk_ctx* ctx, const uint16_t* W, int v0, int V_shard, int H, int T, const int32_t* labels,
                           const uint8_t* mask, int n_loss, float cap, const double* rsum, const float* tgt, float* dX,
                           cudaStream_t s);
tk_status launch_lm_loss(tk_ctx* ctx, int T, const int32_t* labels, const uint8_t* mask, const double* rmax,
                         const double* rsum, const int32_t* amax, const float* tgt, double* loss, int32_t* hits,
                         cudaStream_t s);
tk_status launch_lm_rescale(tk_ctx* ctx, int n, double* rmax_l, double* rsum_l, const double* rmax_g,
                            cudaStream_t s, float* dX = nullptr, int H = 0);

}  // namespace tk
