// Host check of integration/tier_bridge.h: the engine's globals and the
// libtierk calls are stand-ins, so the routing decisions and the argument
// order of each call can be checked without a GPU or a model.  Built and run
// by tests/test_integration_build.py; prints one line per check.
#include <cstdio>
#include <map>
#include <set>

typedef void* cudaStream_t;
enum { cudaSuccess = 0 };
static int cudaGetDevice(int* d) { *d = 0; return cudaSuccess; }

#include "tierk.h"

// ---- stand-ins for the engine state the bridge reads (tier/tier.cpp:97-102) ----
struct RowSplit { const unsigned short* host; int rows, R, K; };
static std::map<const float*, RowSplit> g_split;
static std::set<const void*> g_bf16w, g_fp16w;
static bool g_bf3 = false, g_use_fp16_x3 = false;

// ---- recording stubs of the library ----
static int calls = 0, fail_next = 0;
static tk_weight last_w;
static const void *last_in, *last_out;
static int last_dtype, last_M, last_ldin, last_ldout, last_products, last_qtype, last_N, last_K;
static float last_beta;
static size_t last_rb;
static cudaStream_t last_stream;
static int ret() { ++calls; if (fail_next) { fail_next = 0; return TK_ERR_INVALID; } return TK_OK; }
extern "C" {
tk_status tk_init(int, tk_ctx** out) { *out = reinterpret_cast<tk_ctx*>(0x1000); return TK_OK; }
const char* tk_last_error_string(void) { return "stub failure"; }
tk_status tk_linear_fwd(tk_ctx*, const tk_weight* W, const void* X, int x_dtype, int M, int ldx, float* Y, int ldy,
                        float beta, int products, void* stream) {
    last_w = *W; last_in = X; last_out = Y; last_dtype = x_dtype; last_M = M; last_ldin = ldx; last_ldout = ldy;
    last_beta = beta; last_products = products; last_stream = stream; return (tk_status)ret();
}
tk_status tk_linear_dx(tk_ctx*, const tk_weight* W, const void* dY, int dy_dtype, int M, int lddy, float* dX,
                       int lddx, float beta, int products, void* stream) {
    last_w = *W; last_in = dY; last_out = dX; last_dtype = dy_dtype; last_M = M; last_ldin = lddy; last_ldout = lddx;
    last_beta = beta; last_products = products; last_stream = stream; return (tk_status)ret();
}
tk_status tk_gemv(tk_ctx*, int qtype, const void* W, size_t rb, int N, int K, const float* x, int ldx, int M, float* y,
                  int ldy, void* stream) {
    last_qtype = qtype; last_w.data = W; last_rb = rb; last_N = N; last_K = K; last_in = x; last_ldin = ldx; last_M = M;
    last_out = y; last_ldout = ldy; last_stream = stream; return (tk_status)ret();
}
static int last_v0, last_vs, last_H, last_T, last_chunk, last_nloss;
static float last_cap;
static const void *last_lab, *last_mask, *last_state;
tk_status tk_lmhead_stats(tk_ctx*, const uint16_t* W, int v0, int V_shard, int H, const float* X, int T,
                          const int32_t* labels, const uint8_t* mask, float softcap, int chunk, int products,
                          double* rmax, double*, int32_t*, float*, void* stream) {
    last_w.data = W; last_v0 = v0; last_vs = V_shard; last_H = H; last_in = X; last_T = T; last_lab = labels;
    last_mask = mask; last_cap = softcap; last_chunk = chunk; last_products = products; last_state = rmax;
    last_stream = stream; return (tk_status)ret();
}
tk_status tk_lmhead_grad(tk_ctx*, const uint16_t* W, int v0, int V_shard, int H, const float* X, int T,
                         const int32_t* labels, const uint8_t* mask, int n_loss, float softcap, int chunk, int products,
                         const double* rmax, const double*, float* dX, void* stream) {
    last_w.data = W; last_v0 = v0; last_vs = V_shard; last_H = H; last_in = X; last_T = T; last_lab = labels;
    last_mask = mask; last_nloss = n_loss; last_cap = softcap; last_chunk = chunk; last_products = products;
    last_state = rmax; last_out = dX; last_stream = stream; return (tk_status)ret();
}
}

#include "tier_bridge.h"

struct ChatMat { void* dev; int qt; int rows, cols; size_t rb; };

#define CHECK(name, cond) printf("%s %d\n", name, (cond) ? 1 : 0)

int main() {
    static float W[64], x[64], y[64];
    const int M = 4, K = 32, N = 16;
    // an fp32 weight: the reference path keeps it
    CHECK("fp32_not_routed", !tk_bridge_fwd(x, W, y, M, K, N) && calls == 0);
    // fp16 storage without the x3 mode: still the reference path
    g_fp16w.insert(W); g_bf16w.insert(W);
    CHECK("fp16_without_x3_not_routed", !tk_bridge_fwd(x, W, y, M, K, N) && calls == 0);
    g_bf3 = g_use_fp16_x3 = true;
    // forward: out[M,N] = x[M,K] . W^T on fp16 W[N,K], x fp32 with ld K, out ld N, beta 0, products X3_REF
    bool ok = tk_bridge_fwd(x, W, y, M, K, N);
    CHECK("fwd_routed", ok && calls == 1);
    CHECK("fwd_args", last_w.qtype == TK_F16 && last_w.rows == N && last_w.cols == K && last_w.row_bytes == (size_t)K * 2 &&
                          last_w.data == W && last_in == x && last_out == y && last_dtype == TK_DT_F32 && last_M == M &&
                          last_ldin == K && last_ldout == N && last_beta == 0.0f && last_products == TK_X3_REF &&
                          last_stream == nullptr);
    // dX[M,K] = dY[M,N] . W: dY ld N, dX ld K; linear_dx beta 0, linear_dx_acc beta 1
    ok = tk_bridge_dx(x, W, y, M, K, N, 0.0f);
    CHECK("dx_args", ok && last_ldin == N && last_ldout == K && last_beta == 0.0f && last_w.rows == N &&
                         last_w.cols == K && last_in == x && last_out == y);
    ok = tk_bridge_dx(x, W, y, M, K, N, 1.0f);
    CHECK("dx_acc_beta", ok && last_beta == 1.0f);
    // a weight whose rows are shared with the CPU stays on the reference path
    g_split[W] = RowSplit{nullptr, N, N / 2, K};
    const int before = calls;
    CHECK("row_split_not_routed", !tk_bridge_fwd(x, W, y, M, K, N) && calls == before);
    g_split.clear();
    // a failed library call falls back (returns false)
    fail_next = 1;
    CHECK("failure_falls_back", !tk_bridge_fwd(x, W, y, M, K, N));
    // chat: quantized weight, 1..16 tokens -> tk_gemv with W frozen when resident
    ChatMat m{W, TK_Q4_K, N, 256, 144};
    ok = tk_bridge_chat(m, W, x, y, 3, (cudaStream_t)0x77);
    CHECK("chat_gemv", ok && last_qtype == (TK_Q4_K | TK_WFROZEN) && last_rb == 144 && last_N == N && last_K == 256 &&
                           last_ldin == 256 && last_M == 3 && last_ldout == N && last_stream == (cudaStream_t)0x77);
    ChatMat streamed{nullptr, TK_Q8_0, N, 256, 272};
    ok = tk_bridge_chat(streamed, W, x, y, 1, nullptr);
    CHECK("chat_streamed_not_frozen", ok && last_qtype == TK_Q8_0);
    // above 16 tokens: tk_linear_fwd on the block weight, x3 auto
    ok = tk_bridge_chat(m, W, x, y, 40, (cudaStream_t)0x77);
    CHECK("chat_linear", ok && last_w.qtype == TK_Q4_K && last_w.rows == N && last_w.cols == 256 &&
                             last_w.row_bytes == 144 && last_M == 40 && last_ldin == 256 && last_ldout == N &&
                             last_products == TK_X3_AUTO);
    // not quantized: the reference's chat branches
    ChatMat dense{W, 0, N, 256, 0};
    CHECK("chat_dense_not_routed", !tk_bridge_chat(dense, W, x, y, 1, nullptr));
    // LM head: chunk size rounded to 256 rows; a 256-multiple chunk goes to
    // libtierk on the reference's running state, any other stays on the reference path
    CHECK("lm_chunk_rounding", tk_bridge_lm_chunk(60032) == 59904 && tk_bridge_lm_chunk(1024) == 1024 &&
                                   tk_bridge_lm_chunk(384) == 384);
    static double rmax[8], rsum[8];
    static int amax[8];
    static float tgt[8];
    static int32_t tok[8];
    static unsigned char msk[8];
    ok = tk_bridge_lm_stats(W, 2048, 1024, 64, x, 8, tok, msk, 30.0f, rmax, rsum, amax, tgt);
    CHECK("lm_stats_args", ok && last_w.data == W && last_v0 == 2048 && last_vs == 1024 && last_chunk == 1024 &&
                               last_H == 64 && last_in == x && last_T == 8 && last_lab == tok && last_mask == msk &&
                               last_cap == 30.0f && last_products == TK_X3_REF && last_state == rmax &&
                               last_stream == nullptr);
    ok = tk_bridge_lm_grad(W, 0, 512, 64, x, 8, tok, msk, 7, 0.0f, rmax, rsum, y);
    CHECK("lm_grad_args", ok && last_vs == 512 && last_chunk == 512 && last_nloss == 7 && last_out == y &&
                              last_state == rmax && last_products == TK_X3_REF);
    CHECK("routed_counts", g_tkb_calls[TKB_FWD] >= 1 && g_tkb_calls[TKB_DX] == 2 && g_tkb_calls[TKB_CHAT] == 3 &&
                               g_tkb_calls[TKB_LM1] == 1 && g_tkb_calls[TKB_LM2] == 1);
    const int c0 = calls;
    CHECK("lm_ragged_chunk_not_routed", !tk_bridge_lm_stats(W, 0, 1000, 64, x, 8, tok, msk, 0.0f, rmax, rsum, amax, tgt) &&
                                            !tk_bridge_lm_grad(W, 0, 1000, 64, x, 8, tok, msk, 7, 0.0f, rmax, rsum, y) &&
                                            calls == c0);
    return 0;
}
