// tier_bridge.h -- the glue a maintainer adds to tierlm's engine (tier/tier.cpp)
// so that its frozen-weight linear path runs on libtierk.so.  It is included
// once, just before `linear` (tier/tier.cpp:1202).  Everything it names from
// the engine is declared before that point; the chat part is a template, so
// the ChatMat fields resolve where chat_lin (tier/tier.cpp:2351) uses it.
//
// Routed to libtierk:
//   * linear / linear_dx / linear_dx_acc (tier/tier.cpp:1202-1238) for fp16
//     weights in the fp16-x3 mode (g_fp16w, g_bf3, g_use_fp16_x3).  The
//     reference runs fp3gemm's three cuBLASLt GEMMs (tier/tier.cpp:922-943);
//     here that is one tk_linear_fwd / tk_linear_dx with TK_X3_REF, i.e. the
//     same products W.xl + W.xm + W.xh in one tcgen05 GEMM.
//   * the LM head's two chunk loops (tier/tier.cpp:3209-3266), fp16 head
//     chunks whose row count is a multiple of 256: pass 1 (fp16 -> fp32
//     expansion, fp32 logits GEMM, softcap, lse_chunk_kernel) becomes one
//     tk_lmhead_stats per chunk, pass 2 (the same logits again, dlogit_kernel,
//     linear_dx_acc) one tk_lmhead_grad.  Both update the reference's own
//     running state (double max and sum, int argmax, float target logit), so
//     a chunk the bridge declines runs the reference's code on the same
//     state.  The chunk size is rounded down to a multiple of 256.
//   * chat_lin's quantized branch (tier/tier.cpp:2356-2360): gemv_q for one
//     token and dq_launch + chat_linear_ld slabs beyond it become tk_gemv for
//     up to 16 tokens and tk_linear_fwd above that.  Resident weights
//     (m.dev) are frozen, so they take TK_WFROZEN.  Above 16 tokens the
//     tensor-core path rounds the expanded weight to fp16 (about 2e-4
//     relative), where the reference's chat path expands it to fp32; the
//     GEMV agrees with fp64 to ~1e-7.
// Everything else (row splits shared with the CPU, bf16 and fp32 weights, the
// fallbacks) keeps the reference's own path: each function returns false and
// the caller continues as before.  A failed libtierk call also returns false
// after printing the library's message, so the reference path stays the
// safety net.
#pragma once
#include <cstdio>
#include <cstdlib>

#include "tierk.h"

static tk_ctx* g_tk = nullptr;

// Calls the bridge routed to libtierk, by kind; printed to stderr at exit when
// TIERK_BRIDGE_STATS is set, so a run can show which of its linears took the
// library path.
enum { TKB_FWD, TKB_DX, TKB_CHAT, TKB_LM1, TKB_LM2, TKB_KINDS };
static long g_tkb_calls[TKB_KINDS];
static void tk_bridge_report() {
    fprintf(stderr, "libtierk bridge: fwd %ld dx %ld chat %ld lm_stats %ld lm_grad %ld\n", g_tkb_calls[TKB_FWD],
            g_tkb_calls[TKB_DX], g_tkb_calls[TKB_CHAT], g_tkb_calls[TKB_LM1], g_tkb_calls[TKB_LM2]);
}

// One context per process, on the device current at the first call (the
// engine uses one GPU per process).
static bool tk_bridge_ready() {
    static int state = -1;
    if (state < 0) {
        int dev = 0;
        state = (cudaGetDevice(&dev) == cudaSuccess && tk_init(dev, &g_tk) == TK_OK) ? 1 : 0;
        if (!state) fprintf(stderr, "libtierk: %s (reference path kept)\n", tk_last_error_string());
        if (getenv("TIERK_BRIDGE_STATS")) atexit(tk_bridge_report);
    }
    return state == 1;
}

static bool tk_bridge_ok(tk_status st, int kind) {
    if (st == TK_OK) { ++g_tkb_calls[kind]; return true; }
    fprintf(stderr, "libtierk: %s (reference path used)\n", tk_last_error_string());
    return false;
}

// The fp16-x3 weights of the training path: W[N, K] fp16 on the device.
static bool tk_bridge_fp16_x3(const float* W) {
    return !g_split.count(W) && g_fp16w.count(W) && g_bf16w.count(W) && g_bf3 && g_use_fp16_x3;
}

// out[M, N] = x[M, K] . W^T (linear, beta 0).
static bool tk_bridge_fwd(const float* x, const float* W, float* out, int M, int K, int N) {
    if (!tk_bridge_fp16_x3(W) || !tk_bridge_ready()) return false;
    tk_weight w{TK_F16, N, K, 0, (size_t)K * 2, W};
    return tk_bridge_ok(tk_linear_fwd(g_tk, &w, x, TK_DT_F32, M, K, out, N, 0.0f, TK_X3_REF, nullptr), TKB_FWD);
}

// dX[M, K] (=|+=) dY[M, N] . W (linear_dx with beta 0, linear_dx_acc with beta 1).
static bool tk_bridge_dx(const float* dY, const float* W, float* dX, int M, int K, int N, float beta) {
    if (!tk_bridge_fp16_x3(W) || !tk_bridge_ready()) return false;
    tk_weight w{TK_F16, N, K, 0, (size_t)K * 2, W};
    return tk_bridge_ok(tk_linear_dx(g_tk, &w, dY, TK_DT_F32, M, N, dX, K, beta, TK_X3_REF, nullptr), TKB_DX);
}

// chat_lin, quantized weight m (block type m.qt, m.rows x m.cols, m.rb bytes
// per row) at W: y[M, m.rows] = x[M, m.cols] . W^T on the chat stream.
template <class ChatMatT>
static bool tk_bridge_chat(const ChatMatT& m, const void* W, const float* x, float* y, int M, cudaStream_t s) {
    if (!m.qt || !tk_bridge_ready()) return false;
    if (M <= 16) {
        const int qt = m.qt | (m.dev ? TK_WFROZEN : 0);
        return tk_bridge_ok(tk_gemv(g_tk, qt, W, m.rb, m.rows, m.cols, x, m.cols, M, y, m.rows, s), TKB_CHAT);
    }
    tk_weight w{m.qt, m.rows, m.cols, 0, m.rb, W};
    return tk_bridge_ok(tk_linear_fwd(g_tk, &w, x, TK_DT_F32, M, m.cols, y, m.rows, 0.0f, TK_X3_AUTO, s), TKB_CHAT);
}

// LM head chunk size: the reference's lm_chunk, rounded down to a multiple of
// 256 rows (the tile of libtierk's LM-head kernels) when it is at least 512.
static int tk_bridge_lm_chunk(int chunk) { return chunk >= 512 ? chunk / 256 * 256 : chunk; }

// Pass 1 over one chunk: Wc = the chunk's fp16 rows [vc, H] on the device,
// v0 = its first vocabulary row; X = the final hidden states [T, H] fp32.
static bool tk_bridge_lm_stats(const void* Wc, int v0, int vc, int H, const float* X, int T, const int32_t* tokens,
                               const unsigned char* mask, float softcap, double* rmax, double* rsum, int* amax,
                               float* tgt) {
    if (vc % 256 || H % 8 || !tk_bridge_ready()) return false;
    return tk_bridge_ok(tk_lmhead_stats(g_tk, static_cast<const uint16_t*>(Wc), v0, vc, H, X, T, tokens, mask, softcap,
                                        vc, TK_X3_REF, rmax, rsum, amax, tgt, nullptr),
                        TKB_LM1);
}

// Pass 2 over one chunk: dX[T, H] += dlogit . Wc (linear_dx_acc of the reference).
static bool tk_bridge_lm_grad(const void* Wc, int v0, int vc, int H, const float* X, int T, const int32_t* tokens,
                              const unsigned char* mask, int n_loss, float softcap, const double* rmax,
                              const double* rsum, float* dX) {
    if (vc % 256 || H % 8 || !tk_bridge_ready()) return false;
    return tk_bridge_ok(tk_lmhead_grad(g_tk, static_cast<const uint16_t*>(Wc), v0, vc, H, X, T, tokens, mask, n_loss,
                                       softcap, vc, TK_X3_REF, rmax, rsum, dX, nullptr),
                        TKB_LM2);
}
