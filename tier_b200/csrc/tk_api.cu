// tk_api.cu -- the extern "C" entry points of libtierk.so (include/tierk.h):
// argument validation, workspace management, and the composition of the
// kernels into the reference's operations.
#include <cmath>
#include <cstring>
#include <string>
#include <vector>
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

static thread_local std::string g_last_error;

tk_status fail(tk_status st, const std::string& msg) {
    g_last_error = msg;
    return st;
}
tk_status cuda_fail(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return TK_OK;
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return e == cudaErrorMemoryAllocation ? TK_ERR_NOMEM : TK_ERR_CUDA;
}

tk_status ws_ensure(tk_ctx* ctx, size_t bytes, cudaStream_t stream) {
    ctx->wexp_valid = false;     // the caller is about to carve the workspace
    if (bytes <= ctx->ws_bytes) return TK_OK;
    // Work queued on any stream may still use the old buffer.
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "workspace growth sync");
    (void)stream;
    if (ctx->ws) cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
    size_t want = align256(bytes + (bytes >> 3));
    e = cudaMalloc(&ctx->ws, want);
    if (e != cudaSuccess) {
        cudaGetLastError();
        e = cudaMalloc(&ctx->ws, align256(bytes));
        if (e != cudaSuccess) return cuda_fail(e, "workspace allocation");
        want = align256(bytes);
    }
    ctx->ws_bytes = want;
    return TK_OK;
}

constexpr size_t kProfPairs = 8192;

int prof_begin(tk_ctx* ctx, cudaStream_t s) {
    tk_prof& p = ctx->prof;
    if (!p.on || p.used >= kProfPairs) return -1;
    if (p.ev.size() < 2 * (p.used + 1)) {
        cudaEvent_t a, b;
        if (cudaEventCreate(&a) != cudaSuccess) return -1;
        if (cudaEventCreate(&b) != cudaSuccess) { cudaEventDestroy(a); return -1; }
        p.ev.push_back(a);
        p.ev.push_back(b);
    }
    const int slot = (int)p.used++;
    cudaEventRecord(p.ev[2 * slot], s);
    return slot;
}

void prof_end(tk_ctx* ctx, cudaStream_t s, int slot, int kind) {
    if (slot < 0) return;
    tk_prof& p = ctx->prof;
    cudaEventRecord(p.ev[2 * slot + 1], s);
    if (p.kind.size() <= (size_t)slot) p.kind.resize(slot + 1);
    p.kind[slot] = kind;
}

struct Carve {
    char* p;
    size_t used = 0;
    explicit Carve(void* base) : p(static_cast<char*>(base)) {}
    template <class T>
    T* take(size_t n) {
        T* r = reinterpret_cast<T*>(p + used);
        used += align256(n * sizeof(T));
        return r;
    }
};

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Planes / products for one linear call.
struct Plan {
    int x_planes = 1;
    int nprod = 1;
    int pa[3] = {0, 0, 0}, pb[3] = {0, 0, 0};
    bool w_two = false;
};

static tk_status plan_products(const tk_weight* W, int x_dtype, int products, Plan& pl) {
    const bool wx2 = W->qtype == TK_F16X2;
    int mode = products;
    if (mode == TK_X3_AUTO) mode = wx2 ? TK_X3_HHL : (x_dtype == TK_DT_F32 ? TK_X3_REF : TK_X1);
    switch (mode) {
        case TK_X3_REF:   // W.xl + W.xm + W.xh (low parts first)
            pl.x_planes = 3; pl.nprod = 3;
            pl.pa[0] = 2; pl.pa[1] = 1; pl.pa[2] = 0;
            break;
        case TK_X3_HHL:   // Xl.Wh + Xh.Wl + Xh.Wh
            if (!wx2) return fail(TK_ERR_INVALID, "TK_X3_HHL needs a TK_F16X2 weight");
            pl.x_planes = 2; pl.nprod = 3; pl.w_two = true;
            pl.pa[0] = 1; pl.pb[0] = 0;
            pl.pa[1] = 0; pl.pb[1] = 1;
            pl.pa[2] = 0; pl.pb[2] = 0;
            break;
        case TK_X2:
            pl.x_planes = 2; pl.nprod = 2;
            pl.pa[0] = 1; pl.pa[1] = 0;
            break;
        case TK_X1:
            pl.x_planes = 1; pl.nprod = 1;
            break;
        default: return fail(TK_ERR_INVALID, "unknown product set " + std::to_string(products));
    }
    return TK_OK;
}

static tk_status check_weight(const tk_weight* W, const char* fn) {
    if (!W || !W->data) return fail(TK_ERR_INVALID, std::string(fn) + ": null weight");
    if (W->rows <= 0 || W->cols <= 0) return fail(TK_ERR_INVALID, std::string(fn) + ": empty weight");
    if (!aligned16(W->data)) return fail(TK_ERR_INVALID, std::string(fn) + ": weight must be 16-byte aligned");
    if (W->qtype == TK_F16X2 || W->qtype == TK_F16) {
        if (W->row_bytes != (size_t)W->cols * 2 || W->cols % 8)
            return fail(TK_ERR_INVALID, std::string(fn) + ": fp16 weight rows must be dense with cols % 8 == 0");
        return TK_OK;
    }
    if (!dequant_supported(W->qtype) || W->qtype == TK_F32 || W->qtype == TK_BF16)
        return fail(TK_ERR_UNSUPPORTED, std::string(fn) + ": weight type " + std::to_string(W->qtype) +
                                            " not supported on the tensor-core path");
    if (W->cols % block_elems(W->qtype) || W->row_bytes != (size_t)(W->cols / block_elems(W->qtype)) * block_bytes(W->qtype))
        return fail(TK_ERR_INVALID, std::string(fn) + ": row_bytes does not match the block layout");
    if (W->cols % 8) return fail(TK_ERR_INVALID, std::string(fn) + ": cols must be a multiple of 8");
    return TK_OK;
}

// Shared body of fwd (dx == false) and dX (dx == true).
static tk_status linear(tk_ctx* ctx, const tk_weight* W, const void* A, int a_dtype, int M, int lda, float* D,
                        int ldd, float beta, int products, cudaStream_t s, bool dx, bool rs_scatter = false) {
    const char* fn = dx ? "tk_linear_dx" : "tk_linear_fwd";
    if (!ctx) return fail(TK_ERR_INVALID, std::string(fn) + ": null context");
    tk_status st = check_weight(W, fn);
    if (st != TK_OK) return st;
    if (M < 0) return fail(TK_ERR_INVALID, std::string(fn) + ": negative M");
    if (M == 0) return TK_OK;
    if (!A || !D) return fail(TK_ERR_INVALID, std::string(fn) + ": null activation or output");
    if (beta != 0.0f && beta != 1.0f) return fail(TK_ERR_INVALID, std::string(fn) + ": beta must be 0 or 1");
    const int N = W->rows, K = W->cols;
    const int a_cols = dx ? N : K, d_cols = dx ? K : N;
    if (lda < a_cols || ldd < d_cols) return fail(TK_ERR_INVALID, std::string(fn) + ": leading dimension too small");
    if (a_dtype != TK_DT_F32 && a_dtype != TK_DT_F16 && a_dtype != TK_DT_BF16)
        return fail(TK_ERR_INVALID, std::string(fn) + ": activation dtype");
    if (!aligned16(D) || ldd % 4) return fail(TK_ERR_INVALID, std::string(fn) + ": output must be 16-byte aligned, ld % 4 == 0");
    const bool want_fused = (products & TK_QFUSED) != 0 && !rs_scatter;
    const bool want_reuse = (products & TK_WREUSE) != 0;
    products &= ~(TK_QFUSED | TK_WREUSE);
    Plan pl;
    st = plan_products(W, a_dtype, products, pl);
    if (st != TK_OK) return st;

    const bool quant = W->qtype != TK_F16 && W->qtype != TK_F16X2;
    // Quantized weights go through the fused-dequant GEMM (no fp16 copy of W)
    // when the shape allows it: CTA-pair tiles (M > 128), whole 256-column
    // slabs, 16-byte-aligned rows.
    // On request (TK_QFUSED) the weight is decoded inside the GEMM; the
    // default expands it to fp16 once and runs the plain GEMM (the fused decode
    // repeats for every 256-row tile of M).
    const bool fused = want_fused && quant && gemm_q_supported(W->qtype) && M > 128 && K % 256 == 0 &&
                       W->row_bytes % 16 == 0 && !pl.w_two;
    // split planes use a row stride rounded up to 8 elements (16 bytes, the TMA
    // stride rule); the GEMM's K extent stays a_cols, so the pad is never read.
    const long a_ld = (a_cols + 7) / 8 * 8;
    const size_t plane_elems = (size_t)M * a_ld;
    // split-K slab (fp32, [M, d_cols rounded to 4]) when the GEMM splits K
    GemmDesc probe;
    probe.M = M;
    probe.N = d_cols;
    probe.K = a_cols;
    probe.b_mn = dx;
    const long s_ld = (d_cols + 3) / 4 * 4;
    const bool split = !fused && !rs_scatter && gemm_splits(ctx, probe) == 2;
    // reduce-scatter with several accumulation segments: the earlier segments
    // go to a local fp32 [M, d_cols] scratch, only the last to the owners
    const bool rs_scratch = rs_scatter && pl.nprod > 1;
    const size_t need = align256(plane_elems * 2 * pl.x_planes) + align256((size_t)M * 4) +
                        (quant && !fused ? align256((size_t)N * K * 2) : 0) +
                        (split ? align256((size_t)M * s_ld * 4) : 0) +
                        (rs_scratch ? align256((size_t)M * d_cols * 4) : 0);
    // The fp16 expansion of a quantized W sits at the start of the workspace,
    // so a later call on the same weight (TK_WREUSE) finds it there.
    const bool expand = quant && !fused;
    const bool reuse = expand && want_reuse && ctx->wexp_valid && ctx->wexp_data == W->data &&
                       ctx->wexp_qtype == W->qtype && ctx->wexp_rows == N && ctx->wexp_cols == K &&
                       ctx->wexp_rb == W->row_bytes;
    const void* ws_before = ctx->ws;
    st = ws_ensure(ctx, need, s);
    if (st != TK_OK) return st;
    Carve cv(ctx->ws);
    uint16_t* wf = expand ? cv.take<uint16_t>((size_t)N * K) : nullptr;
    // plane p of the split activation at pbase + p * M * a_cols (16-byte aligned: a_cols % 8 == 0)
    uint16_t* pbase = cv.take<uint16_t>(plane_elems * pl.x_planes);
    int* row_exp = cv.take<int>(M);
    if (fused) {
        st = launch_act_split(ctx, A, a_dtype, M, a_cols, lda, pl.x_planes, true, pbase, row_exp, s, a_ld);
        if (st != TK_OK) return st;
        GemmQDesc q;
        for (int i = 0; i < pl.x_planes; ++i) q.A[i] = pbase + (size_t)i * plane_elems;
        q.lda = a_ld;
        q.nprod = pl.nprod;
        for (int i = 0; i < 3; ++i) q.pa[i] = pl.pa[i];
        q.qtype = W->qtype;
        q.W = W->data;
        q.w_row_bytes = W->row_bytes;
        q.w_rows = N;
        q.dx = dx;
        q.M = M;
        q.N = d_cols;
        q.K = a_cols;
        q.D = D;
        q.ldd = ldd;
        q.beta = beta != 0.0f;
        q.row_exp = row_exp;
        q.seg_kb = pl.nprod > 1 ? kSegKb : 0;
        return launch_gemm_q(ctx, q, s);
    }
    const uint16_t* wplanes[2] = {nullptr, nullptr};
    if (quant) {
        if (!(reuse && ctx->ws == ws_before)) {
            st = launch_dequant(ctx, W->qtype, W->data, W->row_bytes, 0, N, K, TK_DT_F16, wf, s);
            if (st != TK_OK) return st;
        }
        ctx->wexp_valid = true;
        ctx->wexp_data = W->data;
        ctx->wexp_qtype = W->qtype;
        ctx->wexp_rows = N;
        ctx->wexp_cols = K;
        ctx->wexp_rb = W->row_bytes;
        wplanes[0] = wf;
    } else {
        wplanes[0] = static_cast<const uint16_t*>(W->data);
        if (W->qtype == TK_F16X2) wplanes[1] = wplanes[0] + (size_t)N * K;
    }
    if (pl.w_two && !wplanes[1]) return fail(TK_ERR_INVALID, std::string(fn) + ": product set needs two weight planes");
    st = launch_act_split(ctx, A, a_dtype, M, a_cols, lda, pl.x_planes, true, pbase, row_exp, s, a_ld);
    if (st != TK_OK) return st;

    GemmDesc g;
    for (int i = 0; i < pl.x_planes; ++i) g.A[i] = pbase + (size_t)i * plane_elems;
    g.B[0] = wplanes[0];
    g.B[1] = wplanes[1];
    g.lda = a_ld;
    g.ldb = K;
    g.b_mn = dx;
    g.M = M;
    g.N = d_cols;
    g.K = a_cols;
    g.nprod = pl.nprod;
    for (int i = 0; i < 3; ++i) { g.pa[i] = pl.pa[i]; g.pb[i] = pl.pb[i]; }
    g.D = D;
    g.ldd = ldd;
    g.beta = beta != 0.0f;
    g.row_exp = row_exp;
    g.col_exp = W->qtype == TK_F16X2 ? W->scale_log2 : 0;
    // fp32-accurate product sets: sum in fp32 every kSegKb k-blocks (see tk_gemm.cu)
    g.seg_kb = pl.nprod > 1 ? kSegKb : 0;
    if (split) {
        g.split_ws = cv.take<float>((size_t)M * s_ld);
        g.split_ld = s_ld;
    }
    if (!rs_scatter) return launch_gemm(ctx, g, s);
    // reduce-scatter: D (the caller's [M/world, ldd] rows) receives the sum
    // of the owners' slots; the GEMM itself writes [M, K] rows of stride K
    RsDesc rs;
    st = rs_begin(ctx, M, d_cols, rs, s);
    if (st != TK_OK) return st;
    float* out = D;
    const long ldo = ldd;
    g.D = rs_scratch ? cv.take<float>((size_t)M * d_cols) : out;   // unread for a single segment
    g.ldd = d_cols;
    g.beta = 0;
    g.rs = &rs;
    st = launch_gemm(ctx, g, s);
    if (st != TK_OK) return st;
    return rs_finish(ctx, rs, d_cols, out, ldo, s);
}

// Forward and input gradient of one weight in one GEMM launch
// (tk_linear_fwd_dx, tk_linear_fwd_dx_rs): W is expanded once, both
// activations are split, and the two GEMMs share one persistent launch whose
// tiles interleave (launch_gemm_pair), so the dX epilogue's stores (over
// NVLink for the reduce-scatter) overlap the forward's MMAs and neither
// GEMM's last wave leaves SMs idle.
static tk_status linear_pair(tk_ctx* ctx, const tk_weight* W, const void* X, int x_dtype, int Mx, int ldx, float* Y,
                             int ldy, const void* dY, int dy_dtype, int Md, int lddy, float* dX, int ld_dx,
                             int products, cudaStream_t s, bool rs_scatter) {
    const char* fn = rs_scatter ? "tk_linear_fwd_dx_rs" : "tk_linear_fwd_dx";
    if (!ctx) return fail(TK_ERR_INVALID, std::string(fn) + ": null context");
    if (rs_scatter && !ctx->comm) return fail(TK_ERR_INVALID, std::string(fn) + ": tk_comm_init / tk_comm_connect first");
    tk_status st = check_weight(W, fn);
    if (st != TK_OK) return st;
    if (Mx < 0 || Md < 0) return fail(TK_ERR_INVALID, std::string(fn) + ": negative M");
    const bool want_fused = (products & TK_QFUSED) != 0;
    const bool want_reuse = (products & TK_WREUSE) != 0;
    const int prod = products & ~(TK_QFUSED | TK_WREUSE);
    if (Mx <= 128 || Md <= 128 || want_fused) {
        // a side too small for CTA-pair tiles, or the weight decoded inside
        // the GEMM: the two operations one after the other
        st = linear(ctx, W, X, x_dtype, Mx, ldx, Y, ldy, 0.0f, products, s, false);
        if (st != TK_OK) return st;
        return linear(ctx, W, dY, dy_dtype, Md, lddy, dX, ld_dx, 0.0f, products | TK_WREUSE, s, true, rs_scatter);
    }
    if (!X || !Y || !dY || !dX) return fail(TK_ERR_INVALID, std::string(fn) + ": null activation or output");
    const int N = W->rows, K = W->cols;
    if (ldx < K || ldy < N || lddy < N || ld_dx < K)
        return fail(TK_ERR_INVALID, std::string(fn) + ": leading dimension too small");
    for (int dt : {x_dtype, dy_dtype})
        if (dt != TK_DT_F32 && dt != TK_DT_F16 && dt != TK_DT_BF16)
            return fail(TK_ERR_INVALID, std::string(fn) + ": activation dtype");
    if (!aligned16(Y) || ldy % 4 || !aligned16(dX) || ld_dx % 4)
        return fail(TK_ERR_INVALID, std::string(fn) + ": outputs must be 16-byte aligned, ld % 4 == 0");
    Plan px, pd;
    st = plan_products(W, x_dtype, prod, px);
    if (st != TK_OK) return st;
    st = plan_products(W, dy_dtype, prod, pd);
    if (st != TK_OK) return st;
    const bool quant = W->qtype != TK_F16 && W->qtype != TK_F16X2;
    const long ax_ld = (K + 7) / 8 * 8, ad_ld = (N + 7) / 8 * 8;   // split-plane row strides (TMA: 16 bytes)
    const size_t ex = (size_t)Mx * ax_ld, ed = (size_t)Md * ad_ld;
    const bool rs_scratch = rs_scatter && pd.nprod > 1;
    const size_t need = (quant ? align256((size_t)N * K * 2) : 0) + align256(ex * 2 * px.x_planes) +
                        align256((size_t)Mx * 4) + align256(ed * 2 * pd.x_planes) + align256((size_t)Md * 4) +
                        (rs_scratch ? align256((size_t)Md * K * 4) : 0);
    const bool reuse = quant && want_reuse && ctx->wexp_valid && ctx->wexp_data == W->data &&
                       ctx->wexp_qtype == W->qtype && ctx->wexp_rows == N && ctx->wexp_cols == K &&
                       ctx->wexp_rb == W->row_bytes;
    const void* ws_before = ctx->ws;
    st = ws_ensure(ctx, need, s);
    if (st != TK_OK) return st;
    Carve cv(ctx->ws);
    uint16_t* wf = quant ? cv.take<uint16_t>((size_t)N * K) : nullptr;   // at the start of ws (TK_WREUSE)
    uint16_t* xp = cv.take<uint16_t>(ex * px.x_planes);
    int* xexp = cv.take<int>(Mx);
    uint16_t* dp = cv.take<uint16_t>(ed * pd.x_planes);
    int* dexp = cv.take<int>(Md);
    const uint16_t* wplanes[2] = {nullptr, nullptr};
    if (quant) {
        if (!(reuse && ctx->ws == ws_before)) {
            st = launch_dequant(ctx, W->qtype, W->data, W->row_bytes, 0, N, K, TK_DT_F16, wf, s);
            if (st != TK_OK) return st;
        }
        ctx->wexp_valid = true;
        ctx->wexp_data = W->data;
        ctx->wexp_qtype = W->qtype;
        ctx->wexp_rows = N;
        ctx->wexp_cols = K;
        ctx->wexp_rb = W->row_bytes;
        wplanes[0] = wf;
    } else {
        wplanes[0] = static_cast<const uint16_t*>(W->data);
        if (W->qtype == TK_F16X2) wplanes[1] = wplanes[0] + (size_t)N * K;
    }
    if ((px.w_two || pd.w_two) && !wplanes[1])
        return fail(TK_ERR_INVALID, std::string(fn) + ": product set needs two weight planes");
    st = launch_act_split(ctx, X, x_dtype, Mx, K, ldx, px.x_planes, true, xp, xexp, s, ax_ld);
    if (st != TK_OK) return st;
    st = launch_act_split(ctx, dY, dy_dtype, Md, N, lddy, pd.x_planes, true, dp, dexp, s, ad_ld);
    if (st != TK_OK) return st;
    auto desc = [&](const Plan& pl, const uint16_t* planes, size_t elems, long lda, int M, bool dx, float* D, long ldd,
                    const int* rexp) {
        GemmDesc g;
        for (int i = 0; i < pl.x_planes; ++i) g.A[i] = planes + (size_t)i * elems;
        g.B[0] = wplanes[0];
        g.B[1] = wplanes[1];
        g.lda = lda;
        g.ldb = K;
        g.b_mn = dx;
        g.M = M;
        g.N = dx ? K : N;
        g.K = dx ? N : K;
        g.nprod = pl.nprod;
        for (int i = 0; i < 3; ++i) { g.pa[i] = pl.pa[i]; g.pb[i] = pl.pb[i]; }
        g.D = D;
        g.ldd = ldd;
        g.row_exp = rexp;
        g.col_exp = W->qtype == TK_F16X2 ? W->scale_log2 : 0;
        g.seg_kb = pl.nprod > 1 ? kSegKb : 0;
        return g;
    };
    const GemmDesc gx = desc(px, xp, ex, ax_ld, Mx, false, Y, ldy, xexp);
    GemmDesc gd = desc(pd, dp, ed, ad_ld, Md, true, dX, ld_dx, dexp);
    RsDesc rs;
    if (rs_scatter) {
        st = rs_begin(ctx, Md, K, rs, s);
        if (st != TK_OK) return st;
        // the GEMM writes [Md, K] rows of stride K: earlier segments to a local
        // scratch, the last one to the owners (a single segment leaves D unread)
        gd.D = rs_scratch ? cv.take<float>((size_t)Md * K) : dX;
        gd.ldd = K;
        gd.rs = &rs;
    }
    st = gemm_pair_ok(gx, gd) ? launch_gemm_pair(ctx, gx, gd, s) : launch_gemm(ctx, gx, s);
    if (st != TK_OK) return st;
    if (!gemm_pair_ok(gx, gd)) {
        st = launch_gemm(ctx, gd, s);
        if (st != TK_OK) return st;
    }
    return rs_scatter ? rs_finish(ctx, rs, K, dX, ld_dx, s) : TK_OK;
}

}  // namespace tk

using namespace tk;

extern "C" {

const char* tk_last_error_string(void) { return g_last_error.c_str(); }

tk_status tk_init(int device, tk_ctx** out) {
    if (!out) return fail(TK_ERR_INVALID, "tk_init: null out");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(e, "tk_init: cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(TK_ERR_INVALID, "tk_init: no such device");
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "tk_init: cudaSetDevice");
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_fail(e, "tk_init: properties");
    if (prop.major != 10) return fail(TK_ERR_UNSUPPORTED, "tk_init: libtierk is built for sm_100a (B200)");
    tk_ctx* c = new tk_ctx();
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    e = cudaMalloc(&c->status, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->status, 0, sizeof(int));
    if (e == cudaSuccess) {
        c->flags_len = 1 << 16;
        e = cudaMalloc(&c->flags, sizeof(int) * c->flags_len);
        if (e == cudaSuccess) e = cudaMemset(c->flags, 0, sizeof(int) * c->flags_len);
    }
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "tk_init: status word");
    }
    *out = c;
    return TK_OK;
}

void tk_destroy(tk_ctx* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->status) cudaFree(ctx->status);
    if (ctx->flags) cudaFree(ctx->flags);
    if (ctx->iq_tab) cudaFree(ctx->iq_tab);
    if (ctx->sched) cudaFree(ctx->sched);
    comm_destroy(ctx);
    for (cudaEvent_t e : ctx->prof.ev) cudaEventDestroy(e);
    delete ctx;
}

tk_status tk_reserve(tk_ctx* ctx, size_t bytes) {
    if (!ctx) return fail(TK_ERR_INVALID, "tk_reserve: null context");
    return ws_ensure(ctx, bytes, nullptr);
}

size_t tk_workspace_bytes(const tk_ctx* ctx) { return ctx ? ctx->ws_bytes : 0; }

tk_status tk_profile(tk_ctx* ctx, int enable) {
    if (!ctx) return fail(TK_ERR_INVALID, "tk_profile: null context");
    if (enable < 0 || enable > 2) return fail(TK_ERR_INVALID, "tk_profile: enable must be 0, 1 or 2");
    ctx->prof.on = enable != 0;
    if (enable == 1) ctx->prof.used = 0;
    return TK_OK;
}

tk_status tk_profile_read(tk_ctx* ctx, int kind, double* total_ms, uint64_t* launches) {
    if (!ctx || !total_ms || !launches) return fail(TK_ERR_INVALID, "tk_profile_read: null argument");
    if (kind < 0 || kind >= PK_COUNT) return fail(TK_ERR_INVALID, "tk_profile_read: kernel kind");
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "tk_profile_read: sync");
    double t = 0.0;
    uint64_t n = 0;
    const tk_prof& p = ctx->prof;
    for (size_t i = 0; i < p.used; ++i) {
        if (p.kind[i] != kind) continue;
        float ms = 0.0f;
        e = cudaEventElapsedTime(&ms, p.ev[2 * i], p.ev[2 * i + 1]);
        if (e != cudaSuccess) return cuda_fail(e, "tk_profile_read: elapsed");
        t += ms;
        ++n;
    }
    *total_ms = t;
    *launches = n;
    return TK_OK;
}

uint64_t tk_launch_count(const tk_ctx* ctx) { return ctx ? ctx->launches : 0; }

tk_status tk_sync_status(tk_ctx* ctx, void* stream) {
    if (!ctx) return fail(TK_ERR_INVALID, "tk_sync_status: null context");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "tk_sync_status: stream");
    int code = 0;
    e = cudaMemcpy(&code, ctx->status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "tk_sync_status: read");
    if (code) {
        cudaMemset(ctx->status, 0, sizeof(int));
        if (code == DEV_TIMEOUT) return fail(TK_ERR_TIMEOUT, "a device-side bounded wait expired");
        return fail(TK_ERR_DEVICE, "a kernel reported invalid input (code " + std::to_string(code) + ")");
    }
    return TK_OK;
}

tk_status tk_set_iq_grids(tk_ctx* ctx, const tk_iq_grids* g) {
    if (!ctx) return fail(TK_ERR_INVALID, "tk_set_iq_grids: null context");
    if (!g || !g->iq2xxs || !g->iq2xs || !g->iq2s || !g->iq3xxs || !g->iq3s || !g->iq1s)
        return fail(TK_ERR_INVALID, "tk_set_iq_grids: every table pointer is required");
    std::vector<int8_t> h(tkq::GRID_BYTES);
    memcpy(h.data() + tkq::GRID_IQ2XXS, g->iq2xxs, 256 * 8);
    memcpy(h.data() + tkq::GRID_IQ2XS, g->iq2xs, 512 * 8);
    memcpy(h.data() + tkq::GRID_IQ2S, g->iq2s, 1024 * 8);
    memcpy(h.data() + tkq::GRID_IQ3XXS, g->iq3xxs, 256 * 4);
    memcpy(h.data() + tkq::GRID_IQ3S, g->iq3s, 512 * 4);
    memcpy(h.data() + tkq::GRID_IQ1S, g->iq1s, 2048 * 8);
    for (int i = 0; i < 128; ++i) h[tkq::GRID_SIGNS + i] = (int8_t)tkq::sign_byte(i);
    cudaError_t e = cudaDeviceSynchronize();   // no kernel may be reading the old table
    if (e != cudaSuccess) return cuda_fail(e, "tk_set_iq_grids: synchronize");
    if (!ctx->iq_tab) {
        e = cudaMalloc(&ctx->iq_tab, tkq::GRID_BYTES);
        if (e != cudaSuccess) {
            ctx->iq_tab = nullptr;
            return cuda_fail(e, "tk_set_iq_grids: allocate");
        }
    }
    e = cudaMemcpy(ctx->iq_tab, h.data(), tkq::GRID_BYTES, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return e == cudaSuccess ? TK_OK : cuda_fail(e, "tk_set_iq_grids: copy");
}

int tk_lmhead_chunk(size_t device_bytes, int hidden, int seq, int vocab) {
    if (device_bytes == 0) return 8192;
    const size_t per = (size_t)(hidden > 0 ? hidden : 0) * 6 + (size_t)(seq > 1 ? seq : 1) * 8;
    size_t c = device_bytes / 36 / per;
    c = c / 256 * 256;
    const size_t vmax = ((size_t)(vocab > 0 ? vocab : 0) + 255) / 256 * 256;
    if (c > vmax) c = vmax;
    if (c < 1024) c = 1024;
    return c > (size_t)INT32_MAX / 256 * 256 ? INT32_MAX / 256 * 256 : (int)c;
}

size_t tk_row_bytes(int qtype, int cols) {
    const int be = block_elems(qtype), bb = block_bytes(qtype);
    if (be <= 0 || cols < 0 || cols % be) return 0;
    return (size_t)(cols / be) * bb;
}

tk_status tk_dequant(tk_ctx* ctx, int qtype, const void* blocks, size_t row_bytes, int r0, int nrows, int cols,
                     int out_dtype, void* out, void* stream) {
    if (!ctx) return fail(TK_ERR_INVALID, "tk_dequant: null context");
    if (!dequant_supported(qtype)) return fail(TK_ERR_UNSUPPORTED, "tk_dequant: block type " + std::to_string(qtype));
    if (nrows < 0 || r0 < 0 || cols <= 0) return fail(TK_ERR_INVALID, "tk_dequant: bad row range / cols");
    if (nrows == 0) return TK_OK;
    if (!blocks || !out) return fail(TK_ERR_INVALID, "tk_dequant: null pointer");
    if (tk_row_bytes(qtype, cols) == 0 || row_bytes < tk_row_bytes(qtype, cols))
        return fail(TK_ERR_INVALID, "tk_dequant: cols not a block multiple or row_bytes too small");
    if (cols % 8) return fail(TK_ERR_INVALID, "tk_dequant: cols must be a multiple of 8");
    if (out_dtype != TK_DT_F32 && out_dtype != TK_DT_F16 && out_dtype != TK_DT_BF16)
        return fail(TK_ERR_INVALID, "tk_dequant: out dtype");
    if (!aligned16(out)) return fail(TK_ERR_INVALID, "tk_dequant: output must be 16-byte aligned");
    if ((qtype == TK_Q4_K || qtype == TK_Q5_K || qtype == TK_F16) && (!aligned16(blocks) || row_bytes % 16))
        return fail(TK_ERR_INVALID, "tk_dequant: Q4_K/Q5_K/F16 rows must be 16-byte aligned");
    return launch_dequant(ctx, qtype, blocks, row_bytes, r0, nrows, cols, out_dtype, out,
                          static_cast<cudaStream_t>(stream));
}

tk_status tk_gemv(tk_ctx* ctx, int qtype, const void* W, size_t row_bytes, int N, int K, const float* x, int ldx,
                  int M, float* y, int ldy, void* stream) {
    if (!ctx) return fail(TK_ERR_INVALID, "tk_gemv: null context");
    const bool frozen = (qtype & TK_WFROZEN) != 0;
    qtype &= ~TK_WFROZEN;
    if (!gemv_supported(qtype)) return fail(TK_ERR_UNSUPPORTED, "tk_gemv: weight type " + std::to_string(qtype));
    if (M < 1 || M > 16) return fail(TK_ERR_INVALID, "tk_gemv: M must be 1..16 (use tk_linear_fwd beyond)");
    if (N < 0 || K <= 0) return fail(TK_ERR_INVALID, "tk_gemv: bad shape");
    if (N == 0) return TK_OK;
    if (!W || !x || !y) return fail(TK_ERR_INVALID, "tk_gemv: null pointer");
    if (tk_row_bytes(qtype, K) == 0 || row_bytes < tk_row_bytes(qtype, K))
        return fail(TK_ERR_INVALID, "tk_gemv: K not a block multiple or row_bytes too small");
    if (K % 8 || ldx < K || ldx % 4 || !aligned16(x) || ldy < N)
        return fail(TK_ERR_INVALID, "tk_gemv: x must be 16-byte aligned, K % 8 == 0, ldx % 4 == 0");
    const bool staged = qtype == TK_Q8_0 || qtype == TK_Q4_0 || qtype == TK_Q4_K || qtype == TK_Q5_K;
    const bool dense = qtype == TK_F16 || qtype == TK_BF16 || qtype == TK_F32;
    if ((staged || dense) && (!aligned16(W) || row_bytes % 16))
        return fail(TK_ERR_INVALID, "tk_gemv: weight rows must be 16-byte aligned");
    if ((qtype == TK_Q8_0 || qtype == TK_Q4_0) && K % 256)
        return fail(TK_ERR_INVALID, "tk_gemv: Q8_0/Q4_0 rows need K % 256 == 0");
    return launch_gemv(ctx, qtype, W, row_bytes, N, K, x, ldx, M, y, ldy, static_cast<cudaStream_t>(stream), frozen);
}

tk_status tk_gemv_multi(tk_ctx* ctx, int qtype, int nseg, const void* const* W, const int* rows, float* const* y,
                        const int* ldy, size_t row_bytes, int K, const float* x, int ldx, int M, void* stream) {
    if (!ctx) return fail(TK_ERR_INVALID, "tk_gemv_multi: null context");
    if (nseg < 1 || nseg > TK_GEMV_MAXSEG || !W || !rows || !y || !ldy)
        return fail(TK_ERR_INVALID, "tk_gemv_multi: nseg must be 1..TK_GEMV_MAXSEG with W, rows, y, ldy given");
    long total = 0;
    bool aligned = true;
    for (int i = 0; i < nseg; ++i) {
        if (!W[i] || !y[i] || rows[i] <= 0 || ldy[i] < rows[i])
            return fail(TK_ERR_INVALID, "tk_gemv_multi: segment " + std::to_string(i) + ": null pointer or bad rows/ldy");
        total += rows[i];
        aligned = aligned && aligned16(W[i]);
    }
    if (total > (1L << 30)) return fail(TK_ERR_INVALID, "tk_gemv_multi: too many rows");
    const bool frozen = (qtype & TK_WFROZEN) != 0;
    const int t = qtype & ~TK_WFROZEN;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (M >= 1 && M <= 2 && aligned && row_bytes % 16 == 0 && K > 0 && K % 256 == 0 && x && ldx >= K &&
        ldx % 4 == 0 && aligned16(x) && tk_row_bytes(t, K) != 0 && row_bytes >= tk_row_bytes(t, K) &&
        gemv_imma_multi_ok(t, row_bytes, K, M))
        return launch_gemv_imma_multi(ctx, t, nseg, W, rows, y, ldy, row_bytes, K, x, ldx, M, frozen, s);
    for (int i = 0; i < nseg; ++i) {
        tk_status st = tk_gemv(ctx, qtype, W[i], row_bytes, rows[i], K, x, ldx, M, y[i], ldy[i], stream);
        if (st != TK_OK) return st;
    }
    return TK_OK;
}

tk_status tk_linear_fwd(tk_ctx* ctx, const tk_weight* W, const void* X, int x_dtype, int M, int ldx, float* Y, int ldy,
                        float beta, int products, void* stream) {
    return linear(ctx, W, X, x_dtype, M, ldx, Y, ldy, beta, products, static_cast<cudaStream_t>(stream), false);
}

tk_status tk_linear_dx(tk_ctx* ctx, const tk_weight* W, const void* dY, int dy_dtype, int M, int lddy, float* dX,
                       int lddx, float beta, int products, void* stream) {
    return linear(ctx, W, dY, dy_dtype, M, lddy, dX, lddx, beta, products, static_cast<cudaStream_t>(stream), true);
}

tk_status tk_linear_fwd_dx(tk_ctx* ctx, const tk_weight* W, const void* X, int x_dtype, int Mx, int ldx, float* Y,
                           int ldy, const void* dY, int dy_dtype, int Md, int lddy, float* dX, int lddx, int products,
                           void* stream) {
    return linear_pair(ctx, W, X, x_dtype, Mx, ldx, Y, ldy, dY, dy_dtype, Md, lddy, dX, lddx, products,
                       static_cast<cudaStream_t>(stream), false);
}

tk_status tk_linear_fwd_dx_rs(tk_ctx* ctx, const tk_weight* W, const void* X, int x_dtype, int Mx, int ldx, float* Y,
                              int ldy, const void* dY, int dy_dtype, int Md, int lddy, float* dX_rows, int ldd,
                              int products, void* stream) {
    return linear_pair(ctx, W, X, x_dtype, Mx, ldx, Y, ldy, dY, dy_dtype, Md, lddy, dX_rows, ldd, products,
                       static_cast<cudaStream_t>(stream), true);
}

tk_status tk_weight_split_f32(tk_ctx* ctx, const float* W32, int rows, int cols, uint16_t* planes, int* scale_log2,
                              void* stream) {
    if (!ctx || !W32 || !planes || !scale_log2) return fail(TK_ERR_INVALID, "tk_weight_split_f32: null argument");
    if (rows <= 0 || cols <= 0) return fail(TK_ERR_INVALID, "tk_weight_split_f32: empty weight");
    return weight_split_f32(ctx, W32, rows, cols, planes, scale_log2, static_cast<cudaStream_t>(stream));
}

tk_status tk_split3(tk_ctx* ctx, const float* x, size_t n, uint16_t* h, uint16_t* m, uint16_t* l, void* stream) {
    if (!ctx || (n && (!x || !h || !m || !l))) return fail(TK_ERR_INVALID, "tk_split3: null argument");
    return launch_split3_raw(ctx, x, n, h, m, l, static_cast<cudaStream_t>(stream));
}

// ---- LM head -------------------------------------------------------------
static tk_status lm_check(tk_ctx* ctx, const uint16_t* W, int V_shard, int H, const float* X, int T,
                          const int32_t* labels, const uint8_t* mask, int chunk, int products, const char* fn) {
    if (!ctx || !W || !X || !labels || !mask) return fail(TK_ERR_INVALID, std::string(fn) + ": null argument");
    if (V_shard <= 0 || H <= 0 || T < 2) return fail(TK_ERR_INVALID, std::string(fn) + ": bad shape");
    if (H % 8 || !aligned16(W) || !aligned16(X))
        return fail(TK_ERR_INVALID, std::string(fn) + ": H % 8 == 0 and 16-byte aligned W, X required");
    if (chunk <= 0 || chunk % 256 || V_shard % 256)
        return fail(TK_ERR_INVALID, std::string(fn) + ": chunk and V_shard must be multiples of 256");
    if (products != TK_X3_REF && products != TK_X2 && products != TK_X3_AUTO)
        return fail(TK_ERR_INVALID, std::string(fn) + ": products must be TK_X3_REF or TK_X2");
    return TK_OK;
}

// X planes for the head: nplanes x [T-1, H] with per-row exponents.
static tk_status lm_split_x(tk_ctx* ctx, Carve& cv, const float* X, int T, int H, int np, uint16_t** planes,
                            int** row_exp, cudaStream_t s) {
    const size_t pe = (size_t)(T - 1) * H;
    uint16_t* base = cv.take<uint16_t>(pe * np);
    *row_exp = cv.take<int>(T);
    *planes = base;
    return launch_act_split(ctx, X, TK_DT_F32, T - 1, H, H, np, true, base, *row_exp, s);
}

tk_status tk_lmhead_stats(tk_ctx* ctx, const uint16_t* W, int v0, int V_shard, int H, const float* X, int T,
                          const int32_t* labels, const uint8_t* mask, float softcap, int chunk, int products,
                          double* rmax, double* rsum, int32_t* amax, float* tgt, void* stream) {
    tk_status st = lm_check(ctx, W, V_shard, H, X, T, labels, mask, chunk, products, "tk_lmhead_stats");
    if (st != TK_OK) return st;
    if (!rmax || !rsum || !amax || !tgt) return fail(TK_ERR_INVALID, "tk_lmhead_stats: null state");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int np = products == TK_X2 ? 2 : 3;
    const int rows = T - 1;
    const int ntiles = chunk / 256;
    const size_t need = align256((size_t)rows * H * 2 * np) + align256((size_t)T * 4) +
                        align256((size_t)rows * ntiles * 4) * 3 + align256((size_t)rows * ntiles * 8);
    st = ws_ensure(ctx, need, s);
    if (st != TK_OK) return st;
    Carve cv(ctx->ws);
    uint16_t* xp;
    int* rexp;
    st = lm_split_x(ctx, cv, X, T, H, np, &xp, &rexp, s);
    if (st != TK_OK) return st;
    float* pmax = cv.take<float>((size_t)rows * ntiles);
    int32_t* parg = cv.take<int32_t>((size_t)rows * ntiles);
    float* ptgt = cv.take<float>((size_t)rows * ntiles);
    double* psum = cv.take<double>((size_t)rows * ntiles);
    for (int c0 = 0; c0 < V_shard; c0 += chunk) {
        const int vc = V_shard - c0 < chunk ? V_shard - c0 : chunk;
        GemmDesc g;
        for (int p = 0; p < np; ++p) g.A[p] = xp + (size_t)p * rows * H;
        g.B[0] = W + (size_t)c0 * H;
        g.lda = H; g.ldb = H; g.b_mn = false;
        g.M = rows; g.N = vc; g.K = H;
        g.nprod = np;
        for (int p = 0; p < np; ++p) { g.pa[p] = np - 1 - p; g.pb[p] = 0; }
        g.D = reinterpret_cast<float*>(pmax);   // unused by this epilogue; must be valid & aligned
        g.ldd = 4;
        g.row_exp = rexp;
        LseDesc e;
        e.pmax = pmax; e.parg = parg; e.psum = psum; e.ptgt = ptgt;
        e.labels = labels; e.v0 = v0 + c0; e.cap = softcap; e.ld_part = ntiles;
        st = launch_gemm_lse(ctx, g, e, s);
        if (st != TK_OK) return st;
        st = launch_lse_merge(ctx, pmax, parg, psum, ptgt, ntiles, (vc + 255) / 256, rows, vc, v0 + c0, labels, mask,
                              rmax, rsum, amax, tgt, s);
        if (st != TK_OK) return st;
    }
    return TK_OK;
}

tk_status tk_lmhead_grad(tk_ctx* ctx, const uint16_t* W, int v0, int V_shard, int H, const float* X, int T,
                         const int32_t* labels, const uint8_t* mask, int n_loss, float softcap, int chunk, int products,
                         const double* rmax, const double* rsum, float* dX, void* stream) {
    tk_status st = lm_check(ctx, W, V_shard, H, X, T, labels, mask, chunk, products, "tk_lmhead_grad");
    if (st != TK_OK) return st;
    if (!rmax || !rsum || !dX) return fail(TK_ERR_INVALID, "tk_lmhead_grad: null state");
    if (n_loss <= 0) return TK_OK;   // every row masked: dlogit is zero
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int np = products == TK_X2 ? 2 : 3;
    const int rows = T - 1;
    const size_t need = align256((size_t)rows * H * 2 * np) + align256((size_t)T * 4) +
                        align256((size_t)rows * chunk * 2) * np;
    st = ws_ensure(ctx, need, s);
    if (st != TK_OK) return st;
    Carve cv(ctx->ws);
    uint16_t* xp;
    int* rexp;
    st = lm_split_x(ctx, cv, X, T, H, np, &xp, &rexp, s);
    if (st != TK_OK) return st;
    const size_t pstride = (size_t)rows * chunk;
    uint16_t* dl = cv.take<uint16_t>(pstride * np);
    // |dlogit| <= mask/n_loss <= 255/n_loss; 2^dl_exp * 255/n_loss < 2^15.
    const int dl_exp = 7 + (int)std::floor(std::log2((double)n_loss));
    for (int c0 = 0; c0 < V_shard; c0 += chunk) {
        const int vc = V_shard - c0 < chunk ? V_shard - c0 : chunk;
        GemmDesc g;
        for (int p = 0; p < np; ++p) g.A[p] = xp + (size_t)p * rows * H;
        g.B[0] = W + (size_t)c0 * H;
        g.lda = H; g.ldb = H; g.b_mn = false;
        g.M = rows; g.N = vc; g.K = H;
        g.nprod = np;
        for (int p = 0; p < np; ++p) { g.pa[p] = np - 1 - p; g.pb[p] = 0; }
        g.D = dX; g.ldd = H;           // unused by this epilogue
        g.row_exp = rexp;
        DlogitDesc e;
        e.rmax = rmax; e.rsum = rsum; e.labels = labels; e.mask = mask;
        e.T = T; e.v0 = v0 + c0; e.n_loss = n_loss; e.cap = softcap; e.dl_exp = dl_exp; e.nplanes = np;
        e.planes = dl; e.plane_stride = (long)pstride; e.ld = vc;
        st = launch_gemm_dlogit(ctx, g, e, s);
        if (st != TK_OK) return st;
        GemmDesc d;
        for (int p = 0; p < np; ++p) d.A[p] = dl + (size_t)p * pstride;
        d.B[0] = W + (size_t)c0 * H;
        d.lda = vc; d.ldb = H; d.b_mn = true;
        d.M = rows; d.N = H; d.K = vc;
        d.nprod = np;
        for (int p = 0; p < np; ++p) { d.pa[p] = np - 1 - p; d.pb[p] = 0; }
        d.D = dX; d.ldd = H; d.beta = 1;
        d.col_exp = dl_exp;
        d.seg_kb = kSegKb;
        st = launch_gemm(ctx, d, s);
        if (st != TK_OK) return st;
    }
    return TK_OK;
}

tk_status tk_lmhead_fused(tk_ctx* ctx, const uint16_t* W, int v0, int V_shard, int H, const float* X, int T,
                          const int32_t* labels, const uint8_t* mask, float softcap, int chunk, int products,
                          double* rmax, double* rsum, int32_t* amax, float* tgt, float* dX, void* stream) {
    tk_status st = lm_check(ctx, W, V_shard, H, X, T, labels, mask, chunk, products, "tk_lmhead_fused");
    if (st != TK_OK) return st;
    if (!rmax || !rsum || !amax || !tgt || !dX) return fail(TK_ERR_INVALID, "tk_lmhead_fused: null state");
    if (!aligned16(dX)) return fail(TK_ERR_INVALID, "tk_lmhead_fused: dX must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int np = products == TK_X2 ? 2 : 3;
    const int rows = T - 1;
    const int ntiles = chunk / 256;
    const size_t pstride = (size_t)rows * chunk;
    const size_t need = align256((size_t)rows * H * 2 * np) + align256((size_t)T * 4) +
                        align256((size_t)rows * ntiles * 4) * 3 + align256((size_t)rows * ntiles * 8) +
                        align256(pstride * 4) + align256(pstride * 2) * 2 + align256((size_t)rows * 4);
    st = ws_ensure(ctx, need, s);
    if (st != TK_OK) return st;
    Carve cv(ctx->ws);
    uint16_t* xp;
    int* rexp;
    st = lm_split_x(ctx, cv, X, T, H, np, &xp, &rexp, s);
    if (st != TK_OK) return st;
    float* pmax = cv.take<float>((size_t)rows * ntiles);
    int32_t* parg = cv.take<int32_t>((size_t)rows * ntiles);
    float* ptgt = cv.take<float>((size_t)rows * ntiles);
    double* psum = cv.take<double>((size_t)rows * ntiles);
    float* Z = cv.take<float>(pstride);
    uint16_t* P = cv.take<uint16_t>(pstride * 2);
    float* alpha = cv.take<float>(rows);
    for (int c0 = 0; c0 < V_shard; c0 += chunk) {
        const int vc = V_shard - c0 < chunk ? V_shard - c0 : chunk;
        // logits of the chunk: partial statistics + the logits themselves
        GemmDesc g;
        for (int p = 0; p < np; ++p) g.A[p] = xp + (size_t)p * rows * H;
        g.B[0] = W + (size_t)c0 * H;
        g.lda = H; g.ldb = H; g.b_mn = false;
        g.M = rows; g.N = vc; g.K = H;
        g.nprod = np;
        for (int p = 0; p < np; ++p) { g.pa[p] = np - 1 - p; g.pb[p] = 0; }
        g.D = reinterpret_cast<float*>(pmax);   // unused by this epilogue; must be valid & aligned
        g.ldd = 4;
        g.row_exp = rexp;
        LseDesc e;
        e.pmax = pmax; e.parg = parg; e.psum = psum; e.ptgt = ptgt;
        e.labels = labels; e.v0 = v0 + c0; e.cap = softcap; e.ld_part = ntiles;
        e.zout = Z; e.ldz = vc;
        st = launch_gemm_lse(ctx, g, e, s);
        if (st != TK_OK) return st;
        st = launch_lse_merge(ctx, pmax, parg, psum, ptgt, ntiles, (vc + 255) / 256, rows, vc, v0 + c0, labels, mask,
                              rmax, rsum, amax, tgt, s, alpha);
        if (st != TK_OK) return st;
        // P = exp(l - m_new) * softcap' in fp16 hi + lo
        st = launch_lm_prob(ctx, Z, vc, rows, vc, rmax, mask, softcap, P, (long)rows * vc, vc, s);
        if (st != TK_OK) return st;
        // dXacc = alpha * dXacc + P . W_chunk
        GemmDesc d;
        d.A[0] = P;
        d.A[1] = P + (size_t)rows * vc;
        d.B[0] = W + (size_t)c0 * H;
        d.lda = vc; d.ldb = H; d.b_mn = true;
        d.M = rows; d.N = H; d.K = vc;
        d.nprod = 2;
        d.pa[0] = 1; d.pa[1] = 0; d.pb[0] = 0; d.pb[1] = 0;   // low part first
        d.D = dX; d.ldd = H;
        d.beta = c0 > 0;
        d.row_alpha = alpha;
        // The probabilities are in [0, 1]: 64 k-blocks per fp32 segment keep the
        // head's dX within 3.5e-7 of fp64 at C4's shape (16: 2.3e-7, the whole
        // chunk: 8.5e-7; bound 1e-5), with a quarter of the segment epilogues'
        // read-modify-writes of dX (C4 step 80.4 -> 70.6 ms on B200).
        d.seg_kb = 4 * kSegKb;
        st = launch_gemm(ctx, d, s);
        if (st != TK_OK) return st;
    }
    return TK_OK;
}

tk_status tk_lmhead_finish(tk_ctx* ctx, const uint16_t* W, int v0, int V_shard, int H, int T, const int32_t* labels,
                           const uint8_t* mask, int n_loss, float softcap, const double* rsum, const float* tgt,
                           float* dX, void* stream) {
    if (!ctx || !W || !labels || !mask || !rsum || !tgt || !dX) return fail(TK_ERR_INVALID, "tk_lmhead_finish: null argument");
    if (T < 2 || H <= 0 || V_shard <= 0) return fail(TK_ERR_INVALID, "tk_lmhead_finish: bad shape");
    if (n_loss <= 0) return launch_lm_finish(ctx, W, v0, V_shard, H, T, labels, mask, 1, softcap, rsum, tgt, dX,
                                             static_cast<cudaStream_t>(stream));   // every row zero
    return launch_lm_finish(ctx, W, v0, V_shard, H, T, labels, mask, n_loss, softcap, rsum, tgt, dX,
                            static_cast<cudaStream_t>(stream));
}

tk_status tk_quantize(tk_ctx* ctx, int qtype, const void* x, int x_dtype, int rows, int cols, int ldx, void* out,
                      size_t row_bytes, void* stream) {
    if (!ctx || !x || !out) return fail(TK_ERR_INVALID, "tk_quantize: null argument");
    if (qtype != TK_Q8_0 && qtype != TK_Q4_K && qtype != TK_Q5_K && qtype != TK_Q6_K)
        return fail(TK_ERR_UNSUPPORTED, "tk_quantize: the reference quantizes to Q8_0, Q4_K, Q5_K and Q6_K only");
    if (rows < 0 || cols <= 0 || ldx < cols) return fail(TK_ERR_INVALID, "tk_quantize: bad shape");
    if (rows == 0) return TK_OK;
    const size_t need_rb = tk_row_bytes(qtype, cols);
    if (need_rb == 0) return fail(TK_ERR_INVALID, "tk_quantize: cols is not a multiple of the block size");
    if (row_bytes < need_rb) return fail(TK_ERR_INVALID, "tk_quantize: row_bytes too small");
    if (x_dtype != TK_DT_F32 && x_dtype != TK_DT_BF16) return fail(TK_ERR_INVALID, "tk_quantize: x must be fp32 or bf16");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float* xf = static_cast<const float*>(x);
    long ldf = ldx;
    if (x_dtype == TK_DT_BF16) {
        // bf16 sources (safetensors, as quant_main reads them) widen exactly to fp32 first
        tk_status st = ws_ensure(ctx, align256((size_t)rows * cols * 4), s);
        if (st != TK_OK) return st;
        float* w = static_cast<float*>(ctx->ws);
        st = launch_bf16_to_f32(ctx, static_cast<const uint16_t*>(x), ldx, rows, cols, w, s);
        if (st != TK_OK) return st;
        xf = w;
        ldf = cols;
    }
    return launch_quantize(ctx, qtype, xf, ldf, rows, cols, static_cast<uint8_t*>(out), row_bytes, s);
}

tk_status tk_linear_dx_rs(tk_ctx* ctx, const tk_weight* W, const void* dY, int dy_dtype, int M, int lddy,
                          float* dX_rows, int ldd, int products, void* stream) {
    if (!ctx) return fail(TK_ERR_INVALID, "tk_linear_dx_rs: null context");
    if (!ctx->comm) return fail(TK_ERR_INVALID, "tk_linear_dx_rs: tk_comm_init / tk_comm_connect first");
    return linear(ctx, W, dY, dy_dtype, M, lddy, dX_rows, ldd, 0.0f, products, static_cast<cudaStream_t>(stream),
                  true, true);
}

tk_status tk_lmhead_loss(tk_ctx* ctx, int T, const int32_t* labels, const uint8_t* mask, const double* rmax,
                         const double* rsum, const int32_t* amax, const float* tgt, double* loss_sum, int32_t* hits,
                         void* stream) {
    if (!ctx || !labels || !mask || !rmax || !rsum || !amax || !tgt || !loss_sum || !hits)
        return fail(TK_ERR_INVALID, "tk_lmhead_loss: null argument");
    if (T < 2) return fail(TK_ERR_INVALID, "tk_lmhead_loss: T < 2");
    return launch_lm_loss(ctx, T, labels, mask, rmax, rsum, amax, tgt, loss_sum, hits,
                          static_cast<cudaStream_t>(stream));
}

tk_status tk_lmhead_rescale(tk_ctx* ctx, int n, double* rmax_local, double* rsum_local, const double* rmax_global,
                            float* dX, int H, void* stream) {
    if (!ctx || (n > 0 && (!rmax_local || !rsum_local || !rmax_global)))
        return fail(TK_ERR_INVALID, "tk_lmhead_rescale: null argument");
    if (dX && H <= 0) return fail(TK_ERR_INVALID, "tk_lmhead_rescale: H must be positive with dX");
    return launch_lm_rescale(ctx, n, rmax_local, rsum_local, rmax_global, static_cast<cudaStream_t>(stream), dX, H);
}

}  // extern "C"
