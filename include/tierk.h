/*
 * tierk.h -- C ABI of libtierk.so, the B200 (sm_100a) frozen-weight linear
 * path of tierlm: block-quantized weights dequantized for GEMV/GEMM, the fp16
 * "x3" split GEMM, and the chunked-vocabulary LM head with running
 * cross-entropy and its input gradient.
 *
 * The reference engine has no C ABI; its hot path is a set of internal C++
 * statics called with raw device pointers.  Each entry point below names the
 * reference function (file:line in the Eberhard-AIDEV/Tier tree) it replaces
 * and keeps that function's units: row-major W[N,K] (out x in), X[M,K],
 * Y[M,N] = X.W^T, dX[M,K] = dY.W, fp32 outputs, the reference's block
 * layouts (tier/quant.h:25-29) and type codes (tier/quant.h:20-23).
 *
 * Conventions
 *  - All data pointers are DEVICE pointers owned by the caller, except where
 *    noted.  The library owns only its context workspace.
 *  - Every call is asynchronous on `stream` (a cudaStream_t; NULL = legacy
 *    default stream) and returns a status; no call aborts the process.
 *    tk_last_error_string() describes the last failure on the calling thread.
 *  - A context is bound to one device; use it from one host thread at a time.
 *  - Shapes are validated on the host (block multiples, alignment); device
 *    kernels never trap: bounded waits write a code into the context status
 *    word, read by tk_sync_status().
 */
#ifndef TIERK_H
#define TIERK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tk_status {
    TK_OK = 0,
    TK_ERR_INVALID = 1,     /* bad shape, alignment, pointer or type code        */
    TK_ERR_UNSUPPORTED = 2, /* valid request this build does not implement       */
    TK_ERR_CUDA = 3,        /* CUDA runtime/driver error                         */
    TK_ERR_NOMEM = 4,       /* workspace growth failed                           */
    TK_ERR_TIMEOUT = 5,     /* a device-side bounded wait expired                */
    TK_ERR_DEVICE = 6       /* device kernel reported invalid input              */
} tk_status;

/* Weight block types: the reference's QT_* codes (tier/quant.h:20-23). */
enum {
    TK_F32 = 0, TK_F16 = 1, TK_Q4_0 = 2, TK_Q4_1 = 3, TK_Q5_0 = 6, TK_Q5_1 = 7,
    TK_Q8_0 = 8, TK_Q2_K = 10, TK_Q3_K = 11, TK_Q4_K = 12, TK_Q5_K = 13,
    TK_Q6_K = 14, TK_BF16 = 30,
    /* types whose levels come from a 16-entry list or from base-3 digits */
    TK_IQ4_NL = 20, TK_IQ4_XS = 23, TK_TQ1_0 = 34, TK_TQ2_0 = 35, TK_MXFP4 = 39,
    TK_NF4 = 200, TK_FP4 = 201,
    /* lattice types: need the tables of tk_set_iq_grids */
    TK_IQ2_XXS = 16, TK_IQ2_XS = 17, TK_IQ3_XXS = 18, TK_IQ1_S = 19, TK_IQ3_S = 21, TK_IQ2_S = 22,
    TK_IQ1_M = 29,
    /* fp32 weight stored as two fp16 planes hi = f16(W*2^s), lo = f16(W*2^s - hi);
       plane lo starts rows*row_bytes bytes after plane hi (see tk_weight_split_f32) */
    TK_F16X2 = 100
};

/* Element types of activations / gradients / dequant output. */
enum { TK_DT_F32 = 0, TK_DT_F16 = 1, TK_DT_BF16 = 2 };

/* Tensor-core product sets for the split GEMM.
 *  TK_X3_REF : X (fp32) split into three fp16 parts h,m,l; W single fp16;
 *              products W.xl + W.xm + W.xh -- the reference's fp3gemm
 *              (tier/tier.cpp:922-943).
 *  TK_X3_HHL : X split into h,l and W into h,l (TK_F16X2);
 *              products Xh.Wh + Xh.Wl + Xl.Wh (near-fp32 for fp32 W).
 *  TK_X2     : X split into h,l; W single fp16; products W.xl + W.xh.
 *  TK_X1     : one product of fp16 X (or bf16 X converted exactly) and fp16 W.
 *  TK_X3_AUTO: TK_X3_REF for fp32 X with fp16/quant W, TK_X3_HHL for
 *              TK_F16X2 W, TK_X1 for fp16/bf16 X. */
enum { TK_X3_AUTO = 0, TK_X3_REF = 1, TK_X3_HHL = 2, TK_X2 = 3, TK_X1 = 4 };
/* OR-able flag for `products` of tk_linear_fwd / tk_linear_dx with a
 * block-quantized weight: decode W inside the GEMM (converter warps write the
 * fp16 operand tiles in shared memory) instead of expanding it to fp16 in the
 * workspace first.  Needs M > 128 and K % 256 == 0 (otherwise ignored).  The
 * decode is repeated for every 256-row tile of M, so it is slower than the
 * default at every M measured on B200 so far. */
enum { TK_QFUSED = 0x100 };
/* OR-able flag for `products` of tk_linear_fwd / tk_linear_dx with a
 * block-quantized weight: W's bytes have not changed since the previous
 * linear call on this context that expanded it (a frozen weight's forward
 * followed by its dX), so that call's fp16 expansion, kept at the start of
 * the workspace, may be used without dequantizing again.  Reused only when
 * the previous workspace user was a linear call on the same data pointer and
 * shape; otherwise W is dequantized as usual.  Calls on different streams
 * must be ordered by the caller. */
enum { TK_WREUSE = 0x400 };
/* OR-ed into tk_gemv's qtype: W is frozen (see tk_gemv). */
enum { TK_WFROZEN = 0x200 };

typedef struct tk_ctx tk_ctx;

/* A frozen weight W[rows=N, cols=K] resident in device memory. */
typedef struct tk_weight {
    int qtype;          /* TK_* block type                                           */
    int rows;           /* N, output features                                        */
    int cols;           /* K, input features (multiple of the block size)            */
    int scale_log2;     /* TK_F16X2: planes hold W * 2^scale_log2; else 0            */
    size_t row_bytes;   /* bytes per row (q_row_bytes(qtype, cols); fp16 plane row)  */
    const void *data;   /* device pointer to row 0                                   */
} tk_weight;

/* ---- context ------------------------------------------------------------ */
tk_status tk_init(int device, tk_ctx **out);
void tk_destroy(tk_ctx *ctx);
const char *tk_last_error_string(void);
/* Grow the context workspace to at least `bytes` now (entry points grow it on
 * demand otherwise, which synchronizes the device). */
tk_status tk_reserve(tk_ctx *ctx, size_t bytes);
size_t tk_workspace_bytes(const tk_ctx *ctx);
/* Synchronize `stream` and report any device-side status (timeouts, invalid
 * input detected by a kernel) raised since the last call; clears it. */
tk_status tk_sync_status(tk_ctx *ctx, void *stream);
/* Number of kernels this context has launched (diagnostics / bench). */
uint64_t tk_launch_count(const tk_ctx *ctx);

/* Per-kernel timing (diagnostics; no reference counterpart).  While enabled,
 * every launch is bracketed by CUDA events on its own stream (up to 8192
 * launches; later launches are not recorded).  tk_profile(ctx, 1) starts a
 * new record, 2 resumes recording into the current one, 0 pauses (the
 * record is kept), so that a caller can time a sample of its launches
 * without events between all the others (an event between two kernels holds
 * the second back until the first has finished and the event is written).
 * tk_profile_read synchronizes the device and returns the summed event time
 * (ms) and number of recorded launches of one kernel family.  TK_PROF_COMM:
 * the reduce-scatter's owner reduce (with its wait for the peers' tiles) and
 * the peer collectives' kernels. */
enum { TK_PROF_GEMM = 0, TK_PROF_DEQUANT = 1, TK_PROF_SPLIT = 2, TK_PROF_GEMV = 3, TK_PROF_LMHEAD = 4,
       TK_PROF_COMM = 5 };
tk_status tk_profile(tk_ctx *ctx, int enable);
tk_status tk_profile_read(tk_ctx *ctx, int kind, double *total_ms, uint64_t *launches);

/* ---- block formats ------------------------------------------------------ */
/* Bytes of one row of `cols` elements of `qtype`; 0 if unsupported or cols is
 * not a block multiple.  Replaces q_row_bytes (tier/quant.h:33). */
size_t tk_row_bytes(int qtype, int cols);

/* ---- dequant ------------------------------------------------------------ */
/* out[r, c] = value of element c of row r0+r, for r < nrows, as fp32, fp16
 * (round-to-nearest-even of the fp32 value) or bf16.  Bit-exact with
 * q_val / tier_fp16(q_val).  Replaces dq_launch / dq_k (tier/tier.cpp:294-298).
 * Supported qtype: all TK_* block types except TK_F16X2 -- the reference's 27;
 * the lattice types once tk_set_iq_grids has run on the context. */
tk_status tk_dequant(tk_ctx *ctx, int qtype, const void *blocks, size_t row_bytes,
                     int r0, int nrows, int cols, int out_dtype, void *out, void *stream);

/* ---- IQ1 / IQ2 / IQ3 lattice tables --------------------------------------- */
/* TK_IQ2_XXS, TK_IQ2_XS, TK_IQ2_S, TK_IQ3_XXS, TK_IQ3_S, TK_IQ1_S and TK_IQ1_M
 * look groups of 8 (4) values up in fixed lattice tables: the format's data,
 * tier/quant_tables.h qt_iq2xxs_grid ... qt_iq1s_grid (gguf-py's IQ*.grid hold
 * the same numbers).  The library does not carry them: the caller registers
 * its copies (host pointers, int8 entries) once per context; until then these
 * types return TK_ERR_UNSUPPORTED from every entry point.  The sign table
 * (qt_ksigns) follows from a rule and is built here.  The call synchronizes
 * the device before and after the copy. */
typedef struct tk_iq_grids {
    const int8_t *iq2xxs;   /* [256][8]   qt_iq2xxs_grid */
    const int8_t *iq2xs;    /* [512][8]   qt_iq2xs_grid  */
    const int8_t *iq2s;     /* [1024][8]  qt_iq2s_grid   */
    const int8_t *iq3xxs;   /* [256][4]   qt_iq3xxs_grid */
    const int8_t *iq3s;     /* [512][4]   qt_iq3s_grid   */
    const int8_t *iq1s;     /* [2048][8]  qt_iq1s_grid (IQ1_S and IQ1_M) */
} tk_iq_grids;
tk_status tk_set_iq_grids(tk_ctx *ctx, const tk_iq_grids *grids);

/* ---- quantizer ------------------------------------------------------------ */
/* out rows (row_bytes apart) = the blocks of x [rows, cols] (fp32, or bf16
 * widened exactly) in Q8_0, Q4_K, Q5_K or Q6_K, byte for byte what the
 * reference's CPU quantizer writes (q_row, tier/quant.h:201-204: q8_0_row,
 * qk_minmax_row, q6_k_row; run per matrix by quant_main, tier/tier.cpp:2698-2746). */
tk_status tk_quantize(tk_ctx *ctx, int qtype, const void *x, int x_dtype, int rows, int cols, int ldx,
                      void *out, size_t row_bytes, void *stream);

/* ---- `.tq` quantized-base files ------------------------------------------ */
/* Reader: the reference's tq_load (tier/tier.cpp:274-292) -- header
 * "TQB1 <hb> <n>", "#key value" lines, one "<name> <type> <rows> <cols>
 * <offset> <bytes> [err]" line per matrix, 4096-aligned block data.  Entries
 * keep the file's order.  tk_tq_read copies entry i to host memory or (with
 * dst_on_device) to device memory through a pinned 32 MiB stage. */
typedef struct tk_tq tk_tq;
tk_status tk_tq_open(const char *path, tk_tq **out);
void tk_tq_close(tk_tq *tq);
int tk_tq_count(const tk_tq *tq);
int tk_tq_find(const tk_tq *tq, const char *name);          /* index, or -1 */
tk_status tk_tq_entry(const tk_tq *tq, int i, const char **name, int *qtype, int *rows, int *cols,
                      uint64_t *offset, uint64_t *bytes, double *err);
tk_status tk_tq_read(const tk_tq *tq, int i, void *dst, int dst_on_device, void *stream);
/* Writer: the layout of quant_main (tier/tier.cpp:2698-2746) and write_tq
 * (tier/quant.py:60-105): data[i] (host or device pointers) with the header
 * above; `meta` holds "#key value" lines (nullable); errs nullable (writes -1).
 * Writes <path>.part, then renames it to <path>. */
tk_status tk_tq_write(const char *path, int n, const char *const *names, const int *qtypes,
                      const int *rows, const int *cols, const void *const *data, const double *errs,
                      const char *meta);
/* Type names of the format (tier/quant.h:25-31): "Q4_K" <-> TK_Q4_K etc.;
 * -1 / NULL when unknown. */
int tk_qtype_from_name(const char *name);
const char *tk_qtype_name(int qtype);

/* ---- decode GEMV (M = 1..16) -------------------------------------------- */
/* y[m, n] = sum_k W(n, k) * x[m, k] for m < M, n < N, fp32 x and y.
 * qtype: any type tk_dequant takes (the reference's gemv_q decodes every type
 * through q_val; Q8_0 / Q4_K / Q5_K / Q6_K have the fast kernels),
 * optionally OR TK_WFROZEN: the caller guarantees that no kernel enqueued
 * earlier on the stream writes W (frozen weights), so the Q8_0 / Q4_K / Q5_K
 * kernel may start fetching W before the preceding kernel has finished
 * (x is still read only after it); without the flag nothing is read early.
 * For 3..16 tokens with a Q8_0 / Q4_K / Q5_K weight, x is first turned into
 * per-chunk records in the context workspace (calls on one context are
 * stream-ordered, as for the linear entry points).
 * Replaces gemv_q (tier/tier.cpp:300-306) and gemv<T> (tier/tier.cpp:2261-2268)
 * as dispatched by chat_lin (tier/tier.cpp:2351-2378). */
tk_status tk_gemv(tk_ctx *ctx, int qtype, const void *W, size_t row_bytes, int N, int K,
                  const float *x, int ldx, int M, float *y, int ldy, void *stream);
/* Several frozen weights that share one x, in one launch (no counterpart in
 * the reference, which calls gemv_q once per projection): for i < nseg,
 * y_i[m, n] = sum_k W_i(n, k) x[m, k], n < rows[i], with y_i at y[i] and row
 * stride ldy[i].  All W_i have the same qtype (TK_WFROZEN may be OR-ed in),
 * K and row_bytes -- a decoder layer's q/k/v, or gate/up.  x is staged once
 * and the per-launch fixed cost is paid once.  With 1-2 tokens and a Q8_0 /
 * Q4_K / Q5_K / Q6_K weight the rows run in one integer-MMA launch; otherwise
 * each W_i goes through tk_gemv in turn (same results). */
enum { TK_GEMV_MAXSEG = 4 };
tk_status tk_gemv_multi(tk_ctx *ctx, int qtype, int nseg, const void *const *W, const int *rows,
                        float *const *y, const int *ldy, size_t row_bytes, int K, const float *x,
                        int ldx, int M, void *stream);

/* ---- linear layers (tensor cores) --------------------------------------- */
/* Y[M, N] = X[M, K] . W^T (+ Y if beta == 1).  X dtype per x_dtype with row
 * stride ldx (elements); Y fp32 with row stride ldy.  Block-quantized W is
 * dequantized bit-exactly to fp16 first (as the reference's training path,
 * tier/tier.cpp:513-518), then multiplied on tcgen05 tensor cores with fp32
 * accumulation.  Replaces linear / low3_linear (tier/tier.cpp:1186-1216). */
tk_status tk_linear_fwd(tk_ctx *ctx, const tk_weight *W, const void *X, int x_dtype, int M,
                        int ldx, float *Y, int ldy, float beta, int products, void *stream);

/* dX[M, K] = dY[M, N] . W (+ dX if beta == 1).  Replaces linear_dx and
 * linear_dx_acc (tier/tier.cpp:1217-1238). */
tk_status tk_linear_dx(tk_ctx *ctx, const tk_weight *W, const void *dY, int dy_dtype, int M,
                       int lddy, float *dX, int lddx, float beta, int products, void *stream);

/* Y[Mx, N] = X . W^T and dX[Md, K] = dY . W (beta = 0) for one weight in
 * one call: the training step's forward and input gradient, as
 * tk_linear_fwd followed by tk_linear_dx.  W is expanded once, and both
 * GEMMs run in one persistent tensor-core launch whose tiles interleave, so
 * that neither GEMM's last wave of tiles leaves SMs idle.  This call never
 * splits K: Y and dX equal tk_linear_fwd's and tk_linear_dx's bit for bit
 * wherever those run one K split (always for a reduction length below 2048)
 * and are within the product set's tolerance elsewhere.  With Mx or Md <= 128, or TK_QFUSED, the two operations run
 * one after the other.  No counterpart in the reference, whose training step
 * calls linear and linear_dx at different points (tier/tier.cpp:1186-1238). */
tk_status tk_linear_fwd_dx(tk_ctx *ctx, const tk_weight *W, const void *X, int x_dtype, int Mx, int ldx,
                           float *Y, int ldy, const void *dY, int dy_dtype, int Md, int lddy, float *dX,
                           int lddx, int products, void *stream);

/* tk_linear_fwd for callers that cannot allocate device memory -- an engine
 * that budgets all VRAM through its own arena, or code that must not call
 * cudaMalloc once running.  No counterpart in the reference.  Same arguments
 * as tk_linear_fwd, restricted to TK_F16 / TK_F16X2 weights (TK_QFUSED and
 * TK_WREUSE are ignored); it calls no cudaMalloc/cudaFree and never touches
 * the context workspace.  It never splits K, so its result equals
 * tk_linear_fwd's bit for bit wherever tk_linear_fwd runs one K split (always
 * for K < 2048) and within the product set's tolerance elsewhere.  Its
 * scratch is a static 24 MiB device array inside libtierk.so (held on every
 * GPU that loads the library until exit): 2 * parts * M * round8(K) + 4 * M
 * bytes (each term rounded up to 256) must fit, else TK_ERR_INVALID.  The
 * first call on a device looks up the array's address; make it before any
 * stream capture.  Calls on one device share the array, so calls whose GPU
 * work overlaps race: order them on one stream. */
tk_status tk_linear_fwd_noalloc(tk_ctx *ctx, const tk_weight *W, const void *X, int x_dtype, int M,
                                int ldx, float *Y, int ldy, float beta, int products, void *stream);

/* Split an fp32 weight into the TK_F16X2 planes: planes[0 .. rows*cols) = hi,
 * planes[rows*cols .. 2*rows*cols) = lo, both W * 2^s with s chosen so that
 * max|W| * 2^s lies in [2^14, 2^15).  *scale_log2 receives s (written after the
 * stream work completes; the call synchronizes `stream`).  New in this
 * library: the reference keeps one fp16 copy of W (tier/tier.cpp:2507-2512). */
tk_status tk_weight_split_f32(tk_ctx *ctx, const float *W32, int rows, int cols, uint16_t *planes,
                              int *scale_log2, void *stream);

/* h = f16(x), m = f16(x - h), l = f16((x - h) - m) elementwise, unscaled --
 * exactly split3_fp_k (tier/tier.cpp:869-870). */
tk_status tk_split3(tk_ctx *ctx, const float *x, size_t n, uint16_t *h, uint16_t *m, uint16_t *l,
                    void *stream);

/* ---- dX reduce-scatter over peer memory (multi-GPU, one process per GPU) -- */
/* With W split by output rows over `world` GPUs, dX = sum_g dY_g . W_g.  A
 * consumer that takes dX split by token rows (rank r: rows r*M/world ..
 * (r+1)*M/world) needs a reduce-scatter.  tk_linear_dx_rs does it inside the
 * dX GEMM: every finished tile is stored into its owner's receive buffer
 * (peer memory over NVLink) while the remaining tiles compute; the owner adds
 * the world contributions in rank order (deterministic).  No counterpart in
 * the reference (it runs on one GPU; sharding W by output rows is new here).
 *
 * Set-up, once per context: tk_comm_init allocates this rank's buffer
 * (4 KiB + 2 * recv_bytes; recv_bytes >= M * K * 4 for every later call) and
 * writes its CUDA IPC handle (TK_IPC_HANDLE_BYTES) to handle_out; the caller
 * exchanges the handles (e.g. an all-gather), passes all `world` of them in
 * rank order to tk_comm_connect, then runs a barrier across the ranks.
 * Every rank must make the same sequence of tk_linear_dx_rs calls. */
enum { TK_IPC_HANDLE_BYTES = 64 };
tk_status tk_comm_init(tk_ctx *ctx, int rank, int world, size_t recv_bytes, void *handle_out);
tk_status tk_comm_connect(tk_ctx *ctx, const void *handles);
/* dX_rows[M/world, ldd] = rows rank*M/world .. of sum over ranks of dY.W, dY
 * [M, W->rows] (this rank's columns), as tk_linear_dx with beta = 0.
 * M / world must be a multiple of 256.  Bounded device waits (2 s) report
 * TK_ERR_TIMEOUT through tk_sync_status if a rank does not take part. */
tk_status tk_linear_dx_rs(tk_ctx *ctx, const tk_weight *W, const void *dY, int dy_dtype, int M, int lddy,
                          float *dX_rows, int ldd, int products, void *stream);
/* tk_linear_fwd_dx with the dX half reduce-scattered as tk_linear_dx_rs:
 * Y[Mx, W->rows] = X . W^T (this rank's columns) and dX_rows[Md/world, ldd]
 * = this rank's token rows of sum over ranks of dY . W, in one launch whose
 * forward tiles compute while the dX tiles' stores cross NVLink.  Same
 * results as tk_linear_fwd then tk_linear_dx_rs, bit for bit. */
tk_status tk_linear_fwd_dx_rs(tk_ctx *ctx, const tk_weight *W, const void *X, int x_dtype, int Mx, int ldx,
                              float *Y, int ldy, const void *dY, int dy_dtype, int Md, int lddy,
                              float *dX_rows, int ldd, int products, void *stream);

/* Collectives of the sharded path on the same peer buffers (stores over
 * NVLink, no NCCL), so that a C or C++ caller -- the reference's engine is
 * one -- can shard without another communication library.  No counterpart in
 * the reference (it runs on one GPU).  Every rank makes the same sequence of
 * these and tk_linear_dx_rs calls; a rank that does not take part makes the
 * others' bounded waits (2 s) report TK_ERR_TIMEOUT through tk_sync_status.
 * Sizes and pointers 16-byte aligned; world * bytes <= recv_bytes of
 * tk_comm_init. */
/* dst[world * bytes] = every rank's src[bytes], in rank order: the all-gather
 * of output shards (a row-split linear's Y columns, a decode GEMV's y). */
tk_status tk_allgather(tk_ctx *ctx, const void *src, size_t bytes, void *dst, void *stream);
/* Column shards to row shards (an all-to-all): rank g holds A[M, n] = columns
 * g*n .. (g+1)*n of a [M, world*n] matrix (row stride ld_src elements of
 * elem_bytes); afterwards dst[M/world, world*n] (row stride ld_dst) holds rows
 * g*M/world .. (g+1)*M/world of the whole matrix.  Every rank passes the same
 * M and n; M % world == 0; n * elem_bytes % 16 == 0.  Used for dX of a
 * row-split linear: moving dY (bf16, M*N*2*(world-1)/world^2 bytes out per
 * rank) instead of the fp32 partial sums of dX (M*K*4*(world-1)/world). */
tk_status tk_reshard_cols(tk_ctx *ctx, const void *src, int M, int n, size_t ld_src, int elem_bytes,
                          void *dst, size_t ld_dst, void *stream);
/* The same in two halves, so that the transfer overlaps other work: _send
 * pushes this rank's blocks to their owners (stream-ordered after src is
 * ready; it can run beside a GEMM on another stream), _recv (later, any
 * stream ordered after _send) waits for every rank's blocks and assembles
 * dst.  One exchange is open per context at a time. */
tk_status tk_reshard_cols_send(tk_ctx *ctx, const void *src, int M, int n, size_t ld_src, int elem_bytes,
                               void *stream);
tk_status tk_reshard_cols_recv(tk_ctx *ctx, void *dst, size_t ld_dst, int elem_bytes, void *stream);
/* buf[i] = sum over ranks of buf[i] (n % 4 == 0), added in rank order so that
 * every rank holds the same bits: the LM head's dX over vocabulary shards. */
tk_status tk_allreduce_f32(tk_ctx *ctx, float *buf, size_t n, void *stream);
/* Vocabulary-shard merge of the LM head's running state, rank r holding the
 * r-th vocabulary range: afterwards every rank holds the state of the whole
 * vocabulary -- rmax = max over ranks; rsum = sum over ranks (rank order) of
 * rsum_r * exp(rmax_r - rmax); amax = the argmax of the first rank whose
 * rmax_r equals rmax (lowest vocabulary index on ties, as the reference);
 * tgt = sum of tgt_r -- and rows t < n of the single-pass accumulator dX
 * [n, H] (nullable) are scaled by exp(rmax_local - rmax), as
 * tk_lmhead_rescale does.  The step between pass 1 (or tk_lmhead_fused) and
 * tk_lmhead_loss / tk_lmhead_grad / tk_lmhead_finish. */
tk_status tk_lmhead_merge(tk_ctx *ctx, int n, double *rmax, double *rsum, int32_t *amax, float *tgt,
                          float *dX, int H, void *stream);

/* ---- LM head + cross-entropy over a vocabulary shard --------------------- */
/* The reference runs two passes over vocab chunks (tier/tier.cpp:3184-3266).
 * W: fp16 [V_shard, H] rows v0 .. v0+V_shard of the full head; X: fp32 [T, H]
 * (final normed hidden); labels: int32 [T] (row t predicts labels[t+1]);
 * mask: uint8 [T] (loss mask, row T-1 never predicts).  softcap > 0 applies
 * cap*tanh(l/cap).  `chunk` = vocab rows per chunk (multiple of 256).
 * `products`: TK_X3_REF (3 parts of X and of dlogit) or TK_X2 (2 parts).
 *
 * Pass 1 merges this shard's logits into the running state, in vocabulary
 * order: rmax/rsum (fp64, init -1e30 / 0), amax (init -1) and tgt (init 0),
 * each [T-1].  Replaces the lse_chunk_kernel loop (tier/tier.cpp:3209-3222,
 * 750-759). */
tk_status tk_lmhead_stats(tk_ctx *ctx, const uint16_t *W, int v0, int V_shard, int H,
                          const float *X, int T, const int32_t *labels, const uint8_t *mask,
                          float softcap, int chunk, int products, double *rmax, double *rsum,
                          int32_t *amax, float *tgt, void *stream);

/* Pass 2: dX[T, H] += sum_v dlogit[t, v] * W[v, :] with dlogit as
 * dlogit_kernel (tier/tier.cpp:736-748) from the FINAL (all-shard) rmax/rsum.
 * n_loss = number of rows with mask != 0 among rows 0..T-2.
 * Replaces the pass-2 loop (tier/tier.cpp:3247-3266). */
tk_status tk_lmhead_grad(tk_ctx *ctx, const uint16_t *W, int v0, int V_shard, int H,
                         const float *X, int T, const int32_t *labels, const uint8_t *mask,
                         int n_loss, float softcap, int chunk, int products, const double *rmax,
                         const double *rsum, float *dX, void *stream);

/* Single pass (one logits GEMM per chunk, where the reference's two passes
 * need two): runs pass 1 exactly as tk_lmhead_stats (same rmax/rsum/amax/tgt
 * updates) and accumulates, in dX [T, H] (overwritten; rows >= T-1 or
 * masked stay 0), the UNNORMALISED sum_v exp(l[t,v] - rmax[t]) g(l) W[v, :]
 * with g(l) = 1 - (l/softcap)^2 (1 without softcap), rescaled chunk by chunk
 * to the running max.  The probabilities go to the GEMM as fp16 hi + lo
 * (about 2^-22 relative).  tk_lmhead_finish turns dX into the gradient.
 * No counterpart in the reference (tier/tier.cpp:3184-3266 recomputes the
 * logits in pass 2). */
tk_status tk_lmhead_fused(tk_ctx *ctx, const uint16_t *W, int v0, int V_shard, int H,
                          const float *X, int T, const int32_t *labels, const uint8_t *mask,
                          float softcap, int chunk, int products, double *rmax, double *rsum,
                          int32_t *amax, float *tgt, float *dX, void *stream);

/* dX[t] = dX[t] / (n_loss * rsum[t]) - g(tgt[t]) * W[labels[t+1] - v0] / n_loss
 * (the W term only when the label lies in this shard) for rows with loss,
 * 0 for the rest: the dlogit of tier/tier.cpp:736-748 summed against W.
 * rsum must be the final (all-shard) sum relative to the final max. */
tk_status tk_lmhead_finish(tk_ctx *ctx, const uint16_t *W, int v0, int V_shard, int H, int T,
                           const int32_t *labels, const uint8_t *mask, int n_loss, float softcap,
                           const double *rsum, const float *tgt, float *dX, void *stream);

/* loss_sum = sum over masked rows t < T-1 of (rmax + log(rsum) - tgt);
 * hits = count of amax[t] == labels[t+1] (tier/tier.cpp:3227-3228).
 * Writes one double and one int to device memory. */
tk_status tk_lmhead_loss(tk_ctx *ctx, int T, const int32_t *labels, const uint8_t *mask,
                         const double *rmax, const double *rsum, const int32_t *amax,
                         const float *tgt, double *loss_sum, int32_t *hits, void *stream);

/* Vocabulary chunk for the LM head: the reference's lm_chunk rule
 * (tier/tier.cpp:2015-2017) -- device_bytes / 36 / (6*hidden + 8*max(seq,1))
 * rows, clamped to [1024, vocab rounded up] -- rounded down to a multiple of
 * 256 (the reference rounds to 128; these kernels take 256-row tiles).
 * device_bytes = 0 (memory not known) gives 8192, as the reference.  Host
 * only, no context. */
int tk_lmhead_chunk(size_t device_bytes, int hidden, int seq, int vocab);

/* Vocab-sharded merge helper: rsum *= exp(rmax_local - rmax_global) and
 * rmax_local = rmax_global, for rows t < n (run between an all-reduce MAX of
 * rmax and an all-reduce SUM of rsum); with dX (nullable, [n, H]) the
 * single-pass accumulator rows are scaled by the same factor. */
tk_status tk_lmhead_rescale(tk_ctx *ctx, int n, double *rmax_local, double *rsum_local,
                            const double *rmax_global, float *dX, int H, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* TIERK_H */
