// tk_gemm_q.cu -- tensor-core GEMM with the block dequant fused into the
// producer side: the quantized weight never exists in HBM as fp16.
//
//   forward  Y[M, N]  = X[M, K] . W^T       (W[N, K] rows of quant blocks)
//   input-gradient dX[M, K] = dY[M, N] . W
//
// The reference expands the whole weight to fp16 in HBM before every GEMM
// (tier/tier.cpp:513-518) and then runs fp3gemm (tier/tier.cpp:922-943).
// Here each CTA pair (cluster of 2, tcgen05.mma.cta_group::2, 256 x 256
// tiles) streams the raw blocks into shared memory with TMA and eight
// converter warps decode them -- bit-exactly, tier_fp16(q_val) -- straight
// into the 128-byte-swizzled fp16 operand layout the MMA reads (K-major for
// the forward, N-major for dX).
//
// Warp roles (480 threads, one CTA per SM):
//   0       TMA producer of the activation planes (A, 128 rows x 64 per stage)
//   1       TMEM allocation; the leader CTA's lane 0 issues the MMAs
//   2-5     epilogue (TMEM -> registers -> fp32 D, scale, optional beta)
//   6       TMA producer of raw quant slabs
//   7-14    converters: quant slab -> fp16 B stage (128 x 64 per CTA)
// Barriers: A full/empty, quant full/empty, B full/empty (B full lives in the
// leader and counts the converter warps of both CTAs), TMEM full/empty.
// Every wait is bounded (tk_device.cuh).
#include <cuda.h>
#include <cuda_runtime.h>
#include <mutex>
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {
namespace gq {

constexpr int BM = 128, BN = 256, BK = 64, NB = BN / 2;
constexpr int SA = 4, SB = 4, SQ = 2;
constexpr int A_BYTES = BM * BK * 2;          // 16 KB
constexpr int B_BYTES = NB * BK * 2;          // 16 KB
constexpr int Q_SLOT = 128 * 272;             // largest slab: 128 rows x 272 B (Q8_0, 256 columns)
constexpr int CONV_WARPS = 8;
constexpr int THREADS = (7 + CONV_WARPS) * 32;
constexpr int TMEM_COLS = 512;
constexpr size_t SMEM = (size_t)SA * A_BYTES + (size_t)SB * B_BYTES + (size_t)SQ * Q_SLOT + 1024 + 512;

// Quant slab geometry: a slab holds whole super-blocks (256 columns of W).
template <int T> struct QG;
template <> struct QG<QT_Q4_K> { static constexpr int SBB = 144; };
template <> struct QG<QT_Q5_K> { static constexpr int SBB = 176; };
template <> struct QG<QT_Q8_0> { static constexpr int SBB = 272; };   // 8 blocks of 34 B

struct __align__(64) Params {
    CUtensorMap tmA[3];
    CUtensorMap tmQ;       // raw bytes [W rows][row_bytes/16][16], box {16, SBB/16, 128 (fwd) or 64 (dX) rows}
    int M, N, K;           // GEMM dims
    int nprod;             // activation planes (each multiplied by the same dequantized W)
    int pa[3];
    int tiles_m, tiles_n;
    int seg_kb;
    float* D;
    long ldd;
    int beta;
    const int* row_exp;
    int* status;
};

// Convert this thread's 32 weights to fp16 and store them in the B stage.
//   fwd (K-major stage [128 N-rows][64 K]):  thread -> W row r = t & 127,
//       half h = t >> 7 of the 64-wide k-block (a 32-element sub-block).
//   dX (N-major stage, two [64 K-rows][64 N] atoms): thread -> W row
//       r = t & 63 (a k index), quarter cq = t >> 6 of the CTA's 128 columns.
template <int T, bool DX>
__device__ __forceinline__ void convert32(const uint8_t* __restrict__ qslot, uint8_t* __restrict__ bst, int ct,
                                          int g /*k-block within slab (fwd)*/, int rank) {
    constexpr int SBB = QG<T>::SBB;
    int r, sub;                       // slab row, 32-element sub-block within the 256-wide slab
    if constexpr (!DX) { r = ct & 127; sub = 2 * g + (ct >> 7); }
    else { r = ct & 63; sub = 4 * rank + (ct >> 6); }
    uint32_t h16[16];                 // 32 fp16 values, packed pairs
    sub32_to_f16<T>(qslot + (size_t)r * SBB, sub, h16);
    // store: four 16-byte chunks of 8 fp16, 128-byte swizzle (chunk ^ row%8)
    if constexpr (!DX) {
        const int h = ct >> 7;
        uint8_t* base = bst + (size_t)r * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int phys = (h * 4 + c) ^ (r & 7);
            *reinterpret_cast<uint4*>(base + phys * 16) = make_uint4(h16[4 * c], h16[4 * c + 1], h16[4 * c + 2], h16[4 * c + 3]);
        }
    } else {
        const int cq = ct >> 6;
        uint8_t* base = bst + (size_t)(cq >> 1) * (64 * 64 * 2) + (size_t)r * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int phys = (4 * (cq & 1) + c) ^ (r & 7);
            *reinterpret_cast<uint4*>(base + phys * 16) = make_uint4(h16[4 * c], h16[4 * c + 1], h16[4 * c + 2], h16[4 * c + 3]);
        }
    }
}

template <int T, bool DX>
__global__ void __launch_bounds__(THREADS, 1) gemm_q_kernel(const __grid_constant__ Params p) {
    constexpr int SBB = QG<T>::SBB;
    constexpr int KB_PER_SLAB = DX ? 1 : 4;         // fwd: a slab covers 4 k-blocks (256 columns)
    constexpr int Q_ROWS = DX ? BK : NB;
    constexpr uint32_t Q_TX = (uint32_t)Q_ROWS * SBB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + SA * A_BYTES;
    uint8_t* sQ = sB + SB * B_BYTES;
    uint64_t* fa = reinterpret_cast<uint64_t*>(sQ + SQ * Q_SLOT);
    uint64_t* ea = fa + SA;
    uint64_t* fb = ea + SA;
    uint64_t* eb = fb + SB;
    uint64_t* fq = eb + SB;
    uint64_t* eq = fq + SQ;
    uint64_t* tfull = eq + SQ;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; ++s) { mbar_init(&fa[s], 1); mbar_init(&ea[s], 1); }
        for (int s = 0; s < SB; ++s) { mbar_init(&fb[s], 2 * CONV_WARPS); mbar_init(&eb[s], 1); }
        for (int s = 0; s < SQ; ++s) { mbar_init(&fq[s], 1); mbar_init(&eq[s], CONV_WARPS); }
        for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], 8); }
        fence_mbar_init();
        fence_async_shared();
    }
    if (warp == 1) {
        tmem_alloc_cg2(tmem_slot, TMEM_COLS);
        tmem_relinquish_cg2();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int num_tiles = p.tiles_m * p.tiles_n;
    const int kblocks = (p.K + BK - 1) / BK;

    if (warp == 0) {
        // ---------------- activation planes (TMA; both CTAs signal the leader) ----------------
        if (lane == 0) {
            int ia = 0;
            bool ok = true;
            for (int tile = cid; tile < num_tiles && ok; tile += ncl) {
                const int mb = tile % p.tiles_m;
                const int arow = (mb * 2 + (int)rank) * BM;
                for (int kb = 0; kb < kblocks && ok; ++kb)
                    for (int q = 0; q < p.nprod; ++q, ++ia) {
                        const int s = ia % SA;
                        if (!mbar_wait(&ea[s], ((ia / SA) & 1) ^ 1, p.status)) { ok = false; break; }
                        if (rank == 0) mbar_arrive_expect_tx(&fa[s], 2 * A_BYTES);
                        tma_load_2d_cg2(sA + s * A_BYTES, &p.tmA[p.pa[q]], mapa_shared(smem_u32(&fa[s]), 0), kb * BK,
                                        arow);
                    }
            }
        }
        __syncwarp();
    } else if (warp == 6) {
        // ---------------- raw quant slabs (TMA, local) ----------------
        if (lane == 0) {
            int iq = 0;
            bool ok = true;
            for (int tile = cid; tile < num_tiles && ok; tile += ncl) {
                const int nb = tile / p.tiles_m;
                for (int kb = 0; kb < kblocks && ok; kb += KB_PER_SLAB, ++iq) {
                    const int s = iq % SQ;
                    if (!mbar_wait(&eq[s], ((iq / SQ) & 1) ^ 1, p.status)) { ok = false; break; }
                    mbar_arrive_expect_tx(&fq[s], Q_TX);
                    // fwd: W rows of this CTA's 128 output columns, super-block kb/4;
                    // dX: W rows kb*64.., super-block column nb (the pair's 256 columns).
                    const int x = DX ? nb * (SBB / 16) : (kb / 4) * (SBB / 16);   // in 16-byte units
                    const int y = DX ? kb * BK : nb * BN + (int)rank * NB;
                    tma_load_3d(sQ + s * Q_SLOT, &p.tmQ, &fq[s], 0, x, y);
                }
            }
        }
        __syncwarp();
    } else if (warp >= 7) {
        // ---------------- converters ----------------
        const int ct = threadIdx.x - 7 * 32;
        int ib = 0, iq = 0;
        bool ok = true;
        for (int tile = cid; tile < num_tiles && ok; tile += ncl) {
            for (int kb = 0; kb < kblocks && ok; ++kb, ++ib) {
                const int qs = iq % SQ;
                if (kb % KB_PER_SLAB == 0 && !mbar_wait(&fq[qs], (iq / SQ) & 1, p.status)) { ok = false; break; }
                const int bs = ib % SB;
                if (!mbar_wait(&eb[bs], ((ib / SB) & 1) ^ 1, p.status)) { ok = false; break; }
                convert32<T, DX>(sQ + qs * Q_SLOT, sB + bs * B_BYTES, ct, kb % 4, (int)rank);
                fence_async_shared();      // generic stores -> visible to the tensor core's async reads
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&fb[bs]), 0));
                if (kb % KB_PER_SLAB == KB_PER_SLAB - 1 || kb == kblocks - 1) {
                    if (lane == 0) mbar_arrive(&eq[qs]);
                    ++iq;
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader) ----------------
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_f16(BM * 2, BN, 0, 0, DX ? 1 : 0);
            int ia = 0, ib = 0, u = 0;
            bool ok = true;
            for (int tile = cid; tile < num_tiles && ok; tile += ncl) {
                for (int kb0 = 0; kb0 < kblocks && ok; kb0 += p.seg_kb, ++u) {
                    const int kb1 = kb0 + p.seg_kb < kblocks ? kb0 + p.seg_kb : kblocks;
                    const int acc = u & 1;
                    if (!mbar_wait(&tempty[acc], ((u >> 1) & 1) ^ 1, p.status)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * BN;
                    bool first = true;
                    for (int kb = kb0; kb < kb1 && ok; ++kb, ++ib) {
                        const int bs = ib % SB;
                        if (!mbar_wait(&fb[bs], (ib / SB) & 1, p.status)) { ok = false; break; }
                        const uint32_t b0 = smem_u32(sB + bs * B_BYTES);
                        for (int q = 0; q < p.nprod; ++q, ++ia) {
                            const int s = ia % SA;
                            if (!mbar_wait(&fa[s], (ia / SA) & 1, p.status)) { ok = false; break; }
                            tc_fence_after();
                            const uint32_t a0 = smem_u32(sA + s * A_BYTES);
#pragma unroll
                            for (int kk = 0; kk < BK / 16; ++kk) {
                                const uint64_t ad = sdesc_sw128(a0 + kk * 32, 16, 1024);
                                const uint64_t bd = DX ? sdesc_sw128(b0 + kk * 2048, 64 * BK * 2, 1024)
                                                       : sdesc_sw128(b0 + kk * 32, 16, 1024);
                                tc_mma_f16_cg2(d_tmem, ad, bd, idesc, first ? 0u : 1u);
                                first = false;
                            }
                            const uint32_t e = smem_u32(&ea[s]);
                            tc_commit_cg2(mapa_shared(e, 0));
                            tc_commit_cg2(mapa_shared(e, 1));
                        }
                        const uint32_t e = smem_u32(&eb[bs]);
                        tc_commit_cg2(mapa_shared(e, 0));
                        tc_commit_cg2(mapa_shared(e, 1));
                    }
                    if (ok) {
                        const uint32_t f = smem_u32(&tfull[acc]);
                        tc_commit_cg2(mapa_shared(f, 0));
                        tc_commit_cg2(mapa_shared(f, 1));
                    }
                }
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int quarter = warp & 3;
        int u = 0;
        bool ok = true;
        for (int tile = cid; tile < num_tiles && ok; tile += ncl) {
            const int mb = tile % p.tiles_m, nb = tile / p.tiles_m;
            for (int kb0 = 0; kb0 < kblocks; kb0 += p.seg_kb, ++u) {
                const int acc = u & 1;
                if (!mbar_wait(&tfull[acc], (u >> 1) & 1, p.status)) { ok = false; break; }
                tc_fence_after();
                const bool add_prev = kb0 > 0 || p.beta;
                const int row = (mb * 2 + (int)rank) * BM + quarter * 32 + lane;
                const bool row_ok = row < p.M;
                const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
                const float f = ldexpf(1.0f, -(p.row_exp && row_ok ? p.row_exp[row] : 0));
                float* drow = p.D + (size_t)(row_ok ? row : 0) * p.ldd;
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    const int col0 = nb * BN + c;
                    const bool full_chunk = row_ok && col0 + 32 <= p.N;
                    // earlier partial sums are read before the TMEM read and before any
                    // store, so the loads overlap instead of queueing behind stores
                    float4 od[8];
                    if (full_chunk && add_prev) {
#pragma unroll
                        for (int q = 0; q < 8; ++q) od[q] = reinterpret_cast<const float4*>(drow + col0)[q];
                    }
                    uint32_t r[32];
                    tc_ld_32x32b_x32(taddr + c, r);
                    tc_wait_ld();
                    if (full_chunk) {
                        float4* dp = reinterpret_cast<float4*>(drow + col0);
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            float4 v = make_float4(__uint_as_float(r[4 * q]) * f, __uint_as_float(r[4 * q + 1]) * f,
                                                   __uint_as_float(r[4 * q + 2]) * f, __uint_as_float(r[4 * q + 3]) * f);
                            if (add_prev) { v.x += od[q].x; v.y += od[q].y; v.z += od[q].z; v.w += od[q].w; }
                            dp[q] = v;
                        }
                    } else if (row_ok) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < p.N) {
                                float v = __uint_as_float(r[j]) * f;
                                if (add_prev) v += drow[col0 + j];
                                drow[col0 + j] = v;
                            }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_cg2(tmem_base, TMEM_COLS);
    }
}

}  // namespace gq

// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFnQ)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnQ encode_q() {
    static EncodeTiledFnQ fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFnQ>(p);
    });
    return fn;
}

bool gemm_q_supported(int qtype) { return qtype == QT_Q4_K || qtype == QT_Q5_K || qtype == QT_Q8_0; }

template <int T, bool DX>
static tk_status go_q(tk_ctx* ctx, const gq::Params& gp, cudaStream_t s) {
    auto kern = gq::gemm_q_kernel<T, DX>;
    static std::atomic<uint64_t> attr_done{0};   // per instantiation, one bit per device
    {
        const cudaError_t e = smem_attr_once(kern, (int)gq::SMEM, ctx->device, attr_done);
        if (e != cudaSuccess) return cuda_fail(e, "gemm_q smem attribute");
    }
    const int tiles = gp.tiles_m * gp.tiles_n;
    const int groups = tiles < ctx->num_sms / 2 ? tiles : ctx->num_sms / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(groups * 2, 1, 1);
    cfg.blockDim = dim3(gq::THREADS, 1, 1);
    cfg.dynamicSmemBytes = gq::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ProfScope ps(ctx, s, PK_GEMM);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, gp);
    ctx->launches++;
    if (e != cudaSuccess) return cuda_fail(e, "gemm_q launch");
    return cuda_fail(cudaGetLastError(), "gemm_q launch");
}

tk_status launch_gemm_q(tk_ctx* ctx, const GemmQDesc& g, cudaStream_t s) {
    EncodeTiledFnQ fn = encode_q();
    if (!fn) return fail(TK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if (g.M <= 128) return fail(TK_ERR_UNSUPPORTED, "fused quant GEMM needs M > 128");
    gq::Params gp;
    memset(&gp, 0, sizeof(gp));
    for (int i = 0; i < 3; ++i) {
        if (!g.A[i]) continue;
        cuuint64_t dims[2] = {(cuuint64_t)g.K, (cuuint64_t)g.M};
        cuuint64_t strides[1] = {(cuuint64_t)g.lda * 2};
        cuuint32_t box[2] = {64, 128};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = fn(&gp.tmA[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(g.A[i]), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(TK_ERR_CUDA, "tensor map (A planes): " + std::to_string((int)r));
    }
    const int sbb = g.qtype == QT_Q4_K ? 144 : g.qtype == QT_Q5_K ? 176 : 272;
    {
        // bytes viewed as [rows][row_bytes/16][16] so a box of whole super-blocks
        // (144, 176 or 272 B) lands densely packed, whatever its width
        if (g.w_row_bytes % 16) return fail(TK_ERR_INVALID, "fused quant GEMM: row bytes must be a multiple of 16");
        cuuint64_t dims[3] = {16, (cuuint64_t)(g.w_row_bytes / 16), (cuuint64_t)g.w_rows};
        cuuint64_t strides[2] = {16, (cuuint64_t)g.w_row_bytes};
        cuuint32_t box[3] = {16, (cuuint32_t)(sbb / 16), (cuuint32_t)(g.dx ? gq::BK : gq::NB)};
        cuuint32_t estr[3] = {1, 1, 1};
        CUresult r = fn(&gp.tmQ, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(g.W), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(TK_ERR_CUDA, "tensor map (quant rows): " + std::to_string((int)r));
    }
    gp.M = g.M; gp.N = g.N; gp.K = g.K;
    gp.nprod = g.nprod;
    for (int i = 0; i < 3; ++i) gp.pa[i] = g.pa[i];
    gp.tiles_m = (g.M + 255) / 256;
    gp.tiles_n = (g.N + 255) / 256;
    const int kblocks = (g.K + 63) / 64;
    gp.seg_kb = g.seg_kb > 0 && g.seg_kb < kblocks ? g.seg_kb : kblocks;
    gp.D = g.D; gp.ldd = g.ldd; gp.beta = g.beta;
    gp.row_exp = g.row_exp;
    gp.status = ctx->status;
    switch (g.qtype) {
        case QT_Q4_K: return g.dx ? go_q<QT_Q4_K, true>(ctx, gp, s) : go_q<QT_Q4_K, false>(ctx, gp, s);
        case QT_Q5_K: return g.dx ? go_q<QT_Q5_K, true>(ctx, gp, s) : go_q<QT_Q5_K, false>(ctx, gp, s);
        case QT_Q8_0: return g.dx ? go_q<QT_Q8_0, true>(ctx, gp, s) : go_q<QT_Q8_0, false>(ctx, gp, s);
        default: return fail(TK_ERR_UNSUPPORTED, "fused quant GEMM: type");
    }
}

}  // namespace tk
