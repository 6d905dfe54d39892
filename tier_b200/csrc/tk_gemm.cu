// tk_gemm.cu -- the tensor-core GEMM of the path (tcgen05 + TMEM + TMA).
//
//   D[M, N] = sum_p A_{pa[p]}[M, K] . B_{pb[p]}^T     (fp16 x fp16 -> fp32)
//
// One kernel serves every product set of the split GEMM: the reference's
// fp3gemm (tier/tier.cpp:922-943) issues three cuBLASLt GEMMs over the
// planes {xl, xm, xh} and re-reads W three times; here all products of one
// output tile accumulate into the same TMEM accumulator inside one launch,
// each k-block stage pairing one A plane with one B plane.
//
// Layout: persistent CTAs (one per SM), 128 x 256 output tiles, BK = 64.
//   warp 0      TMA producer: A tile [128 x 64] and B tile [256 x 64]
//               (K-major, one box) or [64 x 256] (N-major, four 64-wide boxes)
//               per stage, 128-byte swizzle, 4-stage mbarrier ring.
//   warp 1      allocates 512 TMEM columns (two 256-column fp32
//               accumulators), one lane issues tcgen05.mma (M=128, N=256,
//               K=16) and tcgen05.commit to release stages / publish tiles.
//   warps 2-5   epilogue: tcgen05.ld rows of the finished accumulator while
//               the MMA warp fills the other one; scale, optional beta,
//               store (or the LM-head statistics / dlogit epilogues).
// Accumulation segments: the tensor core's fp32 accumulation loses about one
// ulp per MMA step, so a long K (and the x3 product sets, which triple the
// steps) is cut into segments of seg_kb k-blocks.  Segments alternate between
// the two TMEM accumulators and the epilogue sums them into D in fp32 (RNE),
// so the error grows with the segment length, not with K.
// Split-K (long K, few tiles): work units are (tile, split) for 2 splits,
// every first split ordered before every second one.  Split 0 accumulates
// into D, split 1 into a workspace slab; whichever finishes second adds the
// slab into D ("last arrival fixes up", one atomic per warp quarter, no
// waiting), or split 1 adds straight into D when split 0 is already done.
// Every path computes D = fl(P0 + P1), so the result does not depend on the
// order.  No CTA ever waits for another, so the kernel cannot deadlock when
// other kernels (e.g. NCCL) hold some SMs.
// Two problems in one launch (gemm_pair_kernel): the persistent CTAs walk one
// list of units.  While both problems' operands fit in L2 together, the
// second problem's tiles are spread evenly among the first's, so that e.g. a
// forward GEMM's MMAs and an input-gradient GEMM whose epilogue stores over
// NVLink overlap; otherwise the second problem's tiles come first.  Either
// way neither problem's last wave leaves SMs idle and there is one launch
// gap less.  Each problem keeps its own operands, tile width, B layout,
// products and epilogue target; neither splits K.
// All waits are bounded (tk_device.cuh); a timeout records a status code and
// the roles drain out instead of hanging.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cmath>
#include <mutex>
#include <queue>
#include <vector>
#include "tk_device.cuh"
#include "tk_internal.h"

namespace tk {

constexpr int BM = 128, BN = 256, BK = 64;     // BM: accumulator rows per CTA; BN: tile columns
constexpr int TMEM_COLS = 512;
constexpr int GEMM_THREADS = 192;

// Per CTA-group geometry.  CG = 1: one CTA computes a 128 x 256 tile.
// CG = 2: a CTA pair (cluster of 2) computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2; each CTA holds its 128 rows of A, its 128
// columns of B, and its 128 accumulator rows in TMEM.
template <int CG>
struct Geo {
    static constexpr int STAGES = CG == 1 ? 4 : 6;
    static constexpr int B_ROWS = BN / CG;                 // B rows (output columns) per CTA
    static constexpr int A_BYTES = BM * BK * 2;            // 16 KB
    static constexpr int B_BYTES = B_ROWS * BK * 2;        // 32 KB (CG 1) or 16 KB (CG 2)
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    // + per epilogue warp a 32 x 36 fp32 transpose stage (peer stores)
    static constexpr size_t STAGE_T = 4 * 32 * 36 * 4;
    static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + STAGE_T;
};

enum { EPI_STORE = 0, EPI_LSE = 1, EPI_DLOGIT = 2 };

struct __align__(64) GemmParams {
    CUtensorMap tmA[3];
    CUtensorMap tmB[2];
    int M, N, K;
    int nprod;
    int pa[3], pb[3];
    int tiles_m, tiles_n;  // in tiles of (128 * CG) x bn
    int group_m;           // tile order: bands of group_m tile rows, each swept over every tile column
    int bn;                // tile width (output columns): 256, 224, 192 or 128
    int seg_kb;            // k-blocks per accumulation segment (>= 1)
    int splits;            // K splits per tile: 1 or 2 (work unit = tile x split)
    int* flags;            // split arrivals per (tile, CTA half, warp quarter)
    int epoch;             // this launch's flag stamp (flags of older launches are lower)
    float* sws;            // split 1's partial sums [M, sws_ld] (fp32)
    long sws_ld;
    float* D;
    long ldd;
    int beta;
    const int* row_exp;
    const float* row_alpha;   // beta = 1: D = row_alpha[row] * D + A.B (null: alpha 1)
    // reduce-scatter over peer memory (rs_world > 0): the last segment of a
    // tile row goes to the owner rank's receive slot instead of D
    float* rs_dst[TK_MAX_RANKS];     // per owner: its receive slot for this rank (row 0 of the owner's range)
    int* rs_done[TK_MAX_RANKS];      // per owner: done flag for this rank
    int* rs_counter;                 // CTAs finished (local), reset by the last
    int rs_world, rs_rpo, rs_epoch;
    int col_exp;
    int b_mn;              // B is N-major (read where the kernel picks the layout per problem)
    // pair launches (first problem's copy): CTA pair c runs the units
    // sched[sched_off[c] .. sched_off[c + 1]); unit u < tiles of problem 1 is
    // that problem's tile u, the rest are problem 0's tiles u - tiles(1)
    const int* sched;
    const int* sched_off;
    int* status;
};

struct GemmPair {
    GemmParams p[2];
};

struct EpiParams {
    LseDesc lse;
    DlogitDesc dl;
};

__device__ __forceinline__ float exp2i(int e) {   // exact 2^e for e in [-126, 127]
    return __uint_as_float((uint32_t)(e + 127) << 23);
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Output tile t -> (tile row mb, tile column nb).  Tiles run in bands of
// group_m tile rows; inside a band the row index runs fastest.  The tiles in
// flight at once then form a group_m x (groups / group_m) block, so every A
// panel (a tile row's operand over all of K) and every B panel is shared by
// several concurrent tiles, and a band's A panels stay in L2 while it sweeps
// the columns.  group_m = tiles_m is plain row-fastest order.
__device__ __forceinline__ void tile_coords(const GemmParams& p, int tile, int& mb, int& nb) {
    const int per_band = p.group_m * p.tiles_n;
    const int band = tile / per_band;
    const int m0 = band * p.group_m;
    const int gm = p.tiles_m - m0 < p.group_m ? p.tiles_m - m0 : p.group_m;
    const int r = tile - band * per_band;
    mb = m0 + r % gm;
    nb = r / gm;
}

// A work unit: problem, output tile, K split.
struct Unit {
    int prob, tile, sp;
};

template <int NPROB>
__device__ __forceinline__ int num_units_of(const GemmParams* ps) {
    if constexpr (NPROB == 1) return ps[0].tiles_m * ps[0].tiles_n * ps[0].splits;
    else return ps[0].tiles_m * ps[0].tiles_n + ps[1].tiles_m * ps[1].tiles_n;
}

template <int NPROB>
__device__ __forceinline__ Unit unit_of(const GemmParams* ps, int u) {
    Unit r;
    if constexpr (NPROB == 1) {
        const int nt = ps[0].tiles_m * ps[0].tiles_n;
        r.prob = 0;
        r.tile = u % nt;
        r.sp = u / nt;
    } else {
        const int t1 = ps[1].tiles_m * ps[1].tiles_n;
        r.sp = 0;
        if (u < t1) { r.prob = 1; r.tile = u; }
        else { r.prob = 0; r.tile = u - t1; }
    }
    return r;
}

// The units of CTA group `cid`: a stride over all units for one problem, the
// host-built schedule for a pair.
template <int NPROB>
struct UnitRange {
    int i, end, step;
    const int* list;
    __device__ __forceinline__ UnitRange(const GemmParams* ps, int cid, int ncl) {
        if constexpr (NPROB == 1) {
            i = cid; end = num_units_of<1>(ps); step = ncl; list = nullptr;
        } else {
            i = ps[0].sched_off[cid]; end = ps[0].sched_off[cid + 1]; step = 1; list = ps[0].sched;
        }
    }
    __device__ __forceinline__ int unit(int j) const { return NPROB == 1 ? j : list[j]; }
};

// BMODE: 0 B K-major, 1 B N-major, 2 per problem (GemmParams::b_mn).
template <int CG, int BMODE, int EPI, int NPROB>
__device__ __forceinline__ void gemm_body(const GemmParams* ps, const EpiParams* ep) {
    using G = Geo<CG>;
    constexpr int STAGES = G::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * G::A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * G::B_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    float* tstage = reinterpret_cast<float*>(sB + STAGES * G::B_BYTES + 256);   // 16-byte aligned

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = CG == 2 ? cluster_ctarank() : 0;
    const int cid = blockIdx.x / CG, ncl = gridDim.x / CG;      // tile-group index / count
    int* const status = ps[0].status;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], CG == 1 ? 128 : 8);   // CG 2: one arrival per epilogue warp of both CTAs
        }
        fence_mbar_init();
        fence_async_shared();
    }
    if (warp == 0 && lane == 0) {
        for (int j = 0; j < NPROB; ++j) {
            for (int i = 0; i < ps[j].nprod; ++i) tma_prefetch_desc(&ps[j].tmA[ps[j].pa[i]]);
            tma_prefetch_desc(&ps[j].tmB[0]);
        }
    }
    if (warp == 1) {
        if constexpr (CG == 2) {
            tmem_alloc_cg2(tmem_slot, TMEM_COLS);
            tmem_relinquish_cg2();
        } else {
            tmem_alloc(tmem_slot, TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync();   // peer barriers initialised before any remote signal
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // launched as a programmatic dependent: the set-up above overlapped the
    // previous kernel; its outputs (the operand planes) are read from here on
    pdl_wait();

    if (warp == 0) {
        // ---------------- TMA producer (each CTA loads its own operands) ----------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            const UnitRange<NPROB> ur(ps, cid, ncl);
            for (int j = ur.i; j < ur.end && ok; j += ur.step) {
                const Unit un = unit_of<NPROB>(ps, ur.unit(j));
                const GemmParams& p = ps[un.prob];
                const bool bmn = BMODE == 2 ? p.b_mn != 0 : BMODE == 1;
                const int kblocks = (p.K + BK - 1) / BK;
                const int kb_per_split = (kblocks + p.splits - 1) / p.splits;
                int mb, nb;
                tile_coords(p, un.tile, mb, nb);
                const int arow = (mb * CG + (int)rank) * BM;
                const int brows = p.bn / CG;                          // B rows this CTA loads
                const int bcol = nb * p.bn + (int)rank * brows;
                const int kbs = un.sp * kb_per_split, kbe = kbs + kb_per_split < kblocks ? kbs + kb_per_split : kblocks;
                for (int kb = kbs; kb < kbe && ok; ++kb) {
                    for (int q = 0; q < p.nprod; ++q) {
                        if (!mbar_wait(&empty[s], ph ^ 1, status)) { ok = false; break; }
                        uint8_t* a_dst = sA + s * G::A_BYTES;
                        uint8_t* b_dst = sB + s * G::B_BYTES;
                        const void* ma = &p.tmA[p.pa[q]];
                        const void* mbm = &p.tmB[p.pb[q]];
                        const uint32_t stage_tx = (uint32_t)(G::A_BYTES + brows * BK * 2);
                        if constexpr (CG == 1) {
                            mbar_arrive_expect_tx(&full[s], stage_tx);
                            tma_load_2d(a_dst, ma, &full[s], kb * BK, arow);
                            if (!bmn) {
                                tma_load_2d(b_dst, mbm, &full[s], kb * BK, bcol);
                            } else {
                                for (int j = 0; j < brows / 64; ++j)
                                    tma_load_2d(b_dst + j * (64 * BK * 2), mbm, &full[s], bcol + 64 * j, kb * BK);
                            }
                        } else {
                            // both CTAs' loads complete on the leader's barrier
                            const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
                            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * stage_tx);
                            tma_load_2d_cg2(a_dst, ma, fb, kb * BK, arow);
                            if (!bmn) {
                                tma_load_2d_cg2(b_dst, mbm, fb, kb * BK, bcol);
                            } else {
                                for (int j = 0; j < brows / 64; ++j)
                                    tma_load_2d_cg2(b_dst + j * (64 * BK * 2), mbm, fb, bcol + 64 * j, kb * BK);
                            }
                        }
                        if (++s == STAGES) { s = 0; ph ^= 1; }
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (the leader CTA of a pair) ----------------
        if (lane == 0 && rank == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            int u = 0;   // accumulation units (tile, split, segment) processed
            const UnitRange<NPROB> ur(ps, cid, ncl);
            for (int j = ur.i; j < ur.end && ok; j += ur.step) {
                const Unit un = unit_of<NPROB>(ps, ur.unit(j));
                const GemmParams& p = ps[un.prob];
                const bool bmn = BMODE == 2 ? p.b_mn != 0 : BMODE == 1;
                const uint32_t idesc = idesc_f16(BM * CG, p.bn, 0, 0, bmn ? 1 : 0);
                const int kblocks = (p.K + BK - 1) / BK;
                const int kb_per_split = (kblocks + p.splits - 1) / p.splits;
                const int kbs = un.sp * kb_per_split, kbe = kbs + kb_per_split < kblocks ? kbs + kb_per_split : kblocks;
                const int nprod = p.nprod, seg_kb = p.seg_kb;
                for (int kb0 = kbs; kb0 < kbe && ok; kb0 += seg_kb, ++u) {
                    const int kb1 = kb0 + seg_kb < kbe ? kb0 + seg_kb : kbe;
                    const int acc = u & 1;
                    if (!mbar_wait(&tempty[acc], ((u >> 1) & 1) ^ 1, status)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * 256;
                    const int nst = (kb1 - kb0) * nprod;
                    for (int st = 0; st < nst; ++st) {
                        if (!mbar_wait(&full[s], ph, status)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t a0 = smem_u32(sA + s * G::A_BYTES), b0 = smem_u32(sB + s * G::B_BYTES);
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            const uint64_t ad = sdesc_sw128(a0 + kk * 32, 16, 1024);
                            const uint64_t bd = bmn ? sdesc_sw128(b0 + kk * 2048, 64 * BK * 2, 1024)
                                                    : sdesc_sw128(b0 + kk * 32, 16, 1024);
                            if constexpr (CG == 2) tc_mma_f16_cg2(d_tmem, ad, bd, idesc, (st | kk) ? 1u : 0u);
                            else tc_mma_f16(d_tmem, ad, bd, idesc, (st | kk) ? 1u : 0u);
                        }
                        if constexpr (CG == 2) {
                            const uint32_t e = smem_u32(&empty[s]);
                            tc_commit_cg2(mapa_shared(e, 0));
                            tc_commit_cg2(mapa_shared(e, 1));
                        } else {
                            tc_commit(&empty[s]);
                        }
                        if (++s == STAGES) { s = 0; ph ^= 1; }
                    }
                    if (ok) {
                        if constexpr (CG == 2) {
                            const uint32_t f = smem_u32(&tfull[acc]);
                            tc_commit_cg2(mapa_shared(f, 0));
                            tc_commit_cg2(mapa_shared(f, 1));
                        } else {
                            tc_commit(&tfull[acc]);
                        }
                    }
                }
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int quarter = warp & 3;                 // TMEM lanes this warp may access
        int u = 0;
        bool ok = true;
        const UnitRange<NPROB> ur(ps, cid, ncl);
        for (int j = ur.i; j < ur.end && ok; j += ur.step) {
          const Unit un = unit_of<NPROB>(ps, ur.unit(j));
          const GemmParams& p = ps[un.prob];
          const int tile = un.tile, sp = un.sp;
          int mb, nb;
          tile_coords(p, tile, mb, nb);
          const int kblocks = (p.K + BK - 1) / BK;
          const int kb_per_split = (kblocks + p.splits - 1) / p.splits;
          const int kbs = sp * kb_per_split, kbe = kbs + kb_per_split < kblocks ? kbs + kb_per_split : kblocks;
          // one flag per (tile, CTA half, warp quarter): the same warp quarter of
          // both splits owns the same 32 rows, so warps pair up one to one
          int* flag = p.splits > 1 ? p.flags + ((size_t)tile * CG + rank) * 4 + quarter : nullptr;
          const int arrived = p.epoch * 16 + 1;
          for (int kb0 = kbs; kb0 < kbe; kb0 += p.seg_kb, ++u) {
            const int acc = u & 1;
            const bool w = mbar_wait(&tfull[acc], (u >> 1) & 1, status);
            if (!__all_sync(0xffffffffu, w)) { ok = false; break; }   // warp-uniform exit
            tc_fence_after();
            const int row = (mb * CG + (int)rank) * BM + quarter * 32 + lane;
            const bool row_ok = row < p.M;
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * 256;
            const int e = (p.row_exp && row_ok ? p.row_exp[row] : 0) + p.col_exp;
            const float f = ldexpf(1.0f, -e);
            const int col_base = nb * p.bn;
            if constexpr (EPI == EPI_STORE) {
                const bool last_seg = kb0 + p.seg_kb >= kbe;
                // split 1 on its last segment adds straight into D once split 0
                // has arrived; otherwise it accumulates in the workspace slab
                bool direct = false;
                if (sp > 0 && last_seg) {
                    int v = 0;
                    if (lane == 0) v = ld_acquire_gpu(flag);
                    direct = __shfl_sync(0xffffffffu, v, 0) == arrived;
                }
                float* dst = (sp == 0 || direct) ? p.D : p.sws;
                const long ldst = (sp == 0 || direct) ? p.ldd : p.sws_ld;
                float* drow = dst + (size_t)(row_ok ? row : 0) * ldst;
                // where this segment's result is stored: D, or for the last
                // segment of a reduce-scatter launch the owner's receive slot
                // (peer memory over NVLink); earlier segments stay in D
                float* srow = drow;
                const bool rs_store = p.rs_world && last_seg;
                if (rs_store && row_ok) {
                    const int o = row / p.rs_rpo;
                    srow = p.rs_dst[o] + (size_t)(row - o * p.rs_rpo) * p.ldd;
                }
                // peer stores go through a per-warp transpose so that each store
                // instruction writes whole 128-byte row segments over NVLink
                float4* stg = reinterpret_cast<float4*>(tstage + (size_t)(warp - 2) * 32 * 36);
                const int row_w0 = (mb * CG + (int)rank) * BM + quarter * 32;   // row of lane 0
                const float* wrow = p.sws ? p.sws + (size_t)(row_ok ? row : 0) * p.sws_ld : nullptr;
                // partial of earlier segments of this split: in dst, except for a
                // direct split 1, whose earlier segments sit in the slab
                const bool add_own = kb0 > kbs || (sp == 0 && p.beta);
                const bool own_in_ws = direct && kb0 > kbs;
                // per-row alpha on the caller's D: only where D is read for the
                // first time in this launch (first segment of split 0, beta = 1)
                const float al = (p.row_alpha && row_ok && sp == 0 && kb0 == kbs && p.beta) ? p.row_alpha[row] : 1.0f;
                const bool add_d = add_own || direct;   // direct: D holds split 0's sum
#pragma unroll 1
                for (int c = 0; c < p.bn; c += 32) {
                    const int col0 = col_base + c;
                    const bool full_chunk = row_ok && col0 + 32 <= p.N;
                    const bool t_store = rs_store && col0 + 32 <= p.N;   // warp-uniform
                    // issue this chunk's global reads before the TMEM read and
                    // before any store, so the 8 (or 16) loads overlap instead
                    // of each waiting behind the previous store
                    float4 od[8], ow[8];
                    if (full_chunk && add_d) {
#pragma unroll
                        for (int q = 0; q < 8; ++q) od[q] = reinterpret_cast<const float4*>(drow + col0)[q];
                    }
                    if (full_chunk && own_in_ws) {
#pragma unroll
                        for (int q = 0; q < 8; ++q) ow[q] = reinterpret_cast<const float4*>(wrow + col0)[q];
                    }
                    uint32_t r[32];
                    tc_ld_32x32b_x32(taddr + c, r);
                    tc_wait_ld();
                    if (t_store) {
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            float4 v = make_float4(__uint_as_float(r[4 * q]) * f, __uint_as_float(r[4 * q + 1]) * f,
                                                   __uint_as_float(r[4 * q + 2]) * f, __uint_as_float(r[4 * q + 3]) * f);
                            if (add_d && full_chunk) {
                                v.x = fmaf(al, od[q].x, v.x); v.y = fmaf(al, od[q].y, v.y);
                                v.z = fmaf(al, od[q].z, v.z); v.w = fmaf(al, od[q].w, v.w);
                            }
                            stg[lane * 9 + q] = v;        // row `lane`, stride 36 floats
                        }
                        __syncwarp();
#pragma unroll
                        for (int k = 0; k < 8; ++k) {     // 4 rows x 8 float4 per instruction
                            const int rr = (lane >> 3) + 4 * k, cq = lane & 7;
                            const int rg = row_w0 + rr;
                            if (rg < p.M) {
                                const int o = rg / p.rs_rpo;
                                float* dr = p.rs_dst[o] + (size_t)(rg - o * p.rs_rpo) * p.ldd + col0;
                                reinterpret_cast<float4*>(dr)[cq] = stg[rr * 9 + cq];
                            }
                        }
                        __syncwarp();
                    } else if (full_chunk) {
                        float4* dp = reinterpret_cast<float4*>(srow + col0);
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            float4 v = make_float4(__uint_as_float(r[4 * q]) * f, __uint_as_float(r[4 * q + 1]) * f,
                                                   __uint_as_float(r[4 * q + 2]) * f, __uint_as_float(r[4 * q + 3]) * f);
                            if (own_in_ws) { v.x += ow[q].x; v.y += ow[q].y; v.z += ow[q].z; v.w += ow[q].w; }
                            if (add_d) {
                                v.x = fmaf(al, od[q].x, v.x); v.y = fmaf(al, od[q].y, v.y);
                                v.z = fmaf(al, od[q].z, v.z); v.w = fmaf(al, od[q].w, v.w);
                            }
                            dp[q] = v;
                        }
                    } else if (row_ok) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (col0 + j < p.N) {
                                float v = __uint_as_float(r[j]) * f;
                                if (own_in_ws) v += wrow[col0 + j];
                                if (add_d) v = fmaf(al, drow[col0 + j], v);
                                srow[col0 + j] = v;
                            }
                        }
                    }
                }
                if (flag && last_seg && !direct) {
                    // arrive; the second arrival adds the slab into D
                    __threadfence();
                    __syncwarp();
                    int old = 0;
                    if (lane == 0) old = atomicMax(flag, arrived);
                    old = __shfl_sync(0xffffffffu, old, 0);
                    if (old == arrived) {
                        __threadfence();
                        if (row_ok) {
                            float* drw = p.D + (size_t)row * p.ldd;
                            const int cend = col_base + p.bn < p.N ? col_base + p.bn : p.N;
                            int c = col_base;
                            for (; c + 32 <= cend; c += 32) {   // 8 + 8 loads in flight, then stores
                                float4 o[8], w4[8];
#pragma unroll
                                for (int q = 0; q < 8; ++q) {
                                    o[q] = reinterpret_cast<const float4*>(drw + c)[q];
                                    w4[q] = reinterpret_cast<const float4*>(wrow + c)[q];
                                }
#pragma unroll
                                for (int q = 0; q < 8; ++q) {
                                    o[q].x += w4[q].x; o[q].y += w4[q].y; o[q].z += w4[q].z; o[q].w += w4[q].w;
                                    reinterpret_cast<float4*>(drw + c)[q] = o[q];
                                }
                            }
                            for (; c < cend; ++c) drw[c] += wrow[c];
                        }
                    }
                }
            } else if constexpr (EPI == EPI_LSE) {
                // Per (row, tile) partial statistics of the softcapped logits:
                // max, lowest index of the max, sum exp(l - max), and the
                // label's logit when the label falls in this tile.  The
                // reference (lse_chunk_kernel, tier/tier.cpp:750-759) takes
                // every exp in fp64; here each term is an fp32 expf of l - max
                // <= 0 (relative error ~2^-22), a 32-column chunk's terms are
                // added pairwise in fp32 and the chunk sums in fp64.  With
                // one epilogue warp per SM sub-partition the fp64 exps were
                // the launch's limiter (math-pipe throttle the top stall, the
                // tensor pipe 46 % busy); the single-pass head already scales
                // its probabilities with the same fp32 expf (lm_prob_kernel).
                const LseDesc& L = ep->lse;
                const int label = row_ok ? L.labels[row + 1] - L.v0 : -1;
                float mx = -1e30f;
                int arg = 0x7fffffff;
                double sum = 0.0;
                float tgt = 0.0f;
#pragma unroll 1
                for (int c = 0; c < p.bn; c += 32) {
                    uint32_t r[32];
                    tc_ld_32x32b_x32(taddr + c, r);
                    tc_wait_ld();
                    const int col0 = col_base + c;
                    float v[32];
                    float cm = -1e30f;
                    int ci = 0x7fffffff;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        float l = __uint_as_float(r[j]) * f;
                        if (L.cap > 0.0f) l = L.cap * tanhf(l / L.cap);
                        const bool valid = col0 + j < p.N;
                        v[j] = valid ? l : -INFINITY;
                        if (valid && l > cm) { cm = l; ci = col0 + j; }
                        if (col0 + j == label) tgt = l;
                    }
                    if (L.zout && row_ok && col0 + 32 <= p.N) {
                        // the (softcapped) logits themselves, for the single-pass head
                        float4* zp = reinterpret_cast<float4*>(L.zout + (size_t)row * L.ldz + col0);
#pragma unroll
                        for (int q = 0; q < 8; ++q) zp[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                    }
                    if (cm > mx) {
                        sum *= exp((double)mx - (double)cm);
                        mx = cm;
                        arg = ci;
                    }
                    float e[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) e[j] = expf(v[j] - mx);   // columns past N: exp(-inf) = 0
#pragma unroll
                    for (int w = 16; w >= 1; w >>= 1) {
#pragma unroll
                        for (int j = 0; j < w; ++j) e[j] += e[j + w];
                    }
                    sum += (double)e[0];
                }
                if (row_ok) {
                    const size_t o = (size_t)row * L.ld_part + nb;
                    L.pmax[o] = mx;
                    L.parg[o] = arg;
                    L.psum[o] = sum;
                    L.ptgt[o] = tgt;
                }
            } else {
                // dlogit = ((softmax - onehot) / n_loss) * (1 - y^2) * mask,
                // scaled by 2^dl_exp and split into fp16 planes.
                const DlogitDesc& G = ep->dl;
                const bool live = row_ok && row < G.T - 1 && G.mask[row] != 0;
                const double lse = live ? G.rmax[row] + log(G.rsum[row]) : 0.0;
                const int label = live ? G.labels[row + 1] - G.v0 : -1;
                const float mval = live ? (float)G.mask[row] : 0.0f;
                const float sc = exp2i(G.dl_exp);
#pragma unroll 1
                for (int c = 0; c < p.bn; c += 32) {
                    uint32_t r[32];
                    tc_ld_32x32b_x32(taddr + c, r);
                    tc_wait_ld();
                    if (!row_ok) continue;
                    const int col0 = col_base + c;
                    if (col0 >= p.N) continue;
                    uint32_t hp[16], mp[16], lp[16];
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        float d = 0.0f;
                        if (live) {
                            float l = __uint_as_float(r[j]) * f;
                            if (G.cap > 0.0f) l = G.cap * tanhf(l / G.cap);
                            // fp32 exp of l - lse <= 0, as in the LSE epilogue above
                            const double sm = (double)expf((float)((double)l - lse));
                            const double oh = (col0 + j == label) ? 1.0 : 0.0;
                            const float y = G.cap > 0.0f ? l / G.cap : 0.0f;
                            d = (float)((sm - oh) / G.n_loss) * (1.0f - y * y) * mval;
                        }
                        const float v = d * sc;
                        const uint16_t h = f2h_bits(v);
                        const float rr = v - h2f_bits(h);
                        const uint16_t m = f2h_bits(rr);
                        const uint16_t lo = f2h_bits(rr - h2f_bits(m));
                        const int w = j >> 1, sh = 16 * (j & 1);
                        if (sh == 0) { hp[w] = h; mp[w] = m; lp[w] = lo; }
                        else { hp[w] |= (uint32_t)h << 16; mp[w] |= (uint32_t)m << 16; lp[w] |= (uint32_t)lo << 16; }
                    }
                    // N (the chunk width) is a multiple of 256 on this path.
                    uint16_t* base = G.planes + (size_t)row * G.ld + col0;
                    uint4* d0 = reinterpret_cast<uint4*>(base);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        d0[q] = make_uint4(hp[4 * q], hp[4 * q + 1], hp[4 * q + 2], hp[4 * q + 3]);
                    uint4* d1 = reinterpret_cast<uint4*>(base + G.plane_stride);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        d1[q] = make_uint4(mp[4 * q], mp[4 * q + 1], mp[4 * q + 2], mp[4 * q + 3]);
                    if (G.nplanes > 2) {
                        uint4* d2 = reinterpret_cast<uint4*>(base + 2 * G.plane_stride);
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            d2[q] = make_uint4(lp[4 * q], lp[4 * q + 1], lp[4 * q + 2], lp[4 * q + 3]);
                    }
                }
            }
            tc_fence_before();
            if constexpr (CG == 2) {
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
            } else {
                mbar_arrive(&tempty[acc]);
            }
          }
        }
    }

    // the problem (at most one) whose result is reduce-scattered to its owners
    const GemmParams* rsp = ps[0].rs_world ? &ps[0] : (NPROB == 2 && ps[NPROB - 1].rs_world ? &ps[NPROB - 1] : nullptr);
    if (EPI == EPI_STORE && rsp) __threadfence_system();   // peer stores before the done flag
    tc_fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync();   // the pair finishes together: no remote signal after exit
    if constexpr (EPI == EPI_STORE) {
        if (rsp && threadIdx.x == 0) {
            // every epilogue thread fenced its peer stores (system scope) before
            // the barriers above; the last CTA of the launch tells each owner
            __threadfence_system();
            const int old = atomicAdd(rsp->rs_counter, 1);
            if (old == (int)gridDim.x - 1) {
                *rsp->rs_counter = 0;
                __threadfence_system();
                for (int o = 0; o < rsp->rs_world; ++o) st_release_sys(rsp->rs_done[o], rsp->rs_epoch);
            }
        }
    }
    if (warp == 1) {
        tc_fence_after();
        if constexpr (CG == 2) tmem_dealloc_cg2(tmem_base, TMEM_COLS);
        else tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

template <int CG, bool B_MN, int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ GemmParams p, const __grid_constant__ EpiParams ep) {
    gemm_body<CG, B_MN ? 1 : 0, EPI, 1>(&p, &ep);
}

// Two plain-store problems in one persistent launch (see the file header).
template <int CG>
__global__ void __launch_bounds__(GEMM_THREADS, 1) gemm_pair_kernel(const __grid_constant__ GemmPair pp) {
    gemm_body<CG, 2, EPI_STORE, 2>(pp.p, nullptr);
}

// ---------------------------------------------------------------------------
// Host side: tensor maps (driver entry point fetched at run time) + launch.
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D fp16 tensor [rows, cols] (cols contiguous, row stride ld elements),
// box [box_rows, 64 cols], 128-byte swizzle, zero fill out of bounds.
static tk_status make_map(CUtensorMap* m, const void* base, long cols, long rows, long ld, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(TK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16)
        return fail(TK_ERR_INVALID, "GEMM operand must be 16-byte aligned with a row stride multiple of 8 elements");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TK_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return TK_OK;
}

template <int CG, bool B_MN, int EPI>
static tk_status go(tk_ctx* ctx, const GemmParams& gp, const EpiParams& ep, cudaStream_t s) {
    using G = Geo<CG>;
    static std::atomic<uint64_t> attr_done{0};   // per instantiation, one bit per device
    auto kern = gemm_tc_kernel<CG, B_MN, EPI>;
    {
        const cudaError_t e = smem_attr_once(kern, (int)G::SMEM, ctx->device, attr_done);
        if (e != cudaSuccess) return cuda_fail(e, "gemm smem attribute");
    }
    const int tiles = gp.tiles_m * gp.tiles_n * gp.splits;   // work units
    const int groups_max = ctx->num_sms / CG;
    const int groups = tiles < groups_max ? tiles : groups_max;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(groups * CG, 1, 1);
    cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = G::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CG;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    ProfScope ps(ctx, s, PK_GEMM);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, gp, ep);
    ctx->launches++;
    if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
    return cuda_fail(cudaGetLastError(), "gemm launch");
}

static tk_status build(const GemmDesc& g, tk_ctx* ctx, GemmParams& gp, int cg, int bn) {
    if (g.M <= 0 || g.N <= 0 || g.K <= 0) return fail(TK_ERR_INVALID, "GEMM with empty shape");
    if (g.nprod < 1 || g.nprod > 3) return fail(TK_ERR_INVALID, "GEMM product count must be 1..3");
    if ((reinterpret_cast<uintptr_t>(g.D) & 15) || g.ldd % 4)
        return fail(TK_ERR_INVALID, "output must be 16-byte aligned with a row stride multiple of 4");
    memset(&gp, 0, sizeof(gp));
    for (int i = 0; i < g.nprod; ++i) {
        if (g.pa[i] < 0 || g.pa[i] > 2 || !g.A[g.pa[i]] || g.pb[i] < 0 || g.pb[i] > 1 || !g.B[g.pb[i]])
            return fail(TK_ERR_INVALID, "GEMM product references a missing plane");
    }
    for (int i = 0; i < 3; ++i)
        if (g.A[i]) {
            tk_status st = make_map(&gp.tmA[i], g.A[i], g.K, g.M, g.lda, BM);
            if (st != TK_OK) return st;
        }
    for (int i = 0; i < 2; ++i)
        if (g.B[i]) {
            tk_status st = g.b_mn ? make_map(&gp.tmB[i], g.B[i], g.N, g.K, g.ldb, BK)
                                  : make_map(&gp.tmB[i], g.B[i], g.K, g.N, g.ldb, bn / cg);
            if (st != TK_OK) return st;
        }
    gp.M = g.M; gp.N = g.N; gp.K = g.K;
    gp.nprod = g.nprod;
    for (int i = 0; i < 3; ++i) { gp.pa[i] = g.pa[i]; gp.pb[i] = g.pb[i]; }
    gp.tiles_m = (g.M + BM * cg - 1) / (BM * cg);
    gp.tiles_n = (g.N + bn - 1) / bn;
    gp.bn = bn;
    {
        // Band height: the in-flight block a x b (a x b = CTA groups) that
        // reads the fewest operand bytes per k-step, a * A panel + b * B panel,
        // is a = sqrt(groups * B panel / A panel).  Measured on B200 with plain
        // row-fastest order: the LM-head logits GEMM (A = three X planes over
        // 32 tile rows, 189 MB) read 7.1 GB from DRAM per 315 MB of operands.
        int na = 0, nb_ = 0;
        for (int i = 0; i < 3; ++i) na += g.A[i] != nullptr;
        for (int i = 0; i < 2; ++i) nb_ += g.B[i] != nullptr;
        const double groups = (double)(ctx->num_sms / cg);
        const double a = std::sqrt(groups * (double)(bn * nb_) / (double)(BM * cg * (na > 0 ? na : 1)));
        int gm = (int)(a + 0.5);
        // every A panel fits in L2 at once (<= 48 MB): row-fastest order reads
        // A and B once (the C2 forward, X 32 MB); measured on the C2 step the
        // band choices agree within 1 %, except 4-row bands (3 % slower)
        const double a_all = (double)gp.tiles_m * BM * cg * (double)g.K * 2.0 * (na > 0 ? na : 1);
        if (a_all <= 48.0 * 1048576.0) gm = gp.tiles_m;
        gp.group_m = gm < 1 ? 1 : (gm > gp.tiles_m ? gp.tiles_m : gm);
    }
    gp.splits = 1;
    gp.flags = nullptr;
    gp.epoch = 0;
    gp.sws = nullptr;
    gp.sws_ld = 0;
    {
        const int kblocks = (g.K + BK - 1) / BK;
        int seg = g.seg_kb > 0 ? g.seg_kb : kblocks;
        gp.seg_kb = seg < kblocks ? seg : kblocks;
    }
    gp.D = g.D; gp.ldd = g.ldd; gp.beta = g.beta;
    gp.row_exp = g.row_exp; gp.col_exp = g.col_exp;
    gp.row_alpha = g.row_alpha;
    gp.rs_world = 0;
    if (g.rs) {
        for (int i = 0; i < TK_MAX_RANKS; ++i) { gp.rs_dst[i] = g.rs->dst[i]; gp.rs_done[i] = g.rs->done[i]; }
        gp.rs_counter = g.rs->counter;
        gp.rs_world = g.rs->world;
        gp.rs_rpo = g.rs->rpo;
        gp.rs_epoch = g.rs->epoch;
    }
    gp.b_mn = g.b_mn ? 1 : 0;
    gp.status = ctx->status;
    return TK_OK;
}

// CTA pairs for every GEMM with more than one 128-row block of output rows;
// a single CTA otherwise (a pair would leave half its tensor cores idle).
static int pick_cg(const GemmDesc& g) { return g.M > BM ? 2 : 1; }

// Tile width: the persistent grid runs ceil(tiles / groups) waves of tiles, so
// pick the width with the least (waves x width x per-FLOP premium); narrower
// tiles move more operand bytes per MMA and pay for it.  An N-major B is
// loaded in 64-column boxes per CTA, which allows 256 and 128 (CTA pairs).
static int pick_bn(const GemmDesc& g, int cg, int num_sms) {
    const int groups = num_sms / cg;
    const int tiles_m = (g.M + BM * cg - 1) / (BM * cg);
    static const int cand[4] = {256, 224, 192, 128};
    // measured on B200 (CTA pairs, K = 4096..14336): 224 ~1.12x, 128 ~1.45x
    // the time per FLOP of 256-wide tiles
    static const double premium[4] = {1.0, 1.12, 1.25, 1.45};
    int best = 256;
    double best_cost = 1e300;
    for (int i = 0; i < 4; ++i) {
        const int bn = cand[i];
        if (g.b_mn && (bn / cg) % 64) continue;
        const long tiles = (long)tiles_m * ((g.N + bn - 1) / bn);
        const long waves = (tiles + groups - 1) / groups;
        const double cost = (double)waves * bn * premium[i];
        if (cost < best_cost - 1e-9) { best_cost = cost; best = bn; }
    }
    return best;
}

// K splits: the waves of (tile, split) units against the fp32 read-modify-
// write a later split adds (about 5 k-blocks of MMA time per tile).
static int pick_splits(int tiles_m, int tiles_n, int cg, int num_sms, int kblocks, int max_tiles) {
    const long groups = num_sms / cg, tiles = (long)tiles_m * tiles_n;
    if (tiles > max_tiles) return 1;
    const double c1 = (double)((tiles + groups - 1) / groups) * kblocks;
    const double c2 = (double)((2 * tiles + groups - 1) / groups) * ((kblocks + 1) / 2) + 5.0;
    return (kblocks >= 32 && c2 < 0.95 * c1) ? 2 : 1;
}

int gemm_splits(const tk_ctx* ctx, const GemmDesc& g) {
    if (!ctx->flags || g.M <= 0 || g.N <= 0 || g.K <= 0) return 1;
    const int cg = pick_cg(g), bn = pick_bn(g, cg, ctx->num_sms);
    const int tiles_m = (g.M + BM * cg - 1) / (BM * cg), tiles_n = (g.N + bn - 1) / bn;
    return pick_splits(tiles_m, tiles_n, cg, ctx->num_sms, (g.K + BK - 1) / BK, ctx->flags_len / (4 * cg));
}

tk_status launch_gemm(tk_ctx* ctx, const GemmDesc& g, cudaStream_t s) {
    const int cg = pick_cg(g);
    GemmParams gp;
    tk_status st = build(g, ctx, gp, cg, pick_bn(g, cg, ctx->num_sms));
    if (st != TK_OK) return st;
    if (g.split_ws && gemm_splits(ctx, g) == 2) {
        if ((reinterpret_cast<uintptr_t>(g.split_ws) & 15) || g.split_ld < g.N || g.split_ld % 4)
            return fail(TK_ERR_INVALID, "split-K workspace misaligned");
        // flags hold epoch*16 + 1 once a split arrived; stamps only grow, so no
        // reset is needed until the stamp wraps
        if (++ctx->epoch >= (1u << 26)) {
            cudaError_t e = cudaMemsetAsync(ctx->flags, 0, sizeof(int) * ctx->flags_len, s);
            if (e != cudaSuccess) return fail(TK_ERR_CUDA, "split-K flag reset failed");
            ctx->epoch = 1;
        }
        gp.splits = 2;
        gp.flags = ctx->flags;
        gp.epoch = (int)ctx->epoch;
        gp.sws = g.split_ws;
        gp.sws_ld = g.split_ld;
    }
    EpiParams ep;
    memset(&ep, 0, sizeof(ep));
    if (cg == 2) return g.b_mn ? go<2, true, EPI_STORE>(ctx, gp, ep, s) : go<2, false, EPI_STORE>(ctx, gp, ep, s);
    return g.b_mn ? go<1, true, EPI_STORE>(ctx, gp, ep, s) : go<1, false, EPI_STORE>(ctx, gp, ep, s);
}

// Operand bytes a pair launch reads (A planes, and B planes once when the
// two problems share them, as the forward and dX of one weight do).
static size_t pair_operand_bytes(const GemmDesc& g0, const GemmDesc& g1) {
    auto planes = [](const uint16_t* const* p, int n) {
        int c = 0;
        for (int i = 0; i < n; ++i) c += p[i] != nullptr;
        return c;
    };
    size_t b = 0;
    for (const GemmDesc* g : {&g0, &g1}) b += (size_t)g->M * g->K * 2 * planes(g->A, 3);
    const size_t wb = (size_t)g0.N * g0.K * 2 * planes(g0.B, 2);
    b += wb;
    if (g1.B[0] != g0.B[0]) b += (size_t)g1.N * g1.K * 2 * planes(g1.B, 2);
    return b;
}
constexpr size_t kPairL2Bytes = 96ull << 20;

// The units of a pair launch assigned to the CTA pairs by list scheduling:
// in the launch's unit order (interleaved, or problem 1 first), each unit goes
// to the CTA pair that frees up first, by an estimate of its time (k-blocks x
// products + segments' epilogues).  Unit costs differ between the problems
// (e.g. a dX tile over all 14336 rows of W against a forward tile over 4096
// columns), where a plain stride over the units would leave some CTA pairs
// several units longer than others.  The table goes to the device once per
// shape (ctx->sched, ordered on the stream like the launch that reads it).
static tk_status pair_schedule(tk_ctx* ctx, const GemmParams& p0, const GemmParams& p1, int groups, bool interleave,
                               cudaStream_t s) {
    const int t0 = p0.tiles_m * p0.tiles_n, t1 = p1.tiles_m * p1.tiles_n, t = t0 + t1;
    const std::vector<long> key = {t0, t1, p0.K, p1.K, p0.nprod, p1.nprod, p0.seg_kb, p1.seg_kb, groups, interleave};
    if (ctx->sched && ctx->sched_key == key) return TK_OK;
    std::vector<int> order(t);
    for (int u = 0; u < t; ++u) {
        if (!interleave) { order[u] = u; continue; }
        // ceil(u * t1 / t) units of problem 1 come before position u: its
        // tiles spread evenly, one at the start of each period
        const int c = (int)(((long)u * t1 + t - 1) / t), cn = (int)(((long)(u + 1) * t1 + t - 1) / t);
        order[u] = cn > c ? c : t1 + (u - c);
    }
    auto cost = [&](int id) {
        const GemmParams& q = id < t1 ? p1 : p0;
        const long kb = (q.K + BK - 1) / BK;
        return kb * q.nprod + 4 * ((kb + q.seg_kb - 1) / q.seg_kb);
    };
    std::priority_queue<std::pair<long, int>, std::vector<std::pair<long, int>>, std::greater<std::pair<long, int>>> free_at;
    for (int g = 0; g < groups; ++g) free_at.push({0, g});
    std::vector<std::vector<int>> per(groups);
    for (int id : order) {
        const auto [load, g] = free_at.top();
        free_at.pop();
        per[g].push_back(id);
        free_at.push({load + cost(id), g});
    }
    std::vector<int> host((size_t)groups + 1 + t);
    int o = 0;
    for (int g = 0; g < groups; ++g) {
        host[g] = o;
        for (int id : per[g]) host[groups + 1 + o++] = id;
    }
    host[groups] = o;
    if (host.size() > ctx->sched_cap) {
        cudaError_t e = cudaDeviceSynchronize();   // a launch in flight may still read the old table
        if (e != cudaSuccess) return cuda_fail(e, "pair schedule sync");
        if (ctx->sched) cudaFree(ctx->sched);
        ctx->sched = nullptr;
        ctx->sched_cap = 0;
        e = cudaMalloc(&ctx->sched, host.size() * sizeof(int));
        if (e != cudaSuccess) return cuda_fail(e, "pair schedule table");
        ctx->sched_cap = host.size();
    }
    // from pageable memory: the call returns once the table is staged
    cudaError_t e = cudaMemcpyAsync(ctx->sched, host.data(), host.size() * sizeof(int), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cuda_fail(e, "pair schedule upload");
    ctx->sched_key = key;
    return TK_OK;
}

// Both problems of a pair with CTA pairs and 256-wide tiles (an N-major B
// loads 64-column boxes, so 256 suits both layouts); the combined unit list
// takes care of the waves, so the per-problem tile-width choice is not needed.
bool gemm_pair_ok(const GemmDesc& g0, const GemmDesc& g1) {
    for (const GemmDesc* g : {&g0, &g1})
        if (pick_cg(*g) != 2 || g->split_ws || (g->rs && g != &g1)) return false;
    return true;
}

tk_status launch_gemm_pair(tk_ctx* ctx, const GemmDesc& g0, const GemmDesc& g1, cudaStream_t s) {
    if (!gemm_pair_ok(g0, g1)) return fail(TK_ERR_INVALID, "GEMM pair needs two CTA-pair problems without split-K");
    GemmPair pp;
    tk_status st = build(g0, ctx, pp.p[0], 2, BN);
    if (st != TK_OK) return st;
    st = build(g1, ctx, pp.p[1], 2, BN);
    if (st != TK_OK) return st;
    const int units = pp.p[0].tiles_m * pp.p[0].tiles_n + pp.p[1].tiles_m * pp.p[1].tiles_n;
    const int groups_max = ctx->num_sms / 2;
    const int groups = units < groups_max ? units : groups_max;
    // Interleaving the two tile lists halves each problem's tiles in flight,
    // so each operand panel is shared by fewer concurrent tiles; that only
    // pays while both problems' operands stay in L2 together.  Measured on
    // B200 (forward + dX of W[ng, 4096], M = 4096, bf16): interleaved beats
    // two launches at 61 and 90 MB of operands (ng = 1792, 3584: 125 vs 136,
    // 220 vs 244 us) and loses at 148 and 266 MB (ng = 7168, 14336), where
    // its DRAM reads grew 3.6x.  Above the threshold the problems run one
    // after the other in one launch.
    const bool interleave = pair_operand_bytes(g0, g1) <= kPairL2Bytes;
    st = pair_schedule(ctx, pp.p[0], pp.p[1], groups, interleave, s);
    if (st != TK_OK) return st;
    pp.p[0].sched_off = ctx->sched;
    pp.p[0].sched = ctx->sched + groups + 1;
    using G = Geo<2>;
    static std::atomic<uint64_t> attr_done{0};
    auto kern = gemm_pair_kernel<2>;
    {
        const cudaError_t e = smem_attr_once(kern, (int)G::SMEM, ctx->device, attr_done);
        if (e != cudaSuccess) return cuda_fail(e, "gemm pair smem attribute");
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(groups * 2, 1, 1);
    cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = G::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    ProfScope ps(ctx, s, PK_GEMM);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, pp);
    ctx->launches++;
    if (e != cudaSuccess) return cuda_fail(e, "gemm pair launch");
    return cuda_fail(cudaGetLastError(), "gemm pair launch");
}

tk_status launch_gemm_lse(tk_ctx* ctx, const GemmDesc& g, const LseDesc& e, cudaStream_t s) {
    if (g.b_mn) return fail(TK_ERR_INVALID, "LM-head logits GEMM takes a K-major head");
    const int cg = pick_cg(g);
    GemmParams gp;
    tk_status st = build(g, ctx, gp, cg, BN);
    if (st != TK_OK) return st;
    gp.seg_kb = (g.K + BK - 1) / BK;   // statistics need the complete logit
    EpiParams ep;
    memset(&ep, 0, sizeof(ep));
    ep.lse = e;
    return cg == 2 ? go<2, false, EPI_LSE>(ctx, gp, ep, s) : go<1, false, EPI_LSE>(ctx, gp, ep, s);
}

tk_status launch_gemm_dlogit(tk_ctx* ctx, const GemmDesc& g, const DlogitDesc& e, cudaStream_t s) {
    if (g.b_mn) return fail(TK_ERR_INVALID, "LM-head logits GEMM takes a K-major head");
    if (g.N % BN) return fail(TK_ERR_INVALID, "dlogit epilogue needs a chunk width multiple of 256");
    const int cg = pick_cg(g);
    GemmParams gp;
    tk_status st = build(g, ctx, gp, cg, BN);
    if (st != TK_OK) return st;
    gp.seg_kb = (g.K + BK - 1) / BK;
    EpiParams ep;
    memset(&ep, 0, sizeof(ep));
    ep.dl = e;
    return cg == 2 ? go<2, false, EPI_DLOGIT>(ctx, gp, ep, s) : go<1, false, EPI_DLOGIT>(ctx, gp, ep, s);
}

}  // namespace tk
