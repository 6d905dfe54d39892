// tk_device.cuh -- sm_100a device primitives shared by the tierk kernels:
// mbarrier / TMA / tcgen05 wrappers with bounded waits, the device status
// word, and bit-exact block dequant (restating tier/quant.h:37-121; the
// table-level types in tk_qtypes.h).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "tk_qgrid.h"
#include "tk_qtypes.h"

namespace tk {

// ---------------------------------------------------------------------------
// Status word: kernels never trap; a failed bounded wait or an invalid value
// detected on the device records a code here (first writer wins).
// ---------------------------------------------------------------------------
enum : int { DEV_OK = 0, DEV_TIMEOUT = 5, DEV_INVALID = 6 };

// A bounded wait gives up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void raise_status(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start once every CTA of the kernel
// before it has called pdl_trigger (or exited); it must call pdl_wait before
// it touches anything that kernel writes (pdl_wait returns once that kernel
// has completed and its memory is visible).  The producers of a GEMM's
// operands trigger at their start, so the GEMM's CTAs set up (barriers,
// TMEM, descriptors) while the producer's last wave drains.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase with the given parity to complete.  Returns false (and
// records DEV_TIMEOUT) if it has not completed within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(a, parity)) return true;
        if (globaltimer() - t0 > kWaitLimitNs) {
            raise_status(status, DEV_TIMEOUT);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------
// TMA (tiled tensor loads into shared memory; never with cluster multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
// Untiled bulk copy global -> shared (both 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, accumulators in TMEM)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16/bf16 in, fp32 acc).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on `bar` once all previously issued tcgen05.mma of this thread retire.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets TMEM
// lane (taddr.lane + i), columns taddr.col .. +31.
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// ---- CTA pairs (cluster of 2, cta_group::2) ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier given by its shared::cluster address (possibly the peer's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Tiled TMA load into this CTA's shared memory whose completion is counted on
// an mbarrier that may live in the peer CTA of the pair (cluster address).
// Plain load: no multicast.
__device__ __forceinline__ void tma_load_2d_cg2(void* smem_dst, const void* tmap, uint32_t bar_cluster, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_cg2(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_cg2() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_cg2(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Pair MMA: D (rows split over the two CTAs' TMEM) (+)= A (rows split over the
// two CTAs' shared memory) * B (columns split over the two CTAs' shared memory).
__device__ __forceinline__ void tc_mma_f16_cg2(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on one mbarrier (cluster address) once the pair's issued MMAs retire.
__device__ __forceinline__ void tc_commit_cg2(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
                 : "memory");
}

// Shared-memory matrix descriptor (tcgen05 "version 1"), 128-byte swizzle.
//   K-major tile: rows of 64 fp16 (128 B), 8-row atoms 1024 B apart (SBO).
//   MN-major tile: 64 MN-elements (128 B) per K-row, K-rows 128 B apart,
//   8-K-row groups SBO = 1024 B apart, 64-element MN groups LBO apart.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3fffu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3fffu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3fffu) << 32;
    d |= (uint64_t)1 << 46;   // descriptor version for sm_100
    d |= (uint64_t)2 << 61;   // SWIZZLE_128B
    return d;
}
// Instruction descriptor, kind::f16: D fp32, A/B fp16 (fmt 0) or bf16 (fmt 1).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int ab_fmt, int a_mn_major, int b_mn_major) {
    return (1u << 4) | ((uint32_t)ab_fmt << 7) | ((uint32_t)ab_fmt << 10) | ((uint32_t)a_mn_major << 15) |
           ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// fp16 / bf16 conversions matching the reference's software versions
// (tier/gpu_compat.h:151-190): IEEE round-to-nearest-even with subnormals;
// NaN maps to sign|0x7e00 as tier_fp16::from_float does.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint16_t f2h_bits(float v) {
    uint16_t h = __half_as_ushort(__float2half_rn(v));
    if (v != v) h = (uint16_t)(((__float_as_uint(v) >> 16) & 0x8000u) | 0x7e00u);
    return h;
}
__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2bf_bits(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }

// ---------------------------------------------------------------------------
// Block dequant, bit-exact with tier/quant.h:59-121.  Products and sums use
// the _rn intrinsics so nvcc cannot contract them into FMAs.
// ---------------------------------------------------------------------------
enum : int {
    QT_F32 = 0, QT_F16 = 1, QT_Q4_0 = 2, QT_Q4_1 = 3, QT_Q5_0 = 6, QT_Q5_1 = 7, QT_Q8_0 = 8, QT_Q2_K = 10,
    QT_Q3_K = 11, QT_Q4_K = 12, QT_Q5_K = 13, QT_Q6_K = 14, QT_BF16 = 30,
    QT_IQ4_NL = tkq::IQ4_NL, QT_IQ4_XS = tkq::IQ4_XS, QT_TQ1_0 = tkq::TQ1_0, QT_TQ2_0 = tkq::TQ2_0,
    QT_MXFP4 = tkq::MXFP4, QT_NF4 = tkq::NF4, QT_FP4 = tkq::FP4
};

__device__ __forceinline__ uint16_t ld_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
__device__ __forceinline__ float blk_scale(const uint8_t* p) { return h2f_bits(ld_u16(p)); }

// Q4_K/Q5_K packed 6-bit sub-block scale/min (tier/quant.h:47-48).
__device__ __forceinline__ void kq_scale_min(int j, const uint8_t* s, int& sc, int& mn) {
    if (j < 4) {
        sc = s[j] & 63;
        mn = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// Scalar value of element `col` of a block row.
__device__ __forceinline__ float qval(const uint8_t* row, int type, int col) {
    if (tkq::elems(type)) return tkq::value(row, type, col);   // IQ4_NL, IQ4_XS, MXFP4, NF4, FP4, TQ1_0, TQ2_0
    switch (type) {
        case QT_F32: return __uint_as_float(ld_u32(row + (size_t)col * 4));
        case QT_F16: return h2f_bits(ld_u16(row + (size_t)col * 2));
        case QT_BF16: return __uint_as_float((uint32_t)ld_u16(row + (size_t)col * 2) << 16);
        case QT_Q4_0: {
            const uint8_t* b = row + (size_t)(col >> 5) * 18;
            int i = col & 31, q = (b[2 + (i & 15)] >> ((i >> 4) * 4)) & 15;
            return __fmul_rn(blk_scale(b), (float)(q - 8));
        }
        case QT_Q4_1: {
            const uint8_t* b = row + (size_t)(col >> 5) * 20;
            int i = col & 31, q = (b[4 + (i & 15)] >> ((i >> 4) * 4)) & 15;
            return __fadd_rn(__fmul_rn(blk_scale(b), (float)q), blk_scale(b + 2));
        }
        case QT_Q5_0: {
            const uint8_t* b = row + (size_t)(col >> 5) * 22;
            int i = col & 31;
            int q = ((b[6 + (i & 15)] >> ((i >> 4) * 4)) & 15) | (int)(((ld_u32(b + 2) >> i) & 1u) << 4);
            return __fmul_rn(blk_scale(b), (float)(q - 16));
        }
        case QT_Q5_1: {
            const uint8_t* b = row + (size_t)(col >> 5) * 24;
            int i = col & 31;
            int q = ((b[8 + (i & 15)] >> ((i >> 4) * 4)) & 15) | (int)(((ld_u32(b + 4) >> i) & 1u) << 4);
            return __fadd_rn(__fmul_rn(blk_scale(b), (float)q), blk_scale(b + 2));
        }
        case QT_Q8_0: {
            const uint8_t* b = row + (size_t)(col >> 5) * 34;
            return __fmul_rn(blk_scale(b), (float)(int8_t)b[2 + (col & 31)]);
        }
        default: break;
    }
    const int i = col & 255;
    switch (type) {
        case QT_Q2_K: {
            const uint8_t* b = row + (size_t)(col >> 8) * 84;
            int h = i >> 7, s = (i & 127) >> 5, l = i & 31;
            int q = (b[16 + h * 32 + l] >> (2 * s)) & 3;
            uint8_t sc = b[i >> 4];
            float a = __fmul_rn(blk_scale(b + 80), (float)(sc & 15));
            return __fsub_rn(__fmul_rn(a, (float)q), __fmul_rn(blk_scale(b + 82), (float)(sc >> 4)));
        }
        case QT_Q3_K: {
            const uint8_t* b = row + (size_t)(col >> 8) * 110;
            const uint8_t* s = b + 96;
            int j = i >> 4;
            int lo = j < 8 ? (s[j] & 15) : (s[j - 8] >> 4), hi = (s[8 + (j & 3)] >> (2 * (j >> 2))) & 3;
            int sc = (int)(int8_t)(uint8_t)(lo | (hi << 4)) - 32;
            int h = i >> 7, sh = (i & 127) >> 5, l = i & 31;
            int ql = (b[32 + h * 32 + l] >> (2 * sh)) & 3, hb = ((b[l] >> (i >> 5)) & 1) ^ 1;
            return __fmul_rn(__fmul_rn(blk_scale(b + 108), (float)sc), (float)(ql - (hb << 2)));
        }
        case QT_Q4_K: {
            const uint8_t* b = row + (size_t)(col >> 8) * 144;
            int g = i >> 6, l = i & 63, sc, mn;
            kq_scale_min(2 * g + (l >= 32), b + 4, sc, mn);
            uint8_t y = b[16 + g * 32 + (l & 31)];
            int q = l < 32 ? (y & 15) : (y >> 4);
            return __fsub_rn(__fmul_rn(__fmul_rn(blk_scale(b), (float)sc), (float)q),
                             __fmul_rn(blk_scale(b + 2), (float)mn));
        }
        case QT_Q5_K: {
            const uint8_t* b = row + (size_t)(col >> 8) * 176;
            int g = i >> 6, l = i & 63, sc, mn;
            kq_scale_min(2 * g + (l >= 32), b + 4, sc, mn);
            uint8_t y = b[48 + g * 32 + (l & 31)];
            int q = (l < 32 ? (y & 15) : (y >> 4)) | (((b[16 + (i & 31)] >> (i >> 5)) & 1) << 4);
            return __fsub_rn(__fmul_rn(__fmul_rn(blk_scale(b), (float)sc), (float)q),
                             __fmul_rn(blk_scale(b + 2), (float)mn));
        }
        case QT_Q6_K: {
            const uint8_t* b = row + (size_t)(col >> 8) * 210;
            int a = i >> 7, c = i & 63, nib = (i & 127) >> 6, s = (i & 127) >> 5, l = i & 31;
            int ql = (b[a * 64 + c] >> (4 * nib)) & 15, qh = (b[128 + a * 32 + l] >> (2 * s)) & 3;
            int q = (int)(int8_t)(uint8_t)(ql | (qh << 4)) - 32;
            return __fmul_rn(__fmul_rn(blk_scale(b + 208), (float)(int8_t)b[192 + (i >> 4)]), (float)q);
        }
        default: break;
    }
    return 0.0f;
}

// Eight consecutive elements [c, c+8) of a Q4_K row (c % 8 == 0): they share
// one 32-element sub-block, so one (d*sc, dmin*m) pair and eight nibbles from
// eight consecutive bytes.  (d*sc)*q is exact in fp32 (11+6+4 significant
// bits), so a single fused multiply-subtract rounds exactly like the
// reference's separate multiply and subtract.
// Exact float of a small non-negative integer (< 2^23) without the
// int-to-float conversion pipe: OR it into the mantissa of 2^23, subtract 2^23.
__device__ __forceinline__ float small_u2f(uint32_t q) { return __uint_as_float(0x4B000000u | q) - 8388608.0f; }

// Sub-block scale and min from the 12 packed bytes held in registers
// (hdr.y, hdr.z, hdr.w of the 16-byte super-block header).
// Bytes 0-3 of the packed area are hdr.y, 4-7 hdr.z, 8-11 hdr.w; sub-block
// j and j-4 (or j+4) always sit at the same byte position jj = j & 3.
__device__ __forceinline__ void kq_scale_min_reg(int j, uint4 hdr, int& sc, int& mn) {
    const int sh = 8 * (j & 3);
    const int b0 = (hdr.y >> sh) & 0xff, b1 = (hdr.z >> sh) & 0xff, b2 = (hdr.w >> sh) & 0xff;
    const int sc_lo = b0 & 63, mn_lo = b1 & 63;                                   // j < 4
    const int sc_hi = (b2 & 0x0f) | ((b0 >> 6) << 4), mn_hi = (b2 >> 4) | ((b1 >> 6) << 4);   // j >= 4
    sc = j < 4 ? sc_lo : sc_hi;
    mn = j < 4 ? mn_lo : mn_hi;
}

__device__ __forceinline__ void q4k_decode8(const uint8_t* row, int c, float (&v)[8]) {
    const uint8_t* b = row + (size_t)(c >> 8) * 144;
    const int i = c & 255, g = i >> 6, l = i & 63;
    const uint4 hdr = *reinterpret_cast<const uint4*>(b);           // d, dmin, 12 scale bytes
    const uint2 w = *reinterpret_cast<const uint2*>(b + 16 + g * 32 + (l & 31));
    int sc, mn;
    kq_scale_min_reg(2 * g + (l >= 32), hdr, sc, mn);
    const float a = __fmul_rn(h2f_bits((uint16_t)(hdr.x & 0xffff)), (float)sc);
    const float m = __fmul_rn(h2f_bits((uint16_t)(hdr.x >> 16)), (float)mn);
    const int sh = l < 32 ? 0 : 4;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t word = j < 4 ? w.x : w.y;
        const uint32_t q = (word >> (8 * (j & 3) + sh)) & 15u;
        v[j] = __fmaf_rn(a, small_u2f(q), -m);
    }
}

// Eight consecutive elements of a Q5_K row (c % 8 == 0).  (d*sc)*q has at
// most 11+6+5 significant bits, so it is exact and the fused form is exact.
__device__ __forceinline__ void q5k_decode8(const uint8_t* row, int c, float (&v)[8]) {
    const uint8_t* b = row + (size_t)(c >> 8) * 176;
    const int i = c & 255, g = i >> 6, l = i & 63;
    const uint4 hdr = *reinterpret_cast<const uint4*>(b);
    const uint2 w = *reinterpret_cast<const uint2*>(b + 48 + g * 32 + (l & 31));
    const uint2 hb = *reinterpret_cast<const uint2*>(b + 16 + (i & 31));
    int sc, mn;
    kq_scale_min_reg(2 * g + (l >= 32), hdr, sc, mn);
    const float a = __fmul_rn(h2f_bits((uint16_t)(hdr.x & 0xffff)), (float)sc);
    const float m = __fmul_rn(h2f_bits((uint16_t)(hdr.x >> 16)), (float)mn);
    const int sh = l < 32 ? 0 : 4, hsh = i >> 5;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t word = j < 4 ? w.x : w.y;
        uint32_t hw = j < 4 ? hb.x : hb.y;
        const uint32_t q = ((word >> (8 * (j & 3) + sh)) & 15u) | (((hw >> (8 * (j & 3) + hsh)) & 1u) << 4);
        v[j] = __fmaf_rn(a, small_u2f(q), -m);
    }
}

// One 32-element sub-block of a Q4_K / Q5_K / Q8_0 row as 16 packed fp16
// pairs, bit-exact tier_fp16(q_val) (tier/quant.h:68, 83-87):
//   Q8_0: d*q is exact in fp32 and in the fp16 multiply (11 + 8 bits), so one
//         packed fp16 RNE multiply of d by the exact half q gives the value;
//   K-quants: fp32 fused (d*sc)*q - dmin*m (the product is exact), then RNE.
// Nibbles become floats by byte-permuting them into the mantissa of 2^23.
// A block with a non-finite scale takes the per-element path so that NaN bit
// patterns match the reference's conversion as well.
template <int T>
__device__ __forceinline__ void sub32_to_f16(const uint8_t* __restrict__ row, int sub, uint32_t (&h)[16]) {
    if constexpr (T == QT_Q8_0) {
        const uint8_t* blk = row + (size_t)sub * 34;
        const uint16_t dbits = ld_u16(blk);
        const uint16_t* q = reinterpret_cast<const uint16_t*>(blk + 2);
        if (((dbits >> 10) & 0x1f) == 0x1f) {   // inf/NaN scale
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float d = h2f_bits(dbits);
                const uint16_t w = q[j];
                h[j] = (uint32_t)f2h_bits(__fmul_rn(d, (float)(int8_t)(w & 0xff))) |
                       ((uint32_t)f2h_bits(__fmul_rn(d, (float)(int8_t)(w >> 8))) << 16);
            }
            return;
        }
        const __half2 d2 = __halves2half2(__ushort_as_half(dbits), __ushort_as_half(dbits));
        const __half2 off = __halves2half2(__ushort_as_half((uint16_t)0x6480), __ushort_as_half((uint16_t)0x6480));   // 1152
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint32_t w = (uint32_t)q[j] ^ 0x8080u;                   // int8 pair -> q + 128
            const uint32_t mg = __byte_perm(w, 0x64006400u, 0x7170);        // half2 (1024 + b0, 1024 + b1)
            const __half2 v = __hmul2(d2, __hsub2(*reinterpret_cast<const __half2*>(&mg), off));
            h[j] = *reinterpret_cast<const uint32_t*>(&v);
        }
    } else {
        constexpr int SBB = T == QT_Q4_K ? 144 : 176;
        constexpr int QS = T == QT_Q4_K ? 16 : 48;
        const uint8_t* b = row + (size_t)(sub >> 3) * SBB;
        const int j = sub & 7;
        const uint4 hdr = *reinterpret_cast<const uint4*>(b);
        int sc, mn;
        kq_scale_min_reg(j, hdr, sc, mn);
        const float a = __fmul_rn(h2f_bits((uint16_t)(hdr.x & 0xffff)), (float)sc);
        const float m = __fmul_rn(h2f_bits((uint16_t)(hdr.x >> 16)), (float)mn);
        const uint4 q0 = *reinterpret_cast<const uint4*>(b + QS + 32 * (j >> 1));
        const uint4 q1 = *reinterpret_cast<const uint4*>(b + QS + 32 * (j >> 1) + 16);
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        uint32_t hw[8];
        if constexpr (T == QT_Q5_K) {
            const uint4 a0 = *reinterpret_cast<const uint4*>(b + 16);
            const uint4 a1 = *reinterpret_cast<const uint4*>(b + 32);
            hw[0] = a0.x; hw[1] = a0.y; hw[2] = a0.z; hw[3] = a0.w; hw[4] = a1.x; hw[5] = a1.y; hw[6] = a1.z; hw[7] = a1.w;
        }
        const bool finite = fabsf(a) < INFINITY && fabsf(m) < INFINITY;
        const uint32_t sh = (j & 1) * 4;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            // four nibbles of bytes 4k..4k+3, each placed into the mantissa of 2^23
            uint32_t nib = (qw[k] >> sh) & 0x0F0F0F0Fu;
            if constexpr (T == QT_Q5_K) nib |= ((hw[k] >> j) & 0x01010101u) << 4;
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float q = __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7440 + e)) - 8388608.0f;
                v[e] = __fmaf_rn(a, q, -m);
            }
            if (finite) {
                const __half2 p0 = __floats2half2_rn(v[0], v[1]), p1 = __floats2half2_rn(v[2], v[3]);
                h[2 * k] = *reinterpret_cast<const uint32_t*>(&p0);
                h[2 * k + 1] = *reinterpret_cast<const uint32_t*>(&p1);
            } else {
                h[2 * k] = (uint32_t)f2h_bits(v[0]) | ((uint32_t)f2h_bits(v[1]) << 16);
                h[2 * k + 1] = (uint32_t)f2h_bits(v[2]) | ((uint32_t)f2h_bits(v[3]) << 16);
            }
        }
    }
}


}  // namespace tk
