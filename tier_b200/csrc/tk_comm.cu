// tk_comm.cu -- peer buffers over CUDA IPC and the reduce-scatter that the
// dX GEMM performs through them (tk_linear_dx_rs).
//
// The reference all-reduces nothing (it runs on one GPU); sharding W by
// output rows makes dX = sum over ranks of dY_g . W_g, and a consumer that
// takes dX split by token rows (sequence-parallel) needs only its rows of
// that sum: a reduce-scatter.  Instead of a GEMM followed by a collective,
// the GEMM's epilogue stores every finished tile straight into the owning
// rank's receive buffer (peer memory, NVLink), so the transfer overlaps the
// remaining tiles' MMAs.  The owner then adds the world slots in rank order
// (deterministic) into its output.
//
// Each rank's buffer (same layout on every rank):
//   [0, 64)      done[2][8]  int: done[p][src] = epoch, written by rank src
//   [256, 288)   ack[8]      int: ack[owner] = epoch, written by rank owner
//   [512]        CTA counter of this rank's GEMM launch (local)
//   [516]        block counter of this rank's reduce launch (local)
//   [4096, ...)  recv[2][world][rpo][K] fp32, parity p = epoch & 1
// A launch with epoch e writes recv[e & 1] of every owner; it first waits
// until every owner acknowledged epoch e - 2 (the previous use of that
// parity).  Every wait is bounded (2 s, status TK_ERR_TIMEOUT).
#include "tk_device.cuh"
#include "tk_internal.h"

#include <cstring>
#include <utility>
#include <vector>

struct tk_comm_state {
    int rank = 0, world = 0;
    uint8_t* buf = nullptr;
    size_t recv_bytes = 0;                 // one parity: world * rpo * K * 4 (= M * K * 4)
    uint8_t* peer[tk::TK_MAX_RANKS] = {};  // peer[rank] = buf
    bool connected = false;
    uint32_t epoch = 0;
};

namespace tk {

constexpr size_t kHdr = 4096;
constexpr size_t kDoneOff = 0, kAckOff = 256, kGemmCtr = 512, kRedCtr = 516;

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_c(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait until *p >= want; false (and DEV_TIMEOUT) after 2 s.
__device__ bool wait_ge(const int* p, int want, int* status) {
    if (ld_acquire_sys(p) >= want) return true;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(p) < want) {
        __nanosleep(200);
        if (globaltimer() - t0 > kWaitLimitNs) {
            raise_status(status, DEV_TIMEOUT);
            return false;
        }
    }
    return true;
}

__global__ void rs_wait_ack_kernel(const int* ack, int world, int need, int* status) {
    if (threadIdx.x != 0) return;
    for (int o = 0; o < world; ++o)
        if (!wait_ge(ack + o, need, status)) return;
}

// out[r, c] = sum_src recv[src][r][c] (src in rank order); grid-stride over
// float4s.  The last block to finish acknowledges the epoch to every rank.
__global__ void rs_reduce_kernel(const int* done, const float* recv, int world, int rpo, int K, float* out,
                                 long ldo, int epoch, int* red_ctr, int* const* peer_ack, int me, int* status) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        int good = 1;
        for (int src = 0; src < world && good; ++src) good = wait_ge(done + src, epoch, status);
        ok = good;
    }
    __syncthreads();
    if (ok) {
        const size_t slot = (size_t)rpo * K;
        const int k4 = K / 4;
        const long n4 = (long)rpo * k4;
        for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
            const int r = (int)(i / k4), c = (int)(i - (long)r * k4) * 4;
            float4 acc = *reinterpret_cast<const float4*>(recv + (size_t)r * K + c);
            for (int src = 1; src < world; ++src) {
                const float4 v = *reinterpret_cast<const float4*>(recv + src * slot + (size_t)r * K + c);
                acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
            }
            *reinterpret_cast<float4*>(out + (size_t)r * ldo + c) = acc;
        }
    }
    // acknowledge only a completed reduction: without it the senders' next
    // use of this parity times out instead of overwriting unread data
    __syncthreads();
    if (threadIdx.x == 0 && ok) {
        __threadfence_system();
        const int old = atomicAdd(red_ctr, 1);
        if (old == (int)gridDim.x - 1) {
            *red_ctr = 0;
            __threadfence_system();
            for (int o = 0; o < world; ++o) st_release_sys_c(peer_ack[o] + me, epoch);
        }
    }
}

static int* hdr_int(uint8_t* base, size_t off) { return reinterpret_cast<int*>(base + off); }

tk_status rs_begin(tk_ctx* ctx, int M, int K, RsDesc& rs, cudaStream_t s) {
    tk_comm_state* c = ctx->comm;
    if (!c || !c->connected) return fail(TK_ERR_INVALID, "reduce-scatter: tk_comm_init / tk_comm_connect first");
    const int W = c->world;
    if (M % W || (M / W) % 256) return fail(TK_ERR_INVALID, "reduce-scatter: M / world must be a multiple of 256");
    if (K % 4) return fail(TK_ERR_INVALID, "reduce-scatter: K must be a multiple of 4");
    if ((size_t)M * K * 4 > c->recv_bytes) return fail(TK_ERR_INVALID, "reduce-scatter: M * K exceeds the comm buffer");
    const int epoch = (int)++c->epoch;
    const int par = epoch & 1;
    const int rpo = M / W;
    rs = RsDesc();
    rs.world = W;
    rs.rpo = rpo;
    rs.epoch = epoch;
    rs.counter = hdr_int(c->buf, kGemmCtr);
    for (int o = 0; o < W; ++o) {
        float* recv = reinterpret_cast<float*>(c->peer[o] + kHdr + (size_t)par * c->recv_bytes);
        rs.dst[o] = recv + (size_t)c->rank * rpo * K;             // my slot in owner o's buffer
        rs.done[o] = hdr_int(c->peer[o], kDoneOff) + par * 8 + c->rank;
    }
    // the parity this launch overwrites was last read for epoch - 2
    rs_wait_ack_kernel<<<1, 32, 0, s>>>(hdr_int(c->buf, kAckOff), W, epoch - 2, ctx->status);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "reduce-scatter ack wait launch");
}

tk_status rs_finish(tk_ctx* ctx, const RsDesc& rs, int K, float* out, long ldo, cudaStream_t s) {
    tk_comm_state* c = ctx->comm;
    const int par = rs.epoch & 1;
    const float* recv = reinterpret_cast<const float*>(c->buf + kHdr + (size_t)par * c->recv_bytes);
    // peer ack pointers live in device memory for the kernel: the header's
    // tail holds them (written once at connect)
    int* const* peer_ack = reinterpret_cast<int* const*>(c->buf + 1024);
    const long n4 = (long)rs.rpo * (K / 4);
    int blocks = (int)((n4 + 255) / 256);
    if (blocks > 4 * ctx->num_sms) blocks = 4 * ctx->num_sms;
    ProfScope ps(ctx, s, PK_COMM);
    rs_reduce_kernel<<<blocks, 256, 0, s>>>(hdr_int(c->buf, kDoneOff) + par * 8, recv, rs.world, rs.rpo, K, out, ldo,
                                           rs.epoch, hdr_int(c->buf, kRedCtr), peer_ack, c->rank, ctx->status);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "reduce-scatter reduce launch");
}

// ---------------------------------------------------------------------------
// Collectives on the same buffers (no NCCL): an exchange of epoch e copies
// every rank's contribution into slot `rank` of parity (e & 1) of every rank's
// receive region, publishes done[e & 1][rank] to every rank, and each rank
// consumes its own region and acknowledges -- the reduce-scatter's protocol,
// so both kinds share epochs, flags and acks and may follow each other in any
// order, as long as every rank issues the same sequence.
struct CmPush {
    uint4* dst[TK_MAX_RANKS];    // per rank: my slot in its receive region (this parity)
    int* done[TK_MAX_RANKS];     // per rank: its done flag for me (this parity)
    int world, epoch;
    int* counter;                // blocks finished (local), reset by the last
};

__global__ void cm_push_kernel(const __grid_constant__ CmPush a, const uint4* __restrict__ src, size_t n16) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x) {
        const uint4 v = src[i];
        for (int o = 0; o < a.world; ++o) a.dst[o][i] = v;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int old = atomicAdd(a.counter, 1);
        if (old == (int)gridDim.x - 1) {
            *a.counter = 0;
            __threadfence_system();
            for (int o = 0; o < a.world; ++o) st_release_sys_c(a.done[o], a.epoch);
        }
    }
}

struct CmConsume {
    const int* done;             // my done flags of this parity, [world]
    int* red_ctr;
    int* const* peer_ack;        // device table of every rank's ack array
    int world, epoch, me;
    int* status;
};

// Wait (thread 0, bounded) until every rank's contribution arrived.
__device__ bool cm_wait_all(const CmConsume& c) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        int good = 1;
        for (int src = 0; src < c.world && good; ++src) good = wait_ge(c.done + src, c.epoch, c.status);
        ok = good;
    }
    __syncthreads();
    return ok != 0;
}
// After the block consumed its part: the last block acknowledges the epoch to every rank.
__device__ void cm_ack(const CmConsume& c, bool ok) {
    __syncthreads();
    if (threadIdx.x == 0 && ok) {
        __threadfence_system();
        const int old = atomicAdd(c.red_ctr, 1);
        if (old == (int)gridDim.x - 1) {
            *c.red_ctr = 0;
            __threadfence_system();
            for (int o = 0; o < c.world; ++o) st_release_sys_c(c.peer_ack[o] + c.me, c.epoch);
        }
    }
}

// all-gather: dst = the world slots in rank order
__global__ void cm_gather_kernel(const __grid_constant__ CmConsume c, const uint4* __restrict__ recv, size_t n16_all,
                                 uint4* __restrict__ dst) {
    const bool ok = cm_wait_all(c);
    if (ok)
        for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16_all; i += (size_t)gridDim.x * blockDim.x)
            dst[i] = recv[i];
    cm_ack(c, ok);
}

// all-reduce: out[i] = sum of the world slots' element i, in rank order
__global__ void cm_sum_kernel(const __grid_constant__ CmConsume c, const float4* __restrict__ recv, size_t n4,
                              float4* __restrict__ out) {
    const bool ok = cm_wait_all(c);
    if (ok)
        for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
            float4 acc = recv[i];
            for (int r = 1; r < c.world; ++r) {
                const float4 v = recv[(size_t)r * n4 + i];
                acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
            }
            out[i] = acc;
        }
    cm_ack(c, ok);
}

// LM-head vocabulary-shard merge.  Slot layout per rank (n rows, padded to
// 16 bytes per array): rmax f64 [n], rsum f64 [n], amax i32 [n], tgt f32 [n].
__host__ __device__ inline size_t lm_pack_bytes(int n) {
    return ((size_t)n * 8 + 15) / 16 * 16 * 2 + ((size_t)n * 4 + 15) / 16 * 16 * 2;
}
__global__ void lm_pack_kernel(int n, const double* rmax, const double* rsum, const int32_t* amax, const float* tgt,
                               uint8_t* out) {
    const size_t o1 = ((size_t)n * 8 + 15) / 16 * 16, o2 = 2 * o1, o3 = o2 + ((size_t)n * 4 + 15) / 16 * 16;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += gridDim.x * blockDim.x) {
        reinterpret_cast<double*>(out)[t] = rmax[t];
        reinterpret_cast<double*>(out + o1)[t] = rsum[t];
        reinterpret_cast<int32_t*>(out + o2)[t] = amax[t];
        reinterpret_cast<float*>(out + o3)[t] = tgt[t];
    }
}
// Every rank computes the same merged row from the gathered slots (rank order
// = vocabulary order): max; sum of rsum_r * exp(rmax_r - max); the argmax of
// the first rank that reaches the max; sum of the target logits.  The local
// single-pass accumulator row is rescaled by exp(rmax_local - max).
__global__ void lm_merge_kernel(const __grid_constant__ CmConsume c, const uint8_t* __restrict__ recv, int n,
                                size_t slot, int me, double* rmax, double* rsum, int32_t* amax, float* tgt, float* dX,
                                int H) {
    const bool ok = cm_wait_all(c);
    const size_t o1 = ((size_t)n * 8 + 15) / 16 * 16, o2 = 2 * o1, o3 = o2 + ((size_t)n * 4 + 15) / 16 * 16;
    if (ok)
        for (int t = blockIdx.x; t < n; t += gridDim.x) {
            double m = -1e300;
            int best = 0;
            for (int r = 0; r < c.world; ++r) {
                const double v = reinterpret_cast<const double*>(recv + r * slot)[t];
                if (v > m) { m = v; best = r; }
            }
            const double mine = reinterpret_cast<const double*>(recv + me * slot)[t];
            if (dX) {
                const float f = (float)exp(mine - m);
                for (int h = threadIdx.x; h < H; h += blockDim.x) dX[(size_t)t * H + h] *= f;
            }
            __syncthreads();    // every thread has read this row's state before thread 0 rewrites it
            if (threadIdx.x == 0) {
                double s = 0.0;
                float tg = 0.0f;
                for (int r = 0; r < c.world; ++r) {
                    const uint8_t* b = recv + r * slot;
                    s += reinterpret_cast<const double*>(b + o1)[t] * exp(reinterpret_cast<const double*>(b)[t] - m);
                    tg += reinterpret_cast<const float*>(b + o3)[t];
                }
                rmax[t] = m;
                rsum[t] = s;
                amax[t] = reinterpret_cast<const int32_t*>(recv + best * slot + o2)[t];
                tgt[t] = tg;
            }
        }
    cm_ack(c, ok);
}

// Column shards to row shards: rank g holds A[M, n] (its columns g*n ..
// (g+1)*n of a [M, world*n] matrix, row stride ld_src bytes) and sends rows
// h*M/world .. of it to rank h, packed (row_bytes = n * element bytes).
// Column shards to row shards: rank g holds A[M, n] (its columns g*n ..
// (g+1)*n of a [M, world*n] matrix, row stride ld_src bytes) and sends rows
// h*M/world .. of it to rank h, packed (row_bytes = n * element bytes).  Four
// 16-byte loads are in flight per thread before their stores.
__global__ void cm_push_rows_kernel(const __grid_constant__ CmPush a, const uint8_t* __restrict__ src, size_t ld_src,
                                    int rows_per, size_t row_bytes) {
    const size_t nv = row_bytes / 16, total = (size_t)rows_per * a.world * nv;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i0 = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i0 < total; i0 += 4 * stride) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const size_t i = i0 + u * stride;
            if (i < total) {
                const size_t rg = i / nv, c = i - rg * nv;
                v[u] = *reinterpret_cast<const uint4*>(src + rg * ld_src + c * 16);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const size_t i = i0 + u * stride;
            if (i < total) {
                const size_t rg = i / nv, c = i - rg * nv;
                const int h = (int)(rg / rows_per), r = (int)(rg - (size_t)h * rows_per);
                a.dst[h][(size_t)r * nv + c] = v[u];
            }
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int old = atomicAdd(a.counter, 1);
        if (old == (int)gridDim.x - 1) {
            *a.counter = 0;
            __threadfence_system();
            for (int o = 0; o < a.world; ++o) st_release_sys_c(a.done[o], a.epoch);
        }
    }
}

// ... and assembles its rows: dst[r, g*n + c] = slot g [r, c] (row stride ld_dst bytes).
__global__ void cm_rows_kernel(const __grid_constant__ CmConsume c, const uint8_t* __restrict__ recv, int rows_per,
                               size_t row_bytes, uint8_t* __restrict__ dst, size_t ld_dst) {
    const bool ok = cm_wait_all(c);
    const size_t nv = row_bytes / 16, slot = (size_t)rows_per * row_bytes;
    const size_t total = (size_t)c.world * rows_per * nv;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    if (ok)
        for (size_t i0 = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i0 < total; i0 += 4 * stride) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (i0 + u * stride < total) v[u] = reinterpret_cast<const uint4*>(recv)[i0 + u * stride];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const size_t i = i0 + u * stride;
                if (i < total) {
                    const size_t gr = i / nv, cc = i - gr * nv;
                    const int g = (int)(gr / rows_per), r = (int)(gr - (size_t)g * rows_per);
                    *reinterpret_cast<uint4*>(dst + (size_t)r * ld_dst + g * row_bytes + cc * 16) = v[u];
                }
            }
        }
    cm_ack(c, ok);
    (void)slot;
}

// Start an exchange of `slot` bytes per rank: capacity check, epoch, wait for
// the acks of the parity's previous use, push `src` into every rank's region.
static tk_status cm_start(tk_ctx* ctx, const void* src, size_t slot, CmConsume& c, const uint8_t** recv,
                          cudaStream_t s, const uint8_t* rows_src = nullptr, size_t ld_src = 0, int rows_per = 0,
                          size_t row_bytes = 0) {
    tk_comm_state* cs = ctx->comm;
    if (!cs || !cs->connected) return fail(TK_ERR_INVALID, "collective: tk_comm_init / tk_comm_connect first");
    if (slot % 16 || (reinterpret_cast<uintptr_t>(rows_src ? rows_src : src) & 15))
        return fail(TK_ERR_INVALID, "collective: 16-byte aligned data and sizes required");
    if (slot * cs->world > cs->recv_bytes)
        return fail(TK_ERR_INVALID, "collective: world * bytes exceeds the recv_bytes given to tk_comm_init");
    const int epoch = (int)++cs->epoch;
    const int par = epoch & 1;
    rs_wait_ack_kernel<<<1, 32, 0, s>>>(hdr_int(cs->buf, kAckOff), cs->world, epoch - 2, ctx->status);
    ctx->launches++;
    CmPush a;
    for (int o = 0; o < cs->world; ++o) {
        a.dst[o] = reinterpret_cast<uint4*>(cs->peer[o] + kHdr + (size_t)par * cs->recv_bytes + (size_t)cs->rank * slot);
        a.done[o] = hdr_int(cs->peer[o], kDoneOff) + par * 8 + cs->rank;
    }
    a.world = cs->world;
    a.epoch = epoch;
    a.counter = hdr_int(cs->buf, kGemmCtr);
    const size_t n16 = rows_src ? slot / 16 * cs->world : slot / 16;
    int blocks = (int)((n16 + 255) / 256);
    if (blocks > 2 * ctx->num_sms) blocks = 2 * ctx->num_sms;
    if (blocks < 1) blocks = 1;
    ProfScope ps(ctx, s, PK_COMM);
    if (rows_src) cm_push_rows_kernel<<<blocks, 256, 0, s>>>(a, rows_src, ld_src, rows_per, row_bytes);
    else cm_push_kernel<<<blocks, 256, 0, s>>>(a, static_cast<const uint4*>(src), n16);
    ctx->launches++;
    c.done = hdr_int(cs->buf, kDoneOff) + par * 8;
    c.red_ctr = hdr_int(cs->buf, kRedCtr);
    c.peer_ack = reinterpret_cast<int* const*>(cs->buf + 1024);
    c.world = cs->world;
    c.epoch = epoch;
    c.me = cs->rank;
    c.status = ctx->status;
    *recv = cs->buf + kHdr + (size_t)par * cs->recv_bytes;
    return cuda_fail(cudaGetLastError(), "collective push launch");
}

static int cm_blocks(tk_ctx* ctx, size_t n) {
    size_t b = (n + 255) / 256;
    if (b > (size_t)(2 * ctx->num_sms)) b = 2 * ctx->num_sms;
    return b < 1 ? 1 : (int)b;
}

void comm_destroy(tk_ctx* ctx) {
    tk_comm_state* c = ctx->comm;
    if (!c) return;
    for (int o = 0; o < c->world; ++o)
        if (c->peer[o] && o != c->rank) cudaIpcCloseMemHandle(c->peer[o]);
    if (c->buf) cudaFree(c->buf);
    delete c;
    ctx->comm = nullptr;
}

}  // namespace tk

using namespace tk;

extern "C" {

tk_status tk_comm_init(tk_ctx* ctx, int rank, int world, size_t recv_bytes, void* handle_out) {
    if (!ctx || !handle_out) return fail(TK_ERR_INVALID, "tk_comm_init: null argument");
    if (world < 1 || world > TK_MAX_RANKS || rank < 0 || rank >= world)
        return fail(TK_ERR_INVALID, "tk_comm_init: rank / world out of range (world <= 8)");
    if (recv_bytes == 0 || recv_bytes % 256) return fail(TK_ERR_INVALID, "tk_comm_init: recv_bytes must be a positive multiple of 256");
    cudaSetDevice(ctx->device);
    comm_destroy(ctx);
    tk_comm_state* c = new tk_comm_state();
    c->rank = rank;
    c->world = world;
    c->recv_bytes = recv_bytes;
    cudaError_t e = cudaMalloc(&c->buf, kHdr + 2 * recv_bytes);
    if (e == cudaSuccess) e = cudaMemset(c->buf, 0, kHdr);
    if (e != cudaSuccess) {
        if (c->buf) cudaFree(c->buf);
        delete c;
        return cuda_fail(e, "tk_comm_init: buffer");
    }
    c->peer[rank] = c->buf;
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, c->buf);
    if (e != cudaSuccess) {
        cudaFree(c->buf);
        delete c;
        return cuda_fail(e, "tk_comm_init: IPC handle");
    }
    memcpy(handle_out, &h, sizeof(h));
    ctx->comm = c;
    return TK_OK;
}

tk_status tk_comm_connect(tk_ctx* ctx, const void* handles) {
    if (!ctx || !handles) return fail(TK_ERR_INVALID, "tk_comm_connect: null argument");
    tk_comm_state* c = ctx->comm;
    if (!c) return fail(TK_ERR_INVALID, "tk_comm_connect: tk_comm_init first");
    cudaSetDevice(ctx->device);
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (int o = 0; o < c->world; ++o) {
        if (o == c->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + (size_t)o * TK_IPC_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return fail(TK_ERR_CUDA, "tk_comm_connect: open peer buffer " + std::to_string(o) + ": " + cudaGetErrorString(e));
        c->peer[o] = static_cast<uint8_t*>(p);
    }
    // the reduce kernel reads the owners' ack addresses from device memory
    int* acks[TK_MAX_RANKS] = {};
    for (int o = 0; o < c->world; ++o) acks[o] = reinterpret_cast<int*>(c->peer[o] + kAckOff);
    cudaError_t e = cudaMemcpy(c->buf + 1024, acks, sizeof(acks), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "tk_comm_connect: ack table");
    c->connected = true;
    return TK_OK;
}

tk_status tk_allgather(tk_ctx* ctx, const void* src, size_t bytes, void* dst, void* stream) {
    if (!ctx || (bytes && (!src || !dst))) return fail(TK_ERR_INVALID, "tk_allgather: null argument");
    if (reinterpret_cast<uintptr_t>(dst) & 15) return fail(TK_ERR_INVALID, "tk_allgather: dst must be 16-byte aligned");
    if (bytes == 0) return TK_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    CmConsume c;
    const uint8_t* recv = nullptr;
    tk_status st = cm_start(ctx, src, bytes, c, &recv, s);
    if (st != TK_OK) return st;
    const size_t n16 = bytes / 16 * c.world;
    ProfScope ps(ctx, s, PK_COMM);
    cm_gather_kernel<<<cm_blocks(ctx, n16), 256, 0, s>>>(c, reinterpret_cast<const uint4*>(recv), n16,
                                                        static_cast<uint4*>(dst));
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "tk_allgather launch");
}

// The send half records its exchange here for the receive half.
struct ReshardPending {
    bool open = false;
    CmConsume c;
    const uint8_t* recv = nullptr;
    int rows_per = 0;
    size_t row_bytes = 0;
};
static ReshardPending& reshard_pending(tk_ctx* ctx) {
    static thread_local std::vector<std::pair<tk_ctx*, ReshardPending>> table;
    for (auto& e : table)
        if (e.first == ctx) return e.second;
    table.emplace_back(ctx, ReshardPending());
    return table.back().second;
}

tk_status tk_reshard_cols_send(tk_ctx* ctx, const void* src, int M, int n, size_t ld_src, int elem_bytes,
                               void* stream) {
    if (!ctx || !src) return fail(TK_ERR_INVALID, "tk_reshard_cols_send: null argument");
    tk_comm_state* cs = ctx->comm;
    if (!cs || !cs->connected) return fail(TK_ERR_INVALID, "tk_reshard_cols_send: tk_comm_init / tk_comm_connect first");
    if (M <= 0 || n <= 0 || elem_bytes <= 0 || M % cs->world)
        return fail(TK_ERR_INVALID, "tk_reshard_cols_send: M must be a positive multiple of world");
    const size_t row_bytes = (size_t)n * elem_bytes;
    if (row_bytes % 16 || (ld_src * elem_bytes) % 16 || ld_src < (size_t)n)
        return fail(TK_ERR_INVALID, "tk_reshard_cols_send: rows of whole 16-byte units and a 16-byte aligned source");
    ReshardPending& pe = reshard_pending(ctx);
    if (pe.open) return fail(TK_ERR_INVALID, "tk_reshard_cols_send: the previous exchange was not received");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int rows_per = M / cs->world;
    tk_status st = cm_start(ctx, nullptr, (size_t)rows_per * row_bytes, pe.c, &pe.recv, s,
                            static_cast<const uint8_t*>(src), ld_src * elem_bytes, rows_per, row_bytes);
    if (st != TK_OK) return st;
    pe.open = true;
    pe.rows_per = rows_per;
    pe.row_bytes = row_bytes;
    return TK_OK;
}

tk_status tk_reshard_cols_recv(tk_ctx* ctx, void* dst, size_t ld_dst, int elem_bytes, void* stream) {
    if (!ctx || !dst || elem_bytes <= 0) return fail(TK_ERR_INVALID, "tk_reshard_cols_recv: null argument");
    ReshardPending& pe = reshard_pending(ctx);
    if (!pe.open) return fail(TK_ERR_INVALID, "tk_reshard_cols_recv: no exchange sent (tk_reshard_cols_send first)");
    if ((ld_dst * elem_bytes) % 16 || (reinterpret_cast<uintptr_t>(dst) & 15) ||
        ld_dst * elem_bytes < pe.row_bytes * ctx->comm->world)
        return fail(TK_ERR_INVALID, "tk_reshard_cols_recv: 16-byte aligned rows of at least world * n elements");
    pe.open = false;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t nv = (size_t)pe.c.world * pe.rows_per * (pe.row_bytes / 16);
    ProfScope ps(ctx, s, PK_COMM);
    cm_rows_kernel<<<cm_blocks(ctx, (nv + 3) / 4), 256, 0, s>>>(pe.c, pe.recv, pe.rows_per, pe.row_bytes,
                                                                 static_cast<uint8_t*>(dst), ld_dst * elem_bytes);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "tk_reshard_cols_recv launch");
}

tk_status tk_reshard_cols(tk_ctx* ctx, const void* src, int M, int n, size_t ld_src, int elem_bytes, void* dst,
                          size_t ld_dst, void* stream) {
    tk_status st = tk_reshard_cols_send(ctx, src, M, n, ld_src, elem_bytes, stream);
    if (st != TK_OK) return st;
    return tk_reshard_cols_recv(ctx, dst, ld_dst, elem_bytes, stream);
}

tk_status tk_allreduce_f32(tk_ctx* ctx, float* buf, size_t n, void* stream) {
    if (!ctx || (n && !buf)) return fail(TK_ERR_INVALID, "tk_allreduce_f32: null argument");
    if (n % 4) return fail(TK_ERR_INVALID, "tk_allreduce_f32: n must be a multiple of 4");
    if (n == 0) return TK_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    CmConsume c;
    const uint8_t* recv = nullptr;
    tk_status st = cm_start(ctx, buf, n * 4, c, &recv, s);
    if (st != TK_OK) return st;
    ProfScope ps(ctx, s, PK_COMM);
    cm_sum_kernel<<<cm_blocks(ctx, n / 4), 256, 0, s>>>(c, reinterpret_cast<const float4*>(recv), n / 4,
                                                        reinterpret_cast<float4*>(buf));
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "tk_allreduce_f32 launch");
}

tk_status tk_lmhead_merge(tk_ctx* ctx, int n, double* rmax, double* rsum, int32_t* amax, float* tgt, float* dX, int H,
                          void* stream) {
    if (!ctx || n < 0 || (n && (!rmax || !rsum || !amax || !tgt)))
        return fail(TK_ERR_INVALID, "tk_lmhead_merge: null argument");
    if (dX && H <= 0) return fail(TK_ERR_INVALID, "tk_lmhead_merge: H must be positive with dX");
    if (n == 0) return TK_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t slot = lm_pack_bytes(n);
    tk_status st = ws_ensure(ctx, slot, s);
    if (st != TK_OK) return st;
    uint8_t* pack = static_cast<uint8_t*>(ctx->ws);
    lm_pack_kernel<<<cm_blocks(ctx, (size_t)n), 256, 0, s>>>(n, rmax, rsum, amax, tgt, pack);
    ctx->launches++;
    CmConsume c;
    const uint8_t* recv = nullptr;
    st = cm_start(ctx, pack, slot, c, &recv, s);
    if (st != TK_OK) return st;
    int blocks = n < 4 * ctx->num_sms ? n : 4 * ctx->num_sms;
    ProfScope ps(ctx, s, PK_COMM);
    lm_merge_kernel<<<blocks, 128, 0, s>>>(c, recv, n, slot, c.me, rmax, rsum, amax, tgt, dX, H);
    ctx->launches++;
    return cuda_fail(cudaGetLastError(), "tk_lmhead_merge launch");
}

}  // extern "C"
