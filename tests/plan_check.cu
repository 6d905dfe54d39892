// Host-side check of the decode GEMV launch plans (no GPU needed): every plan
// the kernels can be given fits shared memory, keeps bulk copies on 16-byte
// sizes and offsets and rows on bank-friendly strides, and the decode shapes
// of a 12B-class layer all get a plan.  Built and run by tests/test_plans.py.
#include "../tier_b200/csrc/tk_gemv5.cu"
#include "../tier_b200/csrc/tk_gemv6.cu"
#include "../tier_b200/csrc/tk_gemv7.cu"
#include "../tier_b200/csrc/tk_gemv8.cu"

#include <cstdio>

// the library's other translation units, reduced to what the plans link against
namespace tk {
tk_status fail(tk_status st, const std::string&) { return st; }
tk_status cuda_fail(cudaError_t e, const char*) { return e == cudaSuccess ? TK_OK : TK_ERR_CUDA; }
int prof_begin(tk_ctx*, cudaStream_t) { return -1; }
void prof_end(tk_ctx*, cudaStream_t, int, int) {}
tk_status ws_ensure(tk_ctx*, size_t, cudaStream_t) { return TK_OK; }
}  // namespace tk

using namespace tk;

static int g_bad = 0;
#define CHECK(cond, ...)                        \
    do {                                        \
        if (!(cond)) {                          \
            ++g_bad;                            \
            if (g_bad < 20) {                   \
                printf("FAIL %s: ", #cond);     \
                printf(__VA_ARGS__);            \
                printf("\n");                   \
            }                                   \
        }                                       \
    } while (0)

static size_t rowb(int t, int K) { return (size_t)K / (t == QT_Q8_0 ? 32 : 256) * (t == QT_Q8_0 ? 34 : t == QT_Q4_K ? 144 : t == QT_Q5_K ? 176 : 210); }

int main() {
    const int types[4] = {QT_Q8_0, QT_Q4_K, QT_Q5_K, QT_Q6_K};
    const int Ns[6] = {1, 100, 1024, 5120, 14336, 40000};
    long n1 = 0, n2 = 0, n3 = 0;
    for (int t : types)
        for (int K = 256; K <= 16384; K += 256)
            for (int N : Ns) {
                const int grid = N < 148 ? N : 148;
                const size_t rb = rowb(t, K);
                for (int M = 1; M <= 8; ++M) {            // fp16-MMA kernel
                    GmPlan p;
                    if (!gm_plan(t, N, K, M, grid, p)) continue;
                    ++n1;
                    CHECK(p.smem <= GM_SMEM_MAX + 1024, "gemv5 t %d K %d M %d smem %zu", t, K, M, p.smem);
                    CHECK(p.kcb % 16 == 0 && p.RS % 16 == 0 && p.RS % 128 == 32 && p.RS >= p.kcb,
                          "gemv5 t %d K %d kcb %u RS %u", t, K, p.kcb, p.RS);
                    CHECK(p.KC * p.nchunks == K && p.nslots >= 1 && p.nslots <= GM_MAXSLOTS, "gemv5 t %d K %d", t, K);
                }
                for (int M = 1; M <= 2; ++M)              // integer kernel, one matrix or segments
                    for (int whole = 0; whole <= 1; ++whole) {
                        GiPlan p;
                        if (rb % 16 || !gi_plan(t, N, K, rb, M, grid, p, whole != 0)) continue;
                        ++n2;
                        CHECK(p.smem <= GI_SMEM_MAX + 1024, "gemv6 t %d K %d M %d smem %zu", t, K, M, p.smem);
                        CHECK(p.kcb % 16 == 0 && p.KC * p.nchunks == K, "gemv6 t %d K %d kcb %u", t, K, p.kcb);
                        CHECK(p.teams >= 1 && p.teams <= 2 && p.nslots >= 1 && p.teams * p.nslots >= 2 &&
                                  p.teams * p.nslots <= GI_MAXSLOTS,
                              "gemv6 t %d K %d teams %d nslots %d", t, K, p.teams, p.nslots);
                        if (p.CS) {
                            CHECK(whole && p.nchunks == 1 && p.CS % 128 == 32 && p.CS >= 4 * p.kcb,
                                  "gemv6 t %d K %d CS %u", t, K, p.CS);
                        } else {
                            CHECK(p.RS % 128 == (t == QT_Q6_K ? 16u : 32u) && p.RS >= p.kcb, "gemv6 t %d K %d RS %u", t,
                                  K, p.RS);
                        }
                    }
                for (int M = 3; M <= 16; ++M) {           // x records streamed with the weight
                    GwPlan p;
                    if (rb % 16 || !gw_plan(t, N, K, rb, M, grid, p)) continue;
                    ++n3;
                    const int nh = M > 8 ? 2 : 1;
                    CHECK(p.smem <= GW_SMEM_MAX + 1024, "gemv7 t %d K %d M %d smem %zu", t, K, M, p.smem);
                    CHECK(p.kcb % 16 == 0 && p.KC * p.nchunks == K && p.KC % 256 == 0, "gemv7 t %d K %d", t, K);
                    CHECK(p.xoff % 128 == 0 && ((p.KC / 256) * gw_rec_bytes(nh)) % 16 == 0, "gemv7 t %d K %d xoff %u",
                          t, K, p.xoff);
                    CHECK(p.KC / 64 >= GW_CW / nh && p.nslots >= 1 && p.nslots <= GW_MAXSLOTS, "gemv7 t %d K %d M %d",
                          t, K, M);
                    CHECK(p.CS ? (p.nchunks == 1 && p.CS % 128 == 32) : (p.RS % 16 == 0 && p.RS >= p.kcb),
                          "gemv7 t %d K %d", t, K);
                }
            }
    // one-token dp4a kernel (Q8_0): segments cover K exactly, every bulk copy
    // (one row's segment) starts and ends on 16 bytes, warps divide into teams
    long n4 = 0;
    for (int K = 1024; K <= 65536; K += 1024)
        for (int N : Ns) {
            const int grid = N < 148 ? N : 148;
            GdPlan p;
            if (!gd_plan(N, K, rowb(QT_Q8_0, K), grid, p)) continue;
            ++n4;
            const int J = K / 1024;
            const int nused = (J + p.jseg - 1) / p.jseg;
            CHECK(p.smem <= GD_SMEM_MAX, "gemv8 K %d N %d smem %zu", K, N, p.smem);
            CHECK(GD_CW % p.nseg == 0 && p.jseg >= 1 && p.jseg <= GD_JMAX, "gemv8 K %d nseg %d jseg %d", K, p.nseg,
                  p.jseg);
            CHECK(nused <= p.nseg && (nused - 1) * p.jseg < J && nused * p.jseg >= J, "gemv8 K %d cover", K);
            CHECK(p.slot_bytes % 16 == 0 && (34u * 32u * p.jseg) % 16 == 0 && (34u * 32u * (J - (nused - 1) * p.jseg)) % 16 == 0,
                  "gemv8 K %d copy sizes", K);
            CHECK(p.x_off % 128 == 0 && p.xs_off % 16 == 0 && p.bar_off % 8 == 0, "gemv8 K %d offsets", K);
        }
    for (int K : {4096, 5120, 14336}) {
        GdPlan p;
        CHECK(gd_plan(14336, K, rowb(QT_Q8_0, K), 148, p), "no dp4a plan for K %d", K);
    }
    // every decode shape of a 12B-class layer (hidden 5120, q 4096, k/v 1024,
    // MLP 14336) has an integer plan: Q6_K needs 16-byte rows (K % 2048 == 0)
    const int Ks[3] = {4096, 5120, 14336};
    for (int t : types)
        for (int K : Ks) {
            const size_t rb = rowb(t, K);
            if (rb % 16) continue;
            for (int M = 1; M <= 2; ++M) {
                CHECK(gemv_imma_ok(t, rb, K, M), "no M<=2 plan t %d K %d M %d", t, K, M);
                CHECK(gemv_imma_multi_ok(t, rb, K, M), "no segment plan t %d K %d M %d", t, K, M);
            }
            for (int M = 3; M <= (t == QT_Q6_K ? 8 : 16); ++M)
                CHECK(gemv_wide_ok(t, rb, K, M), "no 3..16 plan t %d K %d M %d", t, K, M);
        }
    printf("plans checked: %ld fp16-MMA, %ld integer, %ld streamed-x, %ld dp4a; %d failures\n", n1, n2, n3, n4, g_bad);
    return g_bad ? 1 : 0;
}
