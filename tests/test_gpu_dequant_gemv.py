"""GPU parity: dequant (bit-exact) and decode GEMV (tolerance vs fp64) through
the C ABI against the golden vectors and the CPU oracle."""
import numpy as np
import pytest

from conftest import GOLDEN
from gen import blocks_for, rel_fro

pytestmark = pytest.mark.gpu

DQ = np.load(GOLDEN / "dequant_golden.npz")
NAMES = sorted({k.rsplit("_", 1)[0] for k in DQ.files if k.endswith("_type")})


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("name", NAMES)
def test_dequant_golden_bit_exact(ctx, name):
    import torch
    import tier_b200 as tk
    b = DQ[f"{name}_blocks"]
    t = int(DQ[f"{name}_type"])
    R, C = DQ[f"{name}_f32"].shape
    if name.startswith(("IQ1", "IQ2", "IQ3")):
        pytest.importorskip("gguf")
        ctx.set_iq_grids()          # lattice tables from gguf-py (= tier/quant_tables.h)
    bd = dev(b)
    o32 = torch.empty(R, C, dtype=torch.float32, device="cuda")
    ctx.dequant(t, bd, R, C, o32, out_dtype=tk.DT_F32)
    assert np.array_equal(host(o32).view(np.uint32), DQ[f"{name}_f32"].view(np.uint32)), name
    o16 = torch.empty(R, C, dtype=torch.float16, device="cuda")
    ctx.dequant(t, bd, R, C, o16, out_dtype=tk.DT_F16)
    assert np.array_equal(host(o16).view(np.uint16), DQ[f"{name}_f16"]), name
    ob = torch.empty(R, C, dtype=torch.bfloat16, device="cuda")
    ctx.dequant(t, bd, R, C, ob, out_dtype=tk.DT_BF16)
    want_bf = torch.from_numpy(DQ[f"{name}_f32"]).to(torch.bfloat16).view(torch.int16).numpy()
    assert np.array_equal(host(ob.view(torch.int16)), want_bf), name
    ctx.sync_status()


@pytest.mark.parametrize("qtype", [8, 12, 13, 14, 2, 10, 11])
def test_dequant_large_rows_and_offset(ctx, oracle, qtype):
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(100 + qtype)
    R, C = 96, 4096
    b = blocks_for(rng, qtype, R, C)
    want = oracle.dequant(b, qtype, R, C, 0)
    bd = dev(b)
    out = torch.empty(R - 5, C, dtype=torch.float32, device="cuda")
    ctx.dequant(qtype, bd, R - 5, C, out, r0=5)
    assert np.array_equal(host(out).view(np.uint32), want[5:].view(np.uint32))
    o16 = torch.empty(R, C, dtype=torch.float16, device="cuda")
    ctx.dequant(qtype, bd, R, C, o16, out_dtype=tk.DT_F16)
    assert np.array_equal(host(o16).view(np.uint16), oracle.dequant(b, qtype, R, C, 1))


@pytest.mark.parametrize("qtype,N,K", [(8, 4096, 4096), (12, 1024, 4096), (13, 512, 5120), (1, 768, 3840),
                                        (30, 256, 2048), (0, 256, 1024), (14, 256, 2048), (2, 256, 2048),
                                        # fewer rows than SMs, ragged slots, shared-memory ring reuse
                                        (8, 100, 256), (8, 32768, 1024), (12, 20000, 2048), (13, 9000, 1280),
                                        # Q6_K: one chunk, 7 chunks of 2048, and 16-byte-unaligned rows (scalar kernel)
                                        (14, 4096, 4096), (14, 3000, 14336), (14, 700, 5120),
                                        # several K-chunks per row group and few slots per ring
                                        (8, 5120, 14336), (12, 5120, 14336),
                                        # one-token Q8_0 dp4a kernel (>= 32 MB of weight): 1, 2 and 4 K
                                        # segments, a short last segment
                                        (8, 14336, 4096), (8, 7000, 5120), (8, 2300, 14336), (8, 4000, 8192)])
@pytest.mark.parametrize("M", [1, 2, 3, 16])
def test_gemv_vs_f64(ctx, oracle, qtype, N, K, M):
    import torch
    rng = np.random.default_rng(qtype * 31 + M)
    b = blocks_for(rng, qtype, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    ctx.gemv(qtype, dev(b), N, K, dev(x), y, M=M)
    got = host(y)
    ref = oracle.qgemm_f64(b, qtype, N, K, x)
    assert rel_fro(got, ref) < 2e-3             # stated decode tolerance; fp32 accumulation gives ~1e-7
    assert rel_fro(got, ref) < 1e-5
    ctx.sync_status()


def test_gemv_c1_matches_reference_order_closely(ctx, oracle):
    """C1: q8_0 4096x4096, M=1 -- also compare with the reference's own
    lane-stride / shuffle-tree summation order."""
    import torch
    rng = np.random.default_rng(0)
    N = K = 4096
    b = blocks_for(rng, 8, N, K)
    x = rng.standard_normal(K).astype(np.float32)
    y = torch.empty(1, N, dtype=torch.float32, device="cuda")
    ctx.gemv(8, dev(b), N, K, dev(x[None]), y)
    got = host(y)[0]
    ref_order = oracle.gemv_warp_order(b[:256], 8, 256, K, x)
    assert np.abs(got[:256] - ref_order).max() / np.abs(ref_order).max() < 1e-5


@pytest.mark.parametrize("qtype,K", [(8, 4096), (12, 4096), (14, 4096), (8, 6144)])
def test_gemv_frozen_chain(ctx, oracle, qtype, K):
    """TK_WFROZEN lets a GEMV fetch its (never written) weight before the
    previous kernel ends, but x is still read after it: a chain whose x is
    the previous GEMV's y gives the same bits as the chain without the flag."""
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(9 + qtype)
    bs = [dev(blocks_for(rng, qtype, K, K)) for _ in range(3)]
    x0 = dev(rng.standard_normal((1, K)).astype(np.float32))
    outs = []
    for flag in (0, tk.WFROZEN):
        ys = [torch.empty(1, K, device="cuda") for _ in bs]
        x = x0
        for b, y in zip(bs, ys):
            ctx.gemv(qtype | flag, b, K, K, x, y)
            x = y
        outs.append([host(y) for y in ys])
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    ctx.sync_status()


@pytest.mark.gpu
@pytest.mark.parametrize("qtype,N,K", [(8, 4096, 5120), (12, 3000, 14336), (13, 700, 4096), (8, 100, 2048),
                                        (14, 3000, 14336), (14, 1000, 4096)])
@pytest.mark.parametrize("M", [5, 8, 9, 13, 10])
def test_gemv_tokens_3_to_16(ctx, oracle, qtype, N, K, M):
    """3..16 tokens: x records streamed with the weight, W read once (both
    token halves in one launch) or, for Q6_K beyond 8 tokens, once per half;
    ragged row groups; a 2-token remainder (M = 10 on Q6_K)."""
    import torch
    rng = np.random.default_rng(qtype * 7 + M)
    b = blocks_for(rng, qtype, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[1] *= 1e-3                                  # per-token scaling
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    n0 = ctx.launches()
    ctx.gemv(qtype, dev(b), N, K, dev(x), y, M=M)
    if qtype != 14 or M <= 8:
        assert ctx.launches() - n0 == 2           # x records + one GEMV
    got = host(y)
    ref = oracle.qgemm_f64(b, qtype, N, K, x)
    assert rel_fro(got, ref) < 1e-5
    assert rel_fro(got[1], ref[1]) < 1e-5
    ctx.sync_status()


@pytest.mark.parametrize("qtype", [8, 12])
@pytest.mark.parametrize("M", [1, 2, 3, 9])
@pytest.mark.parametrize("bad", [float("nan"), float("inf")])
def test_gemv_nonfinite_x(ctx, oracle, qtype, M, bad):
    """A NaN or inf in one token's x makes that token's y non-finite, as the
    reference's fp32 sum does; the other tokens are unaffected."""
    import torch
    rng = np.random.default_rng(17 + M)
    N, K = 600, 4096
    b = blocks_for(rng, qtype, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[M - 1, 1234] = bad
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ctx.gemv(qtype, dev(b), N, K, dev(x), y, M=M)
    got = host(y)
    assert not np.isfinite(got[M - 1]).any()
    if M > 1:
        ref = oracle.qgemm_f64(b, qtype, N, K, x[: M - 1])
        assert rel_fro(got[: M - 1], ref) < 1e-5
    ctx.sync_status()


@pytest.mark.parametrize("qtype", [8, 12, 14])
@pytest.mark.parametrize("M", [1, 2, 5])
def test_gemv_multi_segments(ctx, oracle, qtype, M):
    """tk_gemv_multi: weights sharing x (q/k/v-like row counts, boundaries
    inside row groups and SM ranges) give each weight's own GEMV result; 5
    tokens take the per-weight path."""
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(40 + qtype + M)
    K = 4096
    rows = [700, 130, 129]
    bs = [blocks_for(rng, qtype, n, K) for n in rows]
    x = rng.standard_normal((M, K)).astype(np.float32)
    ys = [torch.full((M, n), float("nan"), device="cuda") for n in rows]
    n0 = ctx.launches()
    ctx.gemv_multi(qtype | tk.WFROZEN, [dev(b) for b in bs], rows, ys, K, dev(x), M=M)
    if M <= 2:
        assert ctx.launches() - n0 == 1
    for b, n, y in zip(bs, rows, ys):
        ref = oracle.qgemm_f64(b, qtype, n, K, x)
        assert rel_fro(host(y), ref) < 1e-5
    ctx.sync_status()
