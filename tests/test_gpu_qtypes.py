"""GPU parity of the block types that have no dedicated decode kernel: the
legacy Q4_1 / Q5_0 / Q5_1 / Q2_K / Q3_K, the table-level IQ4_NL, IQ4_XS,
TQ1_0, TQ2_0, MXFP4, NF4, FP4 and the lattice IQ2_XXS, IQ2_XS, IQ2_S,
IQ3_XXS, IQ3_S, IQ1_S, IQ1_M (tier/quant.h:59-121; lattice tables registered
from gguf-py, the numbers of tier/quant_tables.h).  The reference's gemv_q
(tier/tier.cpp:300-306) and dq_k (294-298) decode every type through q_val;
here the same types go through the generic dequant / GEMV kernels, and the
linear path expands them to fp16 for the tensor-core GEMM.

Bars: dequant bit-exact with the CPU oracle (pinned to gguf-py 0.19.0 and the
reference's quant.h by tests/test_oracle.py and tests/test_qtypes_host.py);
GEMV within 1e-5 of fp64 (fp32 accumulation); linear within 2e-3 of fp64 (the
fp16 rounding of the expanded weight)."""
import numpy as np
import pytest

from gen import blocks_for, rel_fro

pytestmark = pytest.mark.gpu

LEGACY = [3, 6, 7, 10, 11]
TABLE = [20, 23, 34, 35, 39, 200, 201]
GRID = [16, 17, 22, 18, 21, 19, 29]


@pytest.fixture
def gctx(ctx):
    """The session context with the lattice tables registered."""
    pytest.importorskip("gguf")
    ctx.set_iq_grids()
    return ctx


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("qtype", TABLE + GRID)
def test_dequant_rows_offset_all_dtypes(gctx, oracle, qtype):
    ctx = gctx
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(300 + qtype)
    R, C = 72, 4096
    b = blocks_for(rng, qtype, R, C)
    bd = dev(b)
    out = torch.empty(R - 3, C, dtype=torch.float32, device="cuda")
    ctx.dequant(qtype, bd, R - 3, C, out, r0=3)
    assert np.array_equal(host(out).view(np.uint32), oracle.dequant(b, qtype, R, C, 0)[3:].view(np.uint32))
    o16 = torch.empty(R, C, dtype=torch.float16, device="cuda")
    ctx.dequant(qtype, bd, R, C, o16, out_dtype=tk.DT_F16)
    assert np.array_equal(host(o16).view(np.uint16), oracle.dequant(b, qtype, R, C, 1))
    ob = torch.empty(R, C, dtype=torch.bfloat16, device="cuda")
    ctx.dequant(qtype, bd, R, C, ob, out_dtype=tk.DT_BF16)
    assert np.array_equal(host(ob.view(torch.int16)), oracle.dequant(b, qtype, R, C, 2).view(np.int16))
    ctx.sync_status()


@pytest.mark.parametrize("qtype", LEGACY + TABLE + GRID)
@pytest.mark.parametrize("M", [1, 3, 16])
def test_gemv_every_type(gctx, oracle, qtype, M):
    ctx = gctx
    import torch
    rng = np.random.default_rng(400 + qtype * 7 + M)
    N, K = 300, 2048
    b = blocks_for(rng, qtype, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    ctx.gemv(qtype, dev(b), N, K, dev(x), y, M=M)
    assert rel_fro(host(y), oracle.qgemm_f64(b, qtype, N, K, x)) < 1e-5
    ctx.sync_status()


@pytest.mark.parametrize("qtype", [20, 35, 200])
def test_gemv_multi_falls_back_per_segment(ctx, oracle, qtype):
    import torch
    rng = np.random.default_rng(500 + qtype)
    K, rows = 1024, [96, 40]
    bs = [blocks_for(rng, qtype, n, K) for n in rows]
    x = rng.standard_normal((2, K)).astype(np.float32)
    ys = [torch.empty(2, n, dtype=torch.float32, device="cuda") for n in rows]
    ctx.gemv_multi(qtype, [dev(b) for b in bs], rows, ys, K, dev(x), M=2)
    for b, n, y in zip(bs, rows, ys):
        assert rel_fro(host(y), oracle.qgemm_f64(b, qtype, n, K, x)) < 1e-5
    ctx.sync_status()


@pytest.mark.parametrize("qtype", [20, 23, 34, 39, 201, 10, 16, 21, 29])
def test_linear_fwd_dx(gctx, oracle, qtype):
    ctx = gctx
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(600 + qtype)
    M, N, K = 256, 512, 1024
    b = blocks_for(rng, qtype, N, K)
    Wf = oracle.dequant(b, qtype, N, K, 0).astype(np.float64)
    Xb = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16)
    dYb = torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)).to(torch.bfloat16)
    w = tk.make_weight(qtype, N, K, dev(b))
    Y = torch.empty(M, N, dtype=torch.float32, device="cuda")
    ctx.linear(w, Xb.cuda(), M, Y, x_dtype=tk.DT_BF16)
    assert rel_fro(host(Y), Xb.float().numpy().astype(np.float64) @ Wf.T) < 2e-3
    dX = torch.empty(M, K, dtype=torch.float32, device="cuda")
    ctx.linear_dx(w, dYb.cuda(), M, dX, dy_dtype=tk.DT_BF16)
    assert rel_fro(host(dX), dYb.float().numpy().astype(np.float64) @ Wf) < 2e-3
    ctx.sync_status()


def test_grid_types_need_registered_tables():
    """A fresh context rejects the lattice types on the host (no launch) until
    tk_set_iq_grids has run; then the same call decodes bit-exactly."""
    import torch
    import tier_b200 as tk
    pytest.importorskip("gguf")
    from oracle.oracle import Oracle
    c = tk.Context(0)
    try:
        rng = np.random.default_rng(900)
        b = blocks_for(rng, 16, 8, 512)
        out = torch.empty(8, 512, dtype=torch.float32, device="cuda")
        with pytest.raises(tk.TierkError) as e:
            c.dequant(16, dev(b), 8, 512, out)
        assert e.value.status == tk.TK_ERR_UNSUPPORTED and "tk_set_iq_grids" in str(e.value)
        y = torch.empty(1, 8, dtype=torch.float32, device="cuda")
        with pytest.raises(tk.TierkError):
            c.gemv(16, dev(b), 8, 512, dev(np.ones((1, 512), np.float32)), y)
        c.set_iq_grids()
        c.dequant(16, dev(b), 8, 512, out)
        assert np.array_equal(host(out).view(np.uint32), Oracle().dequant(b, 16, 8, 512).view(np.uint32))
        c.sync_status()
    finally:
        torch.cuda.synchronize()
        c.close()
