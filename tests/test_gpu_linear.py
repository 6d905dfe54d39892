"""GPU parity of the tensor-core linear path (tk_linear_fwd / tk_linear_dx)
against fp64 references, for every product set and weight kind.

Tolerances (relative Frobenius vs fp64):
  fp16 / quant-to-fp16 W with fp16 or bf16 activations (one product) : 2e-3
      (the stated bound for the bf16-activation quant GEMM; measured ~2e-4,
       the fp16 rounding of the dequantized W that the reference's training
       path applies too; fp16 W with fp16 X measures ~1e-6)
  x3 product sets with fp32 activations                              : 1e-5
"""
import numpy as np
import pytest

from gen import blocks_for, rel_fro

pytestmark = pytest.mark.gpu


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def f64(a):
    return np.asarray(a, np.float64)


SHAPES = [(128, 256, 64), (200, 300, 192), (384, 512, 1024), (1, 256, 512), (130, 1000, 520)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_fp16_single_product_fwd_dx(ctx, M, N, K):
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(M + N + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    X = rng.standard_normal((M, K)).astype(np.float16)
    dY = rng.standard_normal((M, N)).astype(np.float16)
    Wd = dev(W)
    w = tk.make_weight(tk.F16, N, K, Wd)
    Y = torch.empty(M, N, dtype=torch.float32, device="cuda")
    ctx.linear(w, dev(X), M, Y, x_dtype=tk.DT_F16, products=tk.X1)
    assert rel_fro(host(Y), f64(X) @ f64(W).T) < 1e-5
    dX = torch.empty(M, K, dtype=torch.float32, device="cuda")
    ctx.linear_dx(w, dev(dY), M, dX, dy_dtype=tk.DT_F16, products=tk.X1)
    assert rel_fro(host(dX), f64(dY) @ f64(W)) < 1e-5
    ctx.sync_status()


@pytest.mark.parametrize("M,N,K", SHAPES[:4] + [(256, 512, 5120), (128, 256, 14336)])
def test_x3_ref_products_fp32_activations(ctx, M, N, K):
    """The reference's fp3gemm: fp32 X split into h, m, l; single fp16 W."""
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(7 + M)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    X = rng.standard_normal((M, K)).astype(np.float32)
    dY = rng.standard_normal((M, N)).astype(np.float32)
    w = tk.make_weight(tk.F16, N, K, dev(W))
    Y = torch.empty(M, N, dtype=torch.float32, device="cuda")
    ctx.linear(w, dev(X), M, Y, products=tk.X3_REF)
    assert rel_fro(host(Y), f64(X) @ f64(W).T) < 1e-5
    dX = torch.empty(M, K, dtype=torch.float32, device="cuda")
    ctx.linear_dx(w, dev(dY), M, dX, products=tk.X3_REF)
    assert rel_fro(host(dX), f64(dY) @ f64(W)) < 1e-5
    # one fp16 product alone is far less accurate: the split is doing work
    Y1 = torch.empty(M, N, dtype=torch.float32, device="cuda")
    ctx.linear(w, dev(X), M, Y1, products=tk.X1)
    assert rel_fro(host(Y1), f64(X) @ f64(W).T) > 10 * rel_fro(host(Y), f64(X) @ f64(W).T)


@pytest.mark.parametrize("M,N,K", [(256, 512, 512), (200, 300, 192), (512, 1024, 5120), (256, 512, 14336)])
def test_x3_hhl_fp32_weight(ctx, M, N, K):
    """fp32 W split into fp16 hi/lo: Xh.Wh + Xh.Wl + Xl.Wh vs fp64 of fp32 W (<= 1e-5)."""
    import torch
    import tier_b200 as tk
    from tier_b200.host import LinearPath
    rng = np.random.default_rng(11 + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    dY = rng.standard_normal((M, N)).astype(np.float32)
    lp = LinearPath.from_f32_split(ctx, dev(W))
    assert lp.W.scale_log2 == 14 - int(np.floor(np.log2(np.abs(W).max())))
    Y = lp.forward(dev(X))
    assert rel_fro(host(Y), f64(X) @ f64(W).T) < 1e-5
    dX = lp.dx(dev(dY))
    assert rel_fro(host(dX), f64(dY) @ f64(W)) < 1e-5


@pytest.mark.parametrize("qtype", [12, 8, 13])
@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (300, 384, 2048), (64, 256, 512), (520, 640, 1280)])
def test_quant_weight_bf16_activations(ctx, oracle, qtype, M, N, K):
    """Quant W dequantized bit-exactly to fp16, bf16 X / dY: <= 2e-3 vs fp64."""
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(qtype + M)
    b = blocks_for(rng, qtype, N, K)
    Wf = oracle.dequant(b, qtype, N, K, 0)
    Xb = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16)
    dYb = torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)).to(torch.bfloat16)
    w = tk.make_weight(qtype, N, K, dev(b))
    Y = torch.empty(M, N, dtype=torch.float32, device="cuda")
    ctx.linear(w, Xb.cuda(), M, Y, x_dtype=tk.DT_BF16)
    Xf = Xb.float().numpy()
    err = rel_fro(host(Y), f64(Xf) @ f64(Wf).T)
    assert err < 2e-3
    dX = torch.empty(M, K, dtype=torch.float32, device="cuda")
    ctx.linear_dx(w, dYb.cuda(), M, dX, dy_dtype=tk.DT_BF16)
    errd = rel_fro(host(dX), f64(dYb.float().numpy()) @ f64(Wf))
    assert errd < 2e-3


def test_beta_accumulate_and_ld(ctx):
    """linear_dx_acc (beta = 1) and padded leading dimensions."""
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(5)
    M, N, K = 160, 320, 256
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    X = rng.standard_normal((M, K + 8)).astype(np.float32)
    w = tk.make_weight(tk.F16, N, K, dev(W))
    Y0 = rng.standard_normal((M, N + 4)).astype(np.float32)
    Y = dev(Y0)
    ctx.linear(w, dev(X), M, Y, ldx=K + 8, ldy=N + 4, beta=1.0, products=tk.X3_REF)
    want = Y0.astype(np.float64)
    want[:, :N] += f64(X[:, :K]) @ f64(W).T
    assert rel_fro(host(Y), want) < 1e-6
    dY = rng.standard_normal((M, N)).astype(np.float32)
    D0 = rng.standard_normal((M, K)).astype(np.float32)
    D = dev(D0)
    ctx.linear_dx_acc(w, dev(dY), M, D, products=tk.X3_REF)
    assert rel_fro(host(D), D0 + f64(dY) @ f64(W)) < 1e-6


def test_invalid_shapes_rejected(ctx):
    import torch
    import tier_b200 as tk
    W = torch.zeros(256, 100, dtype=torch.float16, device="cuda")
    w = tk.make_weight(tk.F16, 256, 100, W)       # cols % 8 != 0
    Y = torch.empty(4, 256, device="cuda")
    with pytest.raises(tk.TierkError):
        ctx.linear(w, torch.zeros(4, 100, device="cuda"), 4, Y)


@pytest.mark.parametrize("qtype", [12, 8])
def test_quant_weight_fp32_activations_x3(ctx, oracle, qtype):
    """fp32 X with a quantized W: the three activation parts share one
    dequantized W (the reference's training path: dequant to fp16, then
    fp3gemm), compared with fp64 of the fp16-rounded weight: <= 1e-5."""
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(qtype)
    M, N, K = 384, 512, 2048
    b = blocks_for(rng, qtype, N, K)
    W16 = oracle.dequant(b, qtype, N, K, 1).view(np.float16)
    X = rng.standard_normal((M, K)).astype(np.float32)
    dY = rng.standard_normal((M, N)).astype(np.float32)
    w = tk.make_weight(qtype, N, K, dev(b))
    Y = torch.empty(M, N, dtype=torch.float32, device="cuda")
    ctx.linear(w, dev(X), M, Y, products=tk.X3_REF)
    assert rel_fro(host(Y), f64(X) @ f64(W16).T) < 1e-5
    dX = torch.empty(M, K, dtype=torch.float32, device="cuda")
    ctx.linear_dx(w, dev(dY), M, dX, products=tk.X3_REF)
    assert rel_fro(host(dX), f64(dY) @ f64(W16)) < 1e-5


@pytest.mark.parametrize("qtype", [12, 13, 8])
@pytest.mark.parametrize("M,N,K,prods", [(256, 512, 1024, 4), (300, 384, 2048, 4), (384, 512, 2048, 1)])
def test_quant_fused_decode_matches(ctx, oracle, qtype, M, N, K, prods):
    """TK_QFUSED (decode inside the GEMM) agrees with fp64 of the fp16-rounded
    weight: 2e-3 for one bf16 product, 1e-5 for the fp32 three-part split."""
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(qtype * 7 + M)
    b = blocks_for(rng, qtype, N, K)
    W16 = oracle.dequant(b, qtype, N, K, 1).view(np.float16)
    w = tk.make_weight(qtype, N, K, dev(b))
    if prods == tk.X1:
        X = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16)
        dY = torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)).to(torch.bfloat16)
        xdt, tol = tk.DT_BF16, 2e-3
        Xf, dYf = X.float().numpy(), dY.float().numpy()
        X, dY = X.cuda(), dY.cuda()
    else:
        Xf = rng.standard_normal((M, K)).astype(np.float32)
        dYf = rng.standard_normal((M, N)).astype(np.float32)
        X, dY, xdt, tol = dev(Xf), dev(dYf), tk.DT_F32, 1e-5
    Y = torch.empty(M, N, dtype=torch.float32, device="cuda")
    ctx.linear(w, X, M, Y, x_dtype=xdt, products=prods | tk.QFUSED)
    assert rel_fro(host(Y), f64(Xf) @ f64(W16).T) < tol
    dX = torch.empty(M, K, dtype=torch.float32, device="cuda")
    ctx.linear_dx(w, dY, M, dX, dy_dtype=xdt, products=prods | tk.QFUSED)
    assert rel_fro(host(dX), f64(dYf) @ f64(W16)) < tol
    ctx.sync_status()


@pytest.mark.parametrize("M,N,K,prods", [(300, 1000, 4096, "X1"), (256, 520, 8192, "X3_REF"), (2048, 2048, 14336, "X1")])
def test_split_k_shapes(ctx, M, N, K, prods):
    """Few output tiles and long K: the GEMM splits K in two and adds the
    halves in fp32.  Results hold the path's tolerance, with beta = 1 and a
    padded output stride too, and are bit-identical across runs (every
    arrival order of the two halves computes the same fp32 sum)."""
    import torch
    import tier_b200 as tk
    p = getattr(tk, prods)
    rng = np.random.default_rng(N + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    if p == tk.X1:
        X = rng.standard_normal((M, K)).astype(np.float16)
        dY = rng.standard_normal((M, N)).astype(np.float16)
        # one fp16 product: fp32 tensor-core accumulation over K = 14336 measures ~1.6e-5
        xdt, tol = tk.DT_F16, 5e-5
    else:
        X = rng.standard_normal((M, K)).astype(np.float32)
        dY = rng.standard_normal((M, N)).astype(np.float32)
        xdt, tol = tk.DT_F32, 1e-5
    w = tk.make_weight(tk.F16, N, K, dev(W))
    Xd, dYd = dev(X), dev(dY)
    want = f64(X) @ f64(W).T
    Y0 = rng.standard_normal((M, N + 4)).astype(np.float32)
    outs = []
    for _ in range(2):
        Y = dev(Y0)
        ctx.linear(w, Xd, M, Y, x_dtype=xdt, ldy=N + 4, beta=1.0, products=p)
        outs.append(host(Y))
    assert np.array_equal(outs[0], outs[1])
    full = Y0.astype(np.float64)
    full[:, :N] += want
    assert rel_fro(outs[0], full) < tol
    dX = torch.empty(M, K, dtype=torch.float32, device="cuda")
    ctx.linear_dx(w, dYd, M, dX, dy_dtype=xdt, products=p)
    d1 = host(dX)
    ctx.linear_dx(w, dYd, M, dX, dy_dtype=xdt, products=p)
    assert np.array_equal(d1, host(dX))
    assert rel_fro(d1, f64(dY) @ f64(W)) < tol
    ctx.sync_status()


@pytest.mark.gpu
def test_wreuse_same_bits_and_one_dequant(ctx):
    """TK_WREUSE: the dX call after the forward on the same frozen quantized W
    uses the forward's fp16 expansion (one dequant fewer) and gives the same
    bits as a dX call that dequantizes; a different weight or another
    workspace user in between forces a fresh dequant."""
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(21)
    N, K, M = 768, 1024, 384
    b1, b2 = blocks_for(rng, tk.Q4_K, N, K), blocks_for(rng, tk.Q4_K, N, K)
    w1 = tk.make_weight(tk.Q4_K, N, K, dev(b1))
    w2 = tk.make_weight(tk.Q4_K, N, K, dev(b2))
    X = dev(rng.standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16)
    dY = dev(rng.standard_normal((M, N)).astype(np.float32)).to(torch.bfloat16)
    Y = torch.empty(M, N, device="cuda")
    want = torch.empty(M, K, device="cuda")
    ctx.linear_dx(w1, dY, M, want, dy_dtype=tk.DT_BF16)
    ref = host(want)

    got = torch.empty(M, K, device="cuda")
    ctx.linear(w1, X, M, Y, x_dtype=tk.DT_BF16)
    n0 = ctx.launches()
    ctx.linear_dx(w1, dY, M, got, dy_dtype=tk.DT_BF16, products=tk.WREUSE)
    reused = ctx.launches() - n0
    ctx.linear_dx(w1, dY, M, want, dy_dtype=tk.DT_BF16)
    fresh = ctx.launches() - n0 - reused
    assert np.array_equal(host(got), ref)
    assert reused == fresh - 1                       # the dequant was skipped

    # another weight in between: the flag must not pick up w2's expansion
    ctx.linear(w1, X, M, Y, x_dtype=tk.DT_BF16)
    ctx.linear(w2, X, M, Y, x_dtype=tk.DT_BF16)
    got.fill_(float("nan"))
    ctx.linear_dx(w1, dY, M, got, dy_dtype=tk.DT_BF16, products=tk.WREUSE)
    assert np.array_equal(host(got), ref)

    # the workspace grows (reallocated) in between
    ctx.linear(w1, X, M, Y, x_dtype=tk.DT_BF16)
    ctx.reserve(ctx.lib.tk_workspace_bytes(ctx.h) + (1 << 20))
    got.fill_(float("nan"))
    ctx.linear_dx(w1, dY, M, got, dy_dtype=tk.DT_BF16, products=tk.WREUSE)
    assert np.array_equal(host(got), ref)
    ctx.sync_status()
