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
@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (300, 384, 2048)])
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
