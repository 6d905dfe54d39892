"""tk_linear_fwd_dx: the forward and the input gradient of one weight in one
persistent GEMM launch (tiles of the two GEMMs interleaved).

The pair never splits K, so it must give what the two separate calls give
bit for bit wherever those run one K split (a reduction length below 32
k-blocks of 64: K < 2048 for Y, N < 2048 for dX), and be within the product
set's tolerance against fp64 everywhere:
  * fewer launches: one GEMM launch for both, W expanded once.
Shapes cover ragged M (partial CTA-pair tiles), different token counts on the
two sides, every product set, and the small-M fallback (two launches).
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


CASES = [
    # (weight kind, activation dtype, product set, Mx, Md, N, K)
    ("q4_k", "bf16", "X3_AUTO", 512, 512, 1792, 4096),     # one rank's C2 shard at 8 GPUs, fewer tokens
    ("q4_k", "bf16", "X3_AUTO", 300, 700, 1024, 2048),     # ragged, different token counts
    ("q8_0", "f32", "X3_AUTO", 256, 384, 768, 1024),       # x3 REF products, accumulation segments
    ("f16", "f32", "X3_REF", 384, 256, 1000, 520),         # ragged N and K
    ("f16x2", "f32", "X3_HHL", 384, 384, 768, 1024),       # fp32 W as hi/lo planes
    ("f16", "f16", "X1", 1024, 1024, 512, 256),
    ("q4_k", "bf16", "X3_AUTO", 100, 640, 512, 1024),      # Mx <= 128: two launches
]


def _weight(ctx, rng, kind, N, K):
    """(tk_weight, the fp16-exact operand the GEMM multiplies as a torch tensor
    for the fp64 check: the fp16 expansion of a quantized W, fp16 W, or the
    fp32 W that hi/lo planes represent)."""
    import torch
    import tier_b200 as tk
    from tier_b200.host import LinearPath
    if kind in ("q4_k", "q8_0"):
        qt = tk.Q4_K if kind == "q4_k" else tk.Q8_0
        b = dev(blocks_for(rng, qt, N, K))
        W16 = torch.empty(N, K, dtype=torch.float16, device="cuda")
        ctx.dequant(qt, b, N, K, W16, out_dtype=tk.DT_F16)
        return tk.make_weight(qt, N, K, b), W16
    W32 = torch.from_numpy((rng.standard_normal((N, K)) * 0.02).astype(np.float32)).cuda()
    if kind == "f16":
        W16 = W32.half()
        return tk.make_weight(tk.F16, N, K, W16), W16
    return LinearPath.from_f32_split(ctx, W32).W, W32


def _act(rng, M, C, dt):
    import torch
    a = torch.from_numpy(rng.standard_normal((M, C)).astype(np.float32)).cuda()
    return {"bf16": a.to(torch.bfloat16), "f16": a.half(), "f32": a}[dt]


@pytest.mark.parametrize("kind,adt,prods,Mx,Md,N,K", CASES)
def test_fwd_dx_pair_matches_separate_calls(ctx, kind, adt, prods, Mx, Md, N, K):
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(Mx * 7 + Md + N)
    w, Wop = _weight(ctx, rng, kind, N, K)
    dt = {"bf16": tk.DT_BF16, "f16": tk.DT_F16, "f32": tk.DT_F32}[adt]
    p = getattr(tk, prods)
    X, dY = _act(rng, Mx, K, adt), _act(rng, Md, N, adt)
    Y = torch.full((Mx, N), float("nan"), device="cuda")
    dX = torch.full((Md, K), float("nan"), device="cuda")
    n0 = ctx.launches()
    ctx.linear_fwd_dx(w, X, Mx, Y, dY, Md, dX, x_dtype=dt, products=p)
    pair_launches = ctx.launches() - n0
    Y2 = torch.empty(Mx, N, device="cuda")
    dX2 = torch.empty(Md, K, device="cuda")
    n0 = ctx.launches()
    ctx.linear(w, X, Mx, Y2, x_dtype=dt, products=p)
    ctx.linear_dx(w, dY, Md, dX2, dy_dtype=dt, products=p | tk.WREUSE)
    sep_launches = ctx.launches() - n0
    torch.cuda.synchronize()
    ctx.sync_status()
    if K < 2048:   # tk_linear_fwd runs one K split here
        assert torch.equal(Y, Y2)
    if N < 2048:   # tk_linear_dx runs one K split here
        assert torch.equal(dX, dX2)
    # against fp64 of the operand the GEMM multiplies: one fp16 product of
    # bf16 activations holds 2e-3 (the quant GEMM's stated bound), the x3
    # product sets and fp16 x fp16 hold 1e-5
    Wf = Wop.double()
    tol = 2e-3 if adt == "bf16" else 1e-5
    assert rel_fro(host(Y), host(X.double() @ Wf.T)) < tol
    assert rel_fro(host(dX), host(dY.double() @ Wf)) < tol
    if Mx > 128 and Md > 128:
        # one GEMM launch instead of two (the x3 paths also skip nothing else)
        assert pair_launches == sep_launches - 1, (pair_launches, sep_launches)
    else:
        assert pair_launches == sep_launches
