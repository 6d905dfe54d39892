"""tk_linear_fwd_noalloc -- the forward linear for callers that cannot call
cudaMalloc (an engine that budgets all device memory through its own arena,
or code that must not allocate once running).  Its scratch is a static device
array inside libtierk.so instead of the context workspace.

Checked through the C ABI against tk_linear_fwd on two calls in a row (the
second call reuses the array the first call left behind), within the 1e-5
tolerance the x3 tests use, and shown not to grow the context workspace.
This file is named to be collected last."""
import ctypes

import numpy as np
import pytest

from gen import rel_fro

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _noalloc(lib, ctx, w, X, x_dtype, M, Y, products):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    return lib.tk_linear_fwd_noalloc(ctx.h, ctypes.byref(w), X.data_ptr(), x_dtype, M, X.stride(0), Y.data_ptr(),
                                     Y.stride(0), 0.0, products, stream)


def test_noalloc_matches_linear_fwd_two_calls():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import tier_b200 as tk
    lib = tk.load()
    ctx = tk.Context(0)
    try:
        assert lib.tk_workspace_bytes(ctx.h) == 0
        rng = np.random.default_rng(21)
        cases = [
            # (M, N, K, x dtype, weight kind, product set)
            (192, 640, 1024, tk.DT_F32, tk.F16, tk.X3_REF),
            (130, 384, 520, tk.DT_BF16, tk.F16, tk.X1),
        ]
        for M, N, K, xdt, wkind, prod in cases:
            W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
            Wd = _dev(W)
            w = tk.make_weight(wkind, N, K, Wd)
            Xf = rng.standard_normal((M, K)).astype(np.float32)
            X = _dev(Xf) if xdt == tk.DT_F32 else _dev(Xf).to(torch.bfloat16)
            Y_new = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
            ws_before = lib.tk_workspace_bytes(ctx.h)
            assert _noalloc(lib, ctx, w, X, xdt, M, Y_new, prod) == tk.TK_OK, lib.tk_last_error_string()
            assert lib.tk_workspace_bytes(ctx.h) == ws_before, "the no-alloc path must not grow the workspace"
            Y_old = torch.empty(M, N, dtype=torch.float32, device="cuda")
            ctx.linear(w, X, M, Y_old, x_dtype=xdt, products=prod)
            ctx.sync_status()
            a, b = Y_new.cpu().numpy(), Y_old.cpu().numpy()
            assert np.isfinite(a).all()
            assert rel_fro(a, b) < 1e-5
            ref = X.double().cpu().numpy() @ W.astype(np.float64).T
            tol = 1e-5 if prod == tk.X3_REF else 2e-3
            assert rel_fro(a, ref) < tol
    finally:
        ctx.close()


def test_noalloc_rejects_oversize_and_quant():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import tier_b200 as tk
    lib = tk.load()
    ctx = tk.Context(0)
    try:
        N, K, M = 256, 8192, 1024            # 3 parts * 1024 * 8192 * 2 B = 48 MiB > 24 MiB
        Wd = torch.zeros(N, K, dtype=torch.float16, device="cuda")
        w = tk.make_weight(tk.F16, N, K, Wd)
        X = torch.zeros(M, K, dtype=torch.float32, device="cuda")
        Y = torch.empty(M, N, dtype=torch.float32, device="cuda")
        st = _noalloc(lib, ctx, w, X, tk.DT_F32, M, Y, tk.X3_REF)
        assert st == tk.TK_ERR_INVALID
        assert b"static limit" in lib.tk_last_error_string()
        q = torch.zeros(N, tk.row_bytes(tk.Q4_K, K), dtype=torch.uint8, device="cuda")
        wq = tk.make_weight(tk.Q4_K, N, K, q)
        st = _noalloc(lib, ctx, wq, X[:8], tk.DT_F32, 8, Y[:8], tk.X3_REF)
        assert st == tk.TK_ERR_UNSUPPORTED
    finally:
        ctx.close()
