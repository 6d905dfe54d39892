"""tk_linear_fwd_noalloc -- the forward linear for callers that cannot call
cudaMalloc (an engine that budgets all device memory through its own arena,
or code that must not allocate once running).  Its scratch is a static device
array inside libtierk.so instead of the context workspace.

Checked through the C ABI against tk_linear_fwd on two rounds of calls in a
row (the second reuses the array the first left behind): bit for bit, since
the shapes keep tk_linear_fwd on one K split, and within the x3 tests' 1e-5
of fp64; the calls are shown not to grow the context workspace.
This file is named to be collected last."""
import ctypes

import numpy as np
import pytest

from gen import rel_fro

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _noalloc(lib, ctx, w, X, x_dtype, M, Y, products, beta=0.0):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    return lib.tk_linear_fwd_noalloc(ctx.h, ctypes.byref(w), X.data_ptr(), x_dtype, M, X.stride(0), Y.data_ptr(),
                                     Y.stride(0), beta, products, stream)


def _run_cases(lib, ctx, device):
    """Both entry points on the same inputs; K < 2048 keeps tk_linear_fwd on
    one K split, so the two must agree bit for bit (same kernels, same
    accumulation segments)."""
    import torch
    import tier_b200 as tk
    from tier_b200.host import LinearPath
    rng = np.random.default_rng(21 + device)
    cases = [
        # (M, N, K, x dtype, weight kind, product set, beta)
        (192, 640, 1024, tk.DT_F32, tk.F16, tk.X3_REF, 0.0),
        (130, 384, 520, tk.DT_BF16, tk.F16, tk.X1, 0.0),
        (256, 512, 1024, tk.DT_F32, tk.F16X2, tk.X3_AUTO, 0.0),          # hi/lo weight planes: X3_HHL
        (200, 384, 776, tk.DT_F32, tk.F16, tk.X3_REF | tk.WREUSE, 1.0),  # accumulate; flag ignored for fp16 W
    ]
    for M, N, K, xdt, wkind, prod, beta in cases:
        W32 = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        if wkind == tk.F16X2:
            lp = LinearPath.from_f32_split(ctx, torch.from_numpy(W32).to(device))
            w, Wref = lp.W, W32.astype(np.float64)
        else:
            W = W32.astype(np.float16)
            Wd = torch.from_numpy(W).to(device)
            w, Wref = tk.make_weight(wkind, N, K, Wd), W.astype(np.float64)
        Xf = rng.standard_normal((M, K)).astype(np.float32)
        X = torch.from_numpy(Xf).to(device)
        if xdt == tk.DT_BF16:
            X = X.to(torch.bfloat16)
        Y0 = torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)).to(device)
        Y_new = Y0.clone() if beta else torch.full((M, N), float("nan"), dtype=torch.float32, device=device)
        ws_before = lib.tk_workspace_bytes(ctx.h)
        with torch.cuda.device(device):
            assert _noalloc(lib, ctx, w, X, xdt, M, Y_new, prod, beta) == tk.TK_OK, lib.tk_last_error_string()
        assert lib.tk_workspace_bytes(ctx.h) == ws_before, "the no-alloc path must not grow the workspace"
        Y_old = Y0.clone() if beta else torch.empty(M, N, dtype=torch.float32, device=device)
        with torch.cuda.device(device):
            ctx.linear(w, X, M, Y_old, x_dtype=xdt, products=prod, beta=beta)
        ctx.sync_status()
        a, b = Y_new.cpu().numpy(), Y_old.cpu().numpy()
        assert np.isfinite(a).all()
        assert np.array_equal(a, b), rel_fro(a, b)
        ref = X.double().cpu().numpy() @ Wref.T + (Y0.double().cpu().numpy() if beta else 0.0)
        tol = 2e-3 if prod == tk.X1 else 1e-5
        assert rel_fro(a, ref) < tol


def test_noalloc_matches_linear_fwd_two_calls():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import tier_b200 as tk
    lib = tk.load()
    ctx = tk.Context(0)
    try:
        assert lib.tk_workspace_bytes(ctx.h) == 0
        # two rounds of calls in a row: the second reads the array the first left behind
        for _ in range(2):
            _run_cases(lib, ctx, 0)
    finally:
        ctx.close()


def test_noalloc_second_device():
    """The scratch address is looked up per device: a context on device 1."""
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import tier_b200 as tk
    lib = tk.load()
    ctx = tk.Context(1)
    try:
        for _ in range(2):
            _run_cases(lib, ctx, 1)
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
