"""Full-size LM head (V = 262144, H = 3840, T = 8192, chunk 16384), two-pass
and single-pass: the GPU path runs every row; sampled rows are checked in
fp64 on the host (vocab processed in chunks): per-row lse, target logit,
argmax, loss contribution and the dX row, at the 1e-5 tolerance."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("single_pass", [False, True])
def test_lmhead_full_size_sampled_rows(ctx, single_pass):
    import torch
    import tier_b200 as tk
    from tier_b200.host import LMHead
    V, H, T, chunk = 262144, 3840, 8192, 16384
    g = torch.Generator(device="cuda").manual_seed(3)
    W = (torch.randn(V, H, device="cuda", generator=g) * 0.02).half()
    X = torch.randn(T, H, device="cuda", generator=g)
    labels = torch.randint(0, V, (T,), device="cuda", generator=g, dtype=torch.int32)
    mask = torch.ones(T, dtype=torch.uint8, device="cuda")
    head = LMHead(ctx, W, 0, chunk=chunk, products=tk.X3_REF)
    if single_pass:
        # the single pass leaves the same running state; rebuild it for the checks
        loss, _, hits, amax, dX = head.step_fused(X, labels, mask)
        rmax, rsum, amax2, tgt = head.stats(X, labels, mask)
        assert torch.equal(amax, amax2)
    else:
        rmax, rsum, amax, tgt = head.stats(X, labels, mask)
        loss, hits = head.loss(T, labels, mask, rmax, rsum, amax, tgt)
        dX = head.grad(X, labels, mask, T - 1, rmax, rsum)
    torch.cuda.synchronize()
    ctx.sync_status()

    rows = [0, 1, 4097, T - 2]
    lse_gpu = (rmax + torch.log(rsum)).cpu().numpy()
    tgt_gpu = tgt.cpu().numpy()
    amax_gpu = amax.cpu().numpy()
    dX_gpu = dX.cpu().numpy()
    Xs = X[rows].double().cpu().numpy()                       # [R, H]
    lab = labels.cpu().numpy()
    R = len(rows)
    m = np.full(R, -np.inf)
    s = np.zeros(R)
    am = np.zeros(R, np.int64)
    tg = np.zeros(R)
    # pass 1 in fp64 over vocab chunks (logits rounded to fp32 as the reference's GEMM output is)
    for v0 in range(0, V, chunk):
        Wc = W[v0:v0 + chunk].double().cpu().numpy()
        L = (Xs @ Wc.T).astype(np.float32).astype(np.float64)  # [R, chunk]
        cm = L.max(1)
        ci = L.argmax(1)
        nm = np.maximum(m, cm)
        am = np.where(cm > m, v0 + ci, am)
        s = s * np.exp(m - nm) + np.exp(L - cm[:, None]).sum(1) * np.exp(cm - nm)
        m = nm
        for i, t in enumerate(rows):
            if v0 <= lab[t + 1] < v0 + chunk:
                tg[i] = L[i, lab[t + 1] - v0]
    lse = m + np.log(s)
    # pass 2: dX rows
    n_loss = T - 1
    d = np.zeros((R, H))
    for v0 in range(0, V, chunk):
        Wc = W[v0:v0 + chunk].double().cpu().numpy()
        L = (Xs @ Wc.T).astype(np.float32).astype(np.float64)
        P = np.exp(L - lse[:, None])
        for i, t in enumerate(rows):
            if v0 <= lab[t + 1] < v0 + chunk:
                P[i, lab[t + 1] - v0] -= 1.0
        d += (P / n_loss) @ Wc
    for i, t in enumerate(rows):
        assert abs(lse_gpu[t] - lse[i]) / abs(lse[i]) < 1e-6, (t, lse_gpu[t], lse[i])
        assert abs(tgt_gpu[t] - tg[i]) <= 1e-5 * max(1.0, abs(tg[i])), (t, tgt_gpu[t], tg[i])
        assert amax_gpu[t] == am[i]
        err = np.linalg.norm(dX_gpu[t] - d[i]) / np.linalg.norm(d[i])
        assert err < 1e-5, (t, err)
    # the loss is the sum of the per-row terms the running state holds
    per_row = (lse_gpu - tgt_gpu).astype(np.float64)
    assert abs(loss.item() - per_row.sum()) / abs(per_row.sum()) < 1e-9
    assert hits.item() == int((amax_gpu == lab[1:]).sum())
