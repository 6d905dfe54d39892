"""GPU parity of the chunked-vocabulary LM head + cross-entropy (both passes)
against the fp64 two-pass restatement of tier/tier.cpp:3184-3266.
Tolerance: loss and dX relative <= 1e-5 (x3 product set)."""
import numpy as np
import pytest

from gen import rel_fro

pytestmark = pytest.mark.gpu


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_head(ctx, W, X, labels, mask, cap, chunk, products):
    import torch
    from tier_b200.host import LMHead
    head = LMHead(ctx, dev(W), 0, chunk=chunk, products=products)
    loss, n_loss, hits, amax, dX = head.step(dev(X), dev(labels), dev(mask), softcap=cap)
    torch.cuda.synchronize()
    ctx.sync_status()
    return float(loss.item()), n_loss, int(hits.item()), amax.cpu().numpy(), dX.cpu().numpy()


@pytest.mark.parametrize("cap", [0.0, 30.0])
@pytest.mark.parametrize("V,H,T,chunk", [(2048, 256, 64, 512), (4096, 384, 130, 1024), (1024, 128, 300, 256)])
def test_lmhead_matches_f64(ctx, oracle, cap, V, H, T, chunk):
    import tier_b200 as tk
    rng = np.random.default_rng(V + T)
    W = (rng.standard_normal((V, H)) * 0.02).astype(np.float16)
    X = rng.standard_normal((T, H)).astype(np.float32)
    labels = rng.integers(0, V, T).astype(np.int32)
    mask = np.ones(T, np.uint8)
    mask[rng.integers(0, T - 1, 5)] = 0
    want_loss, want_n, want_amax, want_dX, *_ = oracle.lmhead_f64(W.view(np.uint16), X, labels, mask, cap, chunk)
    loss, n_loss, hits, amax, dX = run_head(ctx, W, X, labels, mask, cap, chunk, tk.X3_REF)
    assert n_loss == want_n
    assert abs(loss - want_loss) / abs(want_loss) < 1e-5
    live = mask[: T - 1] != 0
    assert np.mean(amax[live] == want_amax[live]) > 0.99   # exact ties aside
    assert rel_fro(dX, want_dX) < 1e-5
    assert hits == int(np.sum(amax[live] == labels[1:][live]))


def test_lmhead_two_part_split_is_close(ctx, oracle):
    import tier_b200 as tk
    rng = np.random.default_rng(1)
    V, H, T, chunk = 2048, 256, 64, 512
    W = (rng.standard_normal((V, H)) * 0.02).astype(np.float16)
    X = rng.standard_normal((T, H)).astype(np.float32)
    labels = rng.integers(0, V, T).astype(np.int32)
    mask = np.ones(T, np.uint8)
    want_loss, _, _, want_dX, *_ = oracle.lmhead_f64(W.view(np.uint16), X, labels, mask, 0.0, chunk)
    loss, _, _, _, dX = run_head(ctx, W, X, labels, mask, 0.0, chunk, tk.X2)
    assert abs(loss - want_loss) / abs(want_loss) < 1e-5
    assert rel_fro(dX, want_dX) < 1e-5


def test_lmhead_vocab_shards_merge(ctx, oracle):
    """Two vocab shards processed separately and merged on the host with the
    same rescale the multi-GPU path uses (all-reduce emulated by sums)."""
    import torch
    import tier_b200 as tk
    rng = np.random.default_rng(2)
    V, H, T, chunk = 2048, 256, 40, 512
    W = (rng.standard_normal((V, H)) * 0.02).astype(np.float16)
    X = rng.standard_normal((T, H)).astype(np.float32)
    labels = rng.integers(0, V, T).astype(np.int32)
    mask = np.ones(T, np.uint8)
    want_loss, _, want_amax, want_dX, *_ = oracle.lmhead_f64(W.view(np.uint16), X, labels, mask, 0.0, chunk)
    Xd, Ld, Md = dev(X), dev(labels), dev(mask)
    st = []
    for s in range(2):
        Ws = dev(W[s * 1024:(s + 1) * 1024])
        rmax = torch.full((T - 1,), -1e30, dtype=torch.float64, device="cuda")
        rsum = torch.zeros(T - 1, dtype=torch.float64, device="cuda")
        amax = torch.full((T - 1,), -1, dtype=torch.int32, device="cuda")
        tgt = torch.zeros(T - 1, dtype=torch.float32, device="cuda")
        ctx.lmhead_stats(Ws, s * 1024, 1024, H, Xd, T, Ld, Md, 0.0, chunk, rmax, rsum, amax, tgt)
        st.append((Ws, rmax, rsum, amax, tgt))
    gmax = torch.maximum(st[0][1], st[1][1])
    best = (st[1][1] > st[0][1]).int()
    amax = torch.where(best.bool(), st[1][3], st[0][3])
    for s in range(2):
        ctx.lmhead_rescale(T - 1, st[s][1], st[s][2], gmax)
    rsum = st[0][2] + st[1][2]
    tgt = st[0][4] + st[1][4]
    loss = torch.zeros(1, dtype=torch.float64, device="cuda")
    hits = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctx.lmhead_loss(T, Ld, Md, gmax, rsum, amax, tgt, loss, hits)
    dX = torch.zeros(T, H, dtype=torch.float32, device="cuda")
    for s in range(2):
        ctx.lmhead_grad(st[s][0], s * 1024, 1024, H, Xd, T, Ld, Md, T - 1, 0.0, chunk, gmax, rsum, dX)
    torch.cuda.synchronize()
    assert abs(loss.item() - want_loss) / abs(want_loss) < 1e-5
    assert rel_fro(dX.cpu().numpy(), want_dX) < 1e-5
    assert np.mean(amax.cpu().numpy() == want_amax) > 0.99


def run_fused(ctx, W, X, labels, mask, cap, chunk, products):
    import torch
    from tier_b200.host import LMHead
    head = LMHead(ctx, dev(W), 0, chunk=chunk, products=products)
    loss, n_loss, hits, amax, dX = head.step_fused(dev(X), dev(labels), dev(mask), softcap=cap)
    torch.cuda.synchronize()
    ctx.sync_status()
    return float(loss.item()), n_loss, int(hits.item()), amax.cpu().numpy(), dX.cpu().numpy()


@pytest.mark.parametrize("cap", [0.0, 30.0])
@pytest.mark.parametrize("V,H,T,chunk", [(2048, 256, 64, 512), (4096, 384, 130, 1024), (1024, 128, 300, 256)])
def test_lmhead_single_pass_matches(ctx, oracle, cap, V, H, T, chunk):
    """Single pass (tk_lmhead_fused + tk_lmhead_finish): the pass-1 state is
    the two-pass one bit for bit (same logits GEMM and merge), the loss and
    hits equal, dX within 1e-5 of fp64."""
    import tier_b200 as tk
    rng = np.random.default_rng(V + T)
    W = (rng.standard_normal((V, H)) * 0.02).astype(np.float16)
    X = rng.standard_normal((T, H)).astype(np.float32)
    labels = rng.integers(0, V, T).astype(np.int32)
    mask = np.ones(T, np.uint8)
    mask[rng.integers(0, T - 1, 5)] = 0
    want_loss, want_n, want_amax, want_dX, *_ = oracle.lmhead_f64(W.view(np.uint16), X, labels, mask, cap, chunk)
    loss2, n2, hits2, amax2, dX2 = run_head(ctx, W, X, labels, mask, cap, chunk, tk.X3_REF)
    loss, n_loss, hits, amax, dX = run_fused(ctx, W, X, labels, mask, cap, chunk, tk.X3_REF)
    assert n_loss == want_n == n2
    assert loss == loss2 and hits == hits2 and np.array_equal(amax, amax2)
    assert abs(loss - want_loss) / abs(want_loss) < 1e-5
    assert rel_fro(dX, want_dX) < 1e-5
    assert rel_fro(dX, dX2) < 1e-5
    # rows without loss (masked, and the last row) are exactly zero
    dead = np.ones(T, bool)
    dead[: T - 1] = mask[: T - 1] == 0
    assert not np.any(dX[dead])


def test_lmhead_single_pass_vocab_shards(ctx, oracle):
    """Two vocab shards in single-pass form, merged on the host the way the
    multi-GPU path does (rescale of rsum and of the dX accumulator to the
    global max, finish per shard with the global sum, then a sum)."""
    import torch
    rng = np.random.default_rng(3)
    V, H, T, chunk = 2048, 256, 40, 512
    W = (rng.standard_normal((V, H)) * 0.02).astype(np.float16)
    X = rng.standard_normal((T, H)).astype(np.float32)
    labels = rng.integers(0, V, T).astype(np.int32)
    mask = np.ones(T, np.uint8)
    want_loss, _, _, want_dX, *_ = oracle.lmhead_f64(W.view(np.uint16), X, labels, mask, 30.0, chunk)
    Xd, Ld, Md = dev(X), dev(labels), dev(mask)
    st = []
    for s in range(2):
        Ws = dev(W[s * 1024:(s + 1) * 1024])
        rmax = torch.full((T - 1,), -1e30, dtype=torch.float64, device="cuda")
        rsum = torch.zeros(T - 1, dtype=torch.float64, device="cuda")
        amax = torch.full((T - 1,), -1, dtype=torch.int32, device="cuda")
        tgt = torch.zeros(T - 1, dtype=torch.float32, device="cuda")
        dX = torch.zeros(T, H, dtype=torch.float32, device="cuda")
        ctx.lmhead_fused(Ws, s * 1024, 1024, H, Xd, T, Ld, Md, 30.0, chunk, rmax, rsum, amax, tgt, dX)
        st.append((Ws, rmax, rsum, amax, tgt, dX))
    gmax = torch.maximum(st[0][1], st[1][1])
    best = (st[1][1] > st[0][1]).int()
    amax = torch.where(best.bool(), st[1][3], st[0][3])
    for s in range(2):
        ctx.lmhead_rescale(T - 1, st[s][1], st[s][2], gmax, st[s][5], H)
    rsum = st[0][2] + st[1][2]
    tgt = st[0][4] + st[1][4]
    for s in range(2):
        ctx.lmhead_finish(st[s][0], s * 1024, 1024, H, T, Ld, Md, T - 1, 30.0, rsum, tgt, st[s][5])
    dX = (st[0][5] + st[1][5]).cpu().numpy()
    loss = torch.zeros(1, dtype=torch.float64, device="cuda")
    hits = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctx.lmhead_loss(T, Ld, Md, gmax, rsum, amax, tgt, loss, hits)
    torch.cuda.synchronize()
    ctx.sync_status()
    assert abs(loss.item() - want_loss) / abs(want_loss) < 1e-5
    assert rel_fro(dX, want_dX) < 1e-5
