"""Host-side sharding logic on CPU with gloo, world sizes 2 and 3: the row split
used by the linear path, the vocab-shard merge of the running
cross-entropy state (max, rescaled sum, target, argmax with the reference's
lowest-index tie rule), and the single-pass head's dX accumulator merge
(rescale to the global max, finish against the global sum, all-reduce)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cpu_rescale(rl, sl, rg, dX=None):
    f = torch.exp(rl - rg)
    sl.mul_(f)
    if dX is not None:
        dX[: f.shape[0]].mul_(f.float()[:, None])
    rl.copy_(rg)


def _stats(lg, v0):
    """Running state of one shard's logits [T, V] (rows with mask 1)."""
    m, i = lg.max(dim=1)
    s = torch.exp(lg.double() - m.double()[:, None]).sum(1)
    return m.double(), s, (i + v0).int()


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tier_b200.host import merge_vocab_shards, shard_rows
        g = torch.Generator().manual_seed(0)
        T, V = 33, 1000
        lg = torch.randn(T, V, generator=g, dtype=torch.float64).float()
        lg[5, 100] = lg[5, 900] = lg[5].max() + 1.0          # exact tie across shards
        labels = torch.randint(0, V, (T,), generator=g)
        a, b = shard_rows(V, world, rank, align=8)
        rmax, rsum, amax = _stats(lg[:, a:b], a)
        tgt = torch.tensor([float(lg[t, labels[t]]) if a <= labels[t] < b else 0.0 for t in range(T)])
        amax = merge_vocab_shards(rmax, rsum, amax, tgt, dist.group.WORLD, _cpu_rescale)
        fm, fs, fa = _stats(lg, 0)
        ok = (torch.allclose(rmax, fm) and torch.allclose(rsum, fs, rtol=1e-12)
              and torch.equal(amax, fa) and int(amax[5]) == 100
              and torch.allclose(tgt, lg[torch.arange(T), labels]))
        # row shards tile the range, boundaries aligned
        parts = [shard_rows(14336, 8, r, align=256) for r in range(8)]
        ok = ok and parts[0][0] == 0 and parts[-1][1] == 14336 and all(
            parts[i][1] == parts[i + 1][0] and parts[i][1] % 256 == 0 for i in range(7))
        # single-pass head: per-shard accumulator relative to the shard max,
        # merged, finished (the label's shard subtracts its W row), summed
        H = 7
        W = torch.randn(V, H, generator=g, dtype=torch.float64)
        rmax, rsum, amax = _stats(lg[:, a:b], a)
        tgt = torch.tensor([float(lg[t, labels[t]]) if a <= labels[t] < b else 0.0 for t in range(T)])
        acc = (torch.exp(lg[:, a:b].double() - rmax[:, None]) @ W[a:b]).float()
        amax = merge_vocab_shards(rmax, rsum, amax, tgt, dist.group.WORLD, _cpu_rescale, dX=acc)
        n = T
        d = acc.double() / (n * rsum[:, None])
        for t in range(T):
            if a <= labels[t] < b:
                d[t] -= W[labels[t]] / n
        dist.all_reduce(d)
        P = torch.softmax(lg.double(), dim=1)
        P[torch.arange(T), labels] -= 1.0
        want = P @ W / n
        ok = ok and torch.allclose(d, want, rtol=1e-5, atol=1e-7)
        q.put((rank, bool(ok)))
    except Exception as e:   # report instead of leaving the other rank waiting
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_vocab_merge_and_row_split_gloo(world):
    """world 3 splits the 1000-entry vocabulary unevenly (8-aligned shards)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {r: True for r in range(world)}


class _HostGemv:
    """Stands in for the device context on CPU: gemv and linear on an fp32
    weight (linear finds the weight tensor by its data pointer)."""

    def __init__(self):
        self.weights = {}

    def gemv(self, qtype, W, N, K, x, y, M=1, ldx=None, ldy=None, row_bytes_=None, stream=None):
        y[:M, :N] = x[:M, :K] @ W.view(N, K).T
        return y

    def linear(self, w, X, M, Y, x_dtype=0, ldx=None, ldy=None, beta=0.0, products=0, stream=None):
        W = self.weights[w.data].view(w.rows, w.cols)
        Y[:M, : w.rows] = (beta * Y[:M, : w.rows] if beta else 0) + X[:M] @ W.T
        return Y


def _decode_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tier_b200 import F32
        from tier_b200.host import LinearPath, shard_rows
        g = torch.Generator().manual_seed(3)
        ok = True
        for N, M in ((64, 3), (65, 16), (14336, 2)):       # equal and unequal row shards
            K = 40
            W = torch.randn(N, K, generator=g)
            x = torch.randn(M, K, generator=g)
            a, b = shard_rows(N, world, rank, align=256 if N > 1000 else 1)
            host = _HostGemv()
            Ws = W[a:b].contiguous()
            host.weights[Ws.data_ptr()] = Ws
            lp = LinearPath(host, F32, b - a, K, Ws, group=dist.group.WORLD, n_total=N, row0=a)
            want = x @ W.T
            y = lp.decode(x)
            ok = ok and y.shape == (M, N) and torch.allclose(y, want, rtol=1e-5, atol=1e-5)
            out = torch.empty(M, N)
            ok = ok and lp.decode(x, y=out) is out and torch.allclose(out, want, rtol=1e-5, atol=1e-5)
            # forward (`linear`): the same gather of unequal column shards
            Y = lp.forward(x)
            ok = ok and Y.shape == (M, N) and torch.allclose(Y, want, rtol=1e-5, atol=1e-5)
            Y2 = torch.ones(M, N)
            ok = ok and lp.forward(x, Y=Y2, beta=1.0) is Y2 and torch.allclose(Y2, want + 1, rtol=1e-5, atol=1e-5)
        q.put((rank, bool(ok)))
    except Exception as e:   # report instead of leaving the other rank waiting
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_row_sharded_gather_gloo(world):
    """Decode and forward on row shards: each rank's columns land in the
    gathered [M, N_total] in rank order, for equal and unequal shards
    (14336 rows over 3 ranks in 256-row units: 18 / 18 / 20 units)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_decode_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {r: True for r in range(world)}


class _HostHead:
    """Device context stand-in for LMHead.grad: each rank's pass 2 adds
    (rank + 1) to every dX entry, as a real partial gradient would add."""

    def __init__(self, rank):
        self.rank = rank

    def lmhead_grad(self, W, v0, V_shard, H, X, T, labels, mask, n_loss, softcap, chunk, rmax, rsum, dX,
                    products=0):
        dX += float(self.rank + 1)


def _head_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tier_b200.host import LMHead
        head = LMHead.__new__(LMHead)
        head.ctx, head.W, head.v0, head.V_shard, head.H = _HostHead(rank), None, 0, 8, 4
        head.chunk, head.products, head.group = 256, 0, dist.group.WORLD
        X = torch.zeros(5, 4)
        dX = torch.full((5, 4), 10.0)                       # an existing gradient to accumulate into
        out = head.grad(X, None, None, 4, None, None, dX=dX)
        want = 10.0 + sum(r + 1 for r in range(world))       # 10 once, plus every rank's part
        q.put((rank, bool(out is dX and torch.all(dX == want))))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_lmhead_grad_accumulates_once_gloo():
    """LMHead.grad with a group adds the all-reduced parts to dX without
    summing dX's previous contents across ranks."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_head_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
