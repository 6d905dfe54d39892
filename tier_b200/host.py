"""Host-side mirror of the reference's linear operators and LM-head loop.

The reference (tier/tier.cpp) drives its hot path from C++ statics:
``linear`` / ``linear_dx`` / ``linear_dx_acc`` (1202-1238), ``chat_lin``
(2351-2378) and the two LM-head passes inside main (3184-3266).  These classes
keep those operations' meaning on top of the libtierk C ABI, and add the
row / vocab sharding across GPUs (one process per GPU, NCCL through
torch.distributed) that the reference does not have.

Sharding (weights split by output rows, vocab split by rows of the head):
  * linear fwd: rank g owns W[N_g, K]; Y[:, N_g] is computed locally and, if
    the caller wants the full Y, all-gathered.
  * linear dX: rank g computes dY[:, N_g] . W[N_g, :] and the partial dX are
    all-reduced (SUM), or reduce-scattered by token rows inside the GEMM.
  * decode (chat_lin, 1..16 tokens): rank g runs the GEMV on its rows and the
    y shards are all-gathered into [M, N_total].
  * LM head: rank g owns head rows [v0_g, v0_g + V_g).  After the local pass
    1 the running states are merged with all-reduce MAX of rmax, a local
    rescale, all-reduce SUM of rsum and of the target logit (only the owning
    shard has a non-zero target), and an argmax exchange; pass 2 then uses
    the global lse and dX is all-reduced (SUM).
"""
from __future__ import annotations

import torch

from . import DT_BF16, DT_F16, DT_F32, F16X2, WFROZEN, X3_AUTO, X3_REF, Context, Weight, make_weight

_DT = {torch.float32: DT_F32, torch.float16: DT_F16, torch.bfloat16: DT_BF16}


def shard_rows(n: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """Contiguous row range of `rank` when n rows are split over `world` ranks,
    every boundary a multiple of `align`."""
    units = n // align
    a = units * rank // world * align
    b = units * (rank + 1) // world * align if rank + 1 < world else n
    return a, b


def merge_vocab_shards(rmax, rsum, amax, tgt, group, rescale, dX=None):
    """Merge per-shard running CE state into the global one, in place for
    rmax / rsum / tgt; returns the merged argmax.  Shards are in vocab order
    (rank r holds a lower vocab range than rank r+1).

      argmax: all-gather (max, index); the highest max wins, a tie goes to the
              lower rank, i.e. the lower vocab index (the reference's rule).
      rmax:   all-reduce MAX.
      rsum:   each shard rescales its sum to the global max
              (rescale(rmax_local, rsum_local, rmax_global)), then all-reduce SUM.
      tgt:    all-reduce SUM (only the shard holding the label has it non-zero).
      dX:     (single-pass accumulator, optional) rescaled with rsum; the
              caller all-reduces it after tk_lmhead_finish."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    allm = [torch.empty_like(rmax) for _ in range(world)]
    alla = [torch.empty_like(amax) for _ in range(world)]
    dist.all_gather(allm, rmax.clone(), group=group)
    dist.all_gather(alla, amax.clone(), group=group)
    best = torch.argmax(torch.stack(allm), dim=0)          # first maximal rank
    merged = torch.stack(alla).gather(0, best[None]).squeeze(0).contiguous()
    gmax = rmax.clone()
    dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
    rescale(rmax, rsum, gmax, dX)
    dist.all_reduce(rsum, group=group)
    dist.all_reduce(tgt, group=group)
    return merged


def gather_cols(local: torch.Tensor, group) -> torch.Tensor:
    """All-gather the column shards local [M, n_rank] of every rank, in rank
    order, into [M, sum n_rank].  Shards may differ in width (row splits that
    do not divide evenly): collectives want equal sizes, so short shards are
    padded to the widest and the padding is dropped after the exchange."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    M, n = local.shape
    sizes = [torch.zeros(1, dtype=torch.int64, device=local.device) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([n], dtype=torch.int64, device=local.device), group=group)
    ns = [int(t.item()) for t in sizes]
    nmax = max(ns)
    if n == nmax:
        send = local.contiguous()
    else:
        send = torch.zeros(M, nmax, device=local.device, dtype=local.dtype)
        send[:, :n] = local
    buf = torch.empty(world * M, nmax, device=local.device, dtype=local.dtype)
    dist.all_gather_into_tensor(buf, send, group=group)
    return torch.cat([buf[r * M:(r + 1) * M, : ns[r]] for r in range(world)], dim=1)


def connect_peers(ctx: Context, group, recv_bytes: int) -> None:
    """Set up the library's peer buffers on every rank of `group` (one
    exchange of CUDA IPC handles through torch.distributed, then a barrier).
    Afterwards the context's collectives (tk_allgather, tk_allreduce_f32,
    tk_lmhead_merge, tk_linear_dx_rs) run over NVLink without NCCL; a C++
    caller does the same exchange with its own bootstrap."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    h = ctx.comm_init(rank, world, recv_bytes)
    mine = torch.tensor(list(h), dtype=torch.uint8, device=torch.device("cuda", ctx.device))
    allh = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allh, mine, group=group)
    ctx.comm_connect(bytes(torch.cat(allh).cpu().tolist()))
    dist.barrier(group=group)
    ctx.peers = (rank, world)


def gather_cols_peer(ctx: Context, local: torch.Tensor) -> torch.Tensor:
    """gather_cols over the library's peer buffers (tk_allgather): the ranks'
    widths first (one 16-byte record each), then every rank's [M, n_rank]
    shard padded to the widest, in rank order."""
    M, n = local.shape
    world = ctx.peers[1]
    rec = torch.zeros(4, dtype=torch.int32, device=local.device)
    rec[0] = n
    allrec = torch.empty(4 * world, dtype=torch.int32, device=local.device)
    ctx.allgather(rec, allrec)
    widths = [int(v) for v in allrec.view(world, 4)[:, 0].tolist()]
    nmax = (max(widths) + 3) // 4 * 4        # whole 16-byte rows of fp32
    send = local.contiguous() if n == nmax else torch.zeros(M, nmax, device=local.device, dtype=local.dtype)
    if n != nmax:
        send[:, :n] = local
    buf = torch.empty(world * M, nmax, device=local.device, dtype=local.dtype)
    ctx.allgather(send, buf)
    return torch.cat([buf[r * M:(r + 1) * M, : widths[r]] for r in range(world)], dim=1)


class LinearPath:
    """One frozen projection W[N, K] (block-quantized, fp16, or fp32 split into
    fp16 hi/lo) on this rank's device, optionally row-sharded across `group`."""

    def __init__(self, ctx: Context, qtype: int, rows: int, cols: int, data: torch.Tensor, scale_log2: int = 0,
                 group=None, n_total: int | None = None, row0: int = 0, align: int = 1):
        self.ctx = ctx
        self.data = data
        self.W: Weight = make_weight(qtype, rows, cols, data, scale_log2)
        self.N, self.K = rows, cols
        self.group = group
        self.n_total = n_total if n_total is not None else rows
        self.row0 = row0
        self.align = align          # row-shard boundaries are multiples of this (shard_rows)

    @staticmethod
    def from_f32_split(ctx: Context, W32: torch.Tensor, **kw) -> "LinearPath":
        rows, cols = W32.shape
        planes = torch.empty(2 * rows * cols, dtype=torch.float16, device=W32.device)
        s = ctx.weight_split_f32(W32, rows, cols, planes)
        return LinearPath(ctx, F16X2, rows, cols, planes, scale_log2=s, **kw)

    def forward(self, X: torch.Tensor, Y: torch.Tensor | None = None, beta: float = 0.0, products: int = X3_AUTO,
                gather: bool = True) -> torch.Tensor:
        """Y = X . W^T (the reference's `linear`).  With a group and gather=True
        the output shards are all-gathered into the full [M, N_total]."""
        M = X.shape[0]
        direct = Y is not None and self.group is None      # the GEMM writes (beta: accumulates into) Y itself
        local = Y if direct else torch.empty(M, self.N, device=X.device, dtype=torch.float32)
        self.ctx.linear(self.W, X, M, local, x_dtype=_DT[X.dtype], ldx=X.stride(0), ldy=local.stride(0),
                        beta=beta if direct else 0.0, products=products)
        if self.group is None or not gather:
            return local
        full = self._gather(local)
        if Y is not None:
            if beta:
                Y += full
            else:
                Y.copy_(full)
            return Y
        return full

    def decode(self, x: torch.Tensor, y: torch.Tensor | None = None, frozen: bool = True,
               gather: bool = True) -> torch.Tensor:
        """y = x . W^T for 1..16 tokens x [M, K] fp32 on the decode GEMV
        (`chat_lin`, tier/tier.cpp:2351-2378).  Block-quantized and dense
        weights; `frozen`: W is never rewritten (early weight fetch).  With a
        group and gather=True the rows' y shards are all-gathered into the
        full [M, N_total] (one collective; shorter shards are padded)."""
        M = x.shape[0]
        qt = self.W.qtype | (WFROZEN if frozen else 0)
        local = y if (y is not None and self.group is None) else torch.empty(M, self.N, device=x.device,
                                                                               dtype=torch.float32)
        self.ctx.gemv(qt, self.data, self.N, self.K, x, local, M=M, ldx=x.stride(0), ldy=local.stride(0),
                      row_bytes_=self.W.row_bytes)
        if self.group is None or not gather:
            return local
        full = self._gather(local)
        if y is not None:
            y.copy_(full)
            return y
        return full

    def _gather(self, local: torch.Tensor) -> torch.Tensor:
        """The output shards of every rank side by side: over the library's
        peer buffers once they are connected, else with torch.distributed."""
        if getattr(self.ctx, "peers", None) is None:
            return gather_cols(local, self.group)
        return gather_cols_peer(self.ctx, local)

    def enable_reduce_scatter(self, M_max: int):
        """Set up the peer buffers for `dx_rs` and the peer all-gather (one
        collective exchange of IPC handles, then a barrier); M_max bounds the
        token count."""
        import torch.distributed as dist
        world = dist.get_world_size(self.group)
        nmax = (max(self.N, -(-self.n_total // world)) + self.align + 3) // 4 * 4   # widest output shard
        connect_peers(self.ctx, self.group, max(M_max * self.K * 4, world * M_max * nmax * 4))
        self.rs_world, self.rs_rank = world, self.ctx.peers[0]

    def dx_rs(self, dY: torch.Tensor, out: torch.Tensor | None = None, products: int = X3_AUTO) -> torch.Tensor:
        """This rank's token rows (rank * M/world ...) of dX = sum_g dY_g . W_g,
        reduce-scattered inside the dX GEMM over peer memory."""
        M = dY.shape[0]
        rows = M // self.rs_world
        if out is None:
            out = torch.empty(rows, self.K, device=dY.device, dtype=torch.float32)
        self.ctx.linear_dx_rs(self.W, dY, M, out, dy_dtype=_DT[dY.dtype], lddy=dY.stride(0), ldd=out.stride(0),
                              products=products)
        return out

    def fwd_dx_rs(self, X: torch.Tensor, dY: torch.Tensor, products: int = X3_AUTO):
        """The training step's two passes through this shard in one launch:
        (Y, dX rows) with Y = X . W_g^T (this rank's columns, not gathered)
        and dX rows as `dx_rs`; the forward tiles compute while the dX tiles'
        stores cross NVLink (tk_linear_fwd_dx_rs)."""
        Mx, M = X.shape[0], dY.shape[0]
        Y = torch.empty(Mx, self.N, device=X.device, dtype=torch.float32)
        out = torch.empty(M // self.rs_world, self.K, device=dY.device, dtype=torch.float32)
        self.ctx.linear_fwd_dx_rs(self.W, X, Mx, Y, dY, M, out, x_dtype=_DT[X.dtype], dy_dtype=_DT[dY.dtype],
                                  ldx=X.stride(0), ldy=Y.stride(0), lddy=dY.stride(0), ldd=out.stride(0),
                                  products=products)
        return Y, out

    def dx(self, dY: torch.Tensor, dX: torch.Tensor | None = None, beta: float = 0.0,
           products: int = X3_AUTO) -> torch.Tensor:
        """dX = dY . W (`linear_dx`; beta=1 is `linear_dx_acc`).  dY holds this
        rank's N columns; partial results are all-reduced across the group."""
        M = dY.shape[0]
        if self.group is None:
            out = dX if dX is not None else torch.empty(M, self.K, device=dY.device, dtype=torch.float32)
            self.ctx.linear_dx(self.W, dY, M, out, dy_dtype=_DT[dY.dtype], lddy=dY.stride(0), lddx=out.stride(0),
                               beta=beta if dX is not None else 0.0, products=products)
            return out
        import torch.distributed as dist
        part = torch.empty(M, self.K, device=dY.device, dtype=torch.float32)
        self.ctx.linear_dx(self.W, dY, M, part, dy_dtype=_DT[dY.dtype], lddy=dY.stride(0), lddx=part.stride(0),
                           products=products)
        dist.all_reduce(part, group=self.group)
        if dX is None:
            return part
        if beta:
            dX += part
        else:
            dX.copy_(part)
        return dX


class LMHead:
    """Chunked-vocabulary LM head + cross-entropy over this rank's vocab shard
    (W fp16 [V_shard, H], global rows v0 .. v0+V_shard)."""

    def __init__(self, ctx: Context, W: torch.Tensor, v0: int, chunk: int = 16384, products: int = X3_REF,
                 group=None):
        assert W.dtype == torch.float16 and W.is_contiguous()
        self.ctx, self.W, self.v0 = ctx, W, v0
        self.V_shard, self.H = W.shape
        self.chunk, self.products, self.group = chunk, products, group

    def stats(self, X, labels, mask, softcap=0.0):
        T = X.shape[0]
        dev = X.device
        rmax = torch.full((T - 1,), -1e30, dtype=torch.float64, device=dev)
        rsum = torch.zeros(T - 1, dtype=torch.float64, device=dev)
        amax = torch.full((T - 1,), -1, dtype=torch.int32, device=dev)
        tgt = torch.zeros(T - 1, dtype=torch.float32, device=dev)
        self.ctx.lmhead_stats(self.W, self.v0, self.V_shard, self.H, X, T, labels, mask, softcap, self.chunk, rmax,
                              rsum, amax, tgt, products=self.products)
        if self.group is not None:
            if getattr(self.ctx, "peers", None) is not None:
                self.ctx.lmhead_merge(T - 1, rmax, rsum, amax, tgt)
            else:
                amax = merge_vocab_shards(rmax, rsum, amax, tgt, self.group,
                                          lambda rl, sl, rg, d: self.ctx.lmhead_rescale(T - 1, rl, sl, rg))
        return rmax, rsum, amax, tgt

    def loss(self, T, labels, mask, rmax, rsum, amax, tgt):
        loss = torch.zeros(1, dtype=torch.float64, device=rmax.device)
        hits = torch.zeros(1, dtype=torch.int32, device=rmax.device)
        self.ctx.lmhead_loss(T, labels, mask, rmax, rsum, amax, tgt, loss, hits)
        return loss, hits

    def grad(self, X, labels, mask, n_loss, rmax, rsum, dX=None, softcap=0.0):
        """dX += this head's input gradient (pass 2).  With a group, each rank's
        part goes into a zeroed buffer that is all-reduced before it is added,
        so a dX that already holds a gradient is not summed across ranks."""
        T, H = X.shape
        if dX is None:
            dX = torch.zeros(T, H, dtype=torch.float32, device=X.device)
        part = dX if self.group is None else torch.zeros(T, H, dtype=torch.float32, device=X.device)
        self.ctx.lmhead_grad(self.W, self.v0, self.V_shard, self.H, X, T, labels, mask, n_loss, softcap, self.chunk,
                             rmax, rsum, part, products=self.products)
        if self.group is not None:
            self._allreduce(part)
            dX += part
        return dX

    def _allreduce(self, buf):
        if getattr(self.ctx, "peers", None) is not None:
            self.ctx.allreduce_f32(buf)
        else:
            import torch.distributed as dist
            dist.all_reduce(buf, group=self.group)

    def step(self, X, labels, mask, softcap=0.0, dX=None):
        """Both passes: returns (loss_sum, n_loss, hits, amax, dX)."""
        T = X.shape[0]
        n_loss = int(mask[: T - 1].count_nonzero().item())
        rmax, rsum, amax, tgt = self.stats(X, labels, mask, softcap)
        loss, hits = self.loss(T, labels, mask, rmax, rsum, amax, tgt)
        dX = self.grad(X, labels, mask, n_loss, rmax, rsum, dX=dX, softcap=softcap)
        return loss, n_loss, hits, amax, dX

    def step_fused(self, X, labels, mask, softcap=0.0, n_loss=None):
        """Single pass (one logits GEMM per chunk): returns (loss_sum, n_loss,
        hits, amax, dX), the same quantities as `step`.  With a group, every
        rank's accumulator is rescaled to the global max, finished against
        the global sum, and the per-rank dX are all-reduced (SUM)."""
        T, H = X.shape
        dev = X.device
        if n_loss is None:
            n_loss = int(mask[: T - 1].count_nonzero().item())
        rmax = torch.full((T - 1,), -1e30, dtype=torch.float64, device=dev)
        rsum = torch.zeros(T - 1, dtype=torch.float64, device=dev)
        amax = torch.full((T - 1,), -1, dtype=torch.int32, device=dev)
        tgt = torch.zeros(T - 1, dtype=torch.float32, device=dev)
        dX = torch.zeros(T, H, dtype=torch.float32, device=dev)
        self.ctx.lmhead_fused(self.W, self.v0, self.V_shard, self.H, X, T, labels, mask, softcap, self.chunk, rmax,
                              rsum, amax, tgt, dX, products=self.products)
        if self.group is not None:
            if getattr(self.ctx, "peers", None) is not None:
                self.ctx.lmhead_merge(T - 1, rmax, rsum, amax, tgt, dX, H)
            else:
                amax = merge_vocab_shards(rmax, rsum, amax, tgt, self.group,
                                          lambda rl, sl, rg, d: self.ctx.lmhead_rescale(T - 1, rl, sl, rg, d, H),
                                          dX=dX)
        self.ctx.lmhead_finish(self.W, self.v0, self.V_shard, self.H, T, labels, mask, n_loss, softcap, rsum, tgt, dX)
        if self.group is not None:
            self._allreduce(dX)
        loss, hits = self.loss(T, labels, mask, rmax, rsum, amax, tgt)
        return loss, n_loss, hits, amax, dX


__all__ = ["LinearPath", "LMHead", "shard_rows", "merge_vocab_shards", "gather_cols", "gather_cols_peer",
           "connect_peers"]
