"""Data-parallel gradient reduction for the PKM layers.

Tokens are independent in the memory lookup, so the layer shards over the
batch: every rank holds the full (replicated) value table and runs its own
tokens, and the gradients are summed across ranks.  The value table's
gradient is the large one (``[n_keys^2, v_dim]``, 512 MiB in bf16 at
benchmark config 2); ``ShardedTableGrad`` fuses its exchange into the bag
backward (rows stored to their owners over NVLink while the segment pass
computes, owner-side reduction and all-gather beside the rest of the
backward); ``RowOwnerSGD`` instead shards the table's optimizer by rows
(reduce-scatter inside the bag backward, owner update, all-gather of the
updated rows).  ``GradReducer`` all-reduces every other gradient from its
post-accumulate hook as soon as it exists, and without either of them the
table's too (plain NCCL).  BatchNorm statistics
stay per rank, as the reference's ``nn.BatchNorm1d`` does under data
parallelism.
"""
from __future__ import annotations

from typing import Iterable, List, Optional

import torch
import torch.distributed as dist


def _symm_offset(h, t: torch.Tensor, rank: int) -> int:
    """Byte offset of ``t`` inside its symmetric allocation (handle ``h``)."""
    off = t.data_ptr() - int(h.buffer_ptrs[rank])
    if off < 0 or off + t.numel() * t.element_size() > int(h.buffer_size):
        raise RuntimeError("tensor lies outside its symmetric allocation")
    return off


def _symm_peers(h, t: torch.Tensor, rank: int, world: int) -> List[int]:
    """Device addresses of ``t``'s counterpart on every rank."""
    off = _symm_offset(h, t, rank)
    return [int(h.buffer_ptrs[i]) + off for i in range(world)]


class ShardedTableGrad:
    """Data-parallel gradient of a value table, exchanged over NVLink inside
    the backward.

    Rank ``o`` owns table rows ``[o*S, (o+1)*S)`` (``S = ceil(K / world)``);
    every buffer below is symmetric memory (peer-addressable, and with a
    multicast mapping where the system has NVLink SHARP).

    * ``mode="nvls"`` (``auto`` above two ranks, where multicast exists): the bag
      backward writes this rank's gradient into a symmetric buffer; after a
      barrier each owner reads its rows through the multicast address with
      ``multimem.ld_reduce`` (the switch sums the ranks' copies) and stores
      them with ``multimem.st`` into every rank's gradient
      (``pkm_grad_multimem_allreduce``); a second barrier ends the exchange.
      Each rank's link carries its rows out once and the reduced shard out
      once.
    * ``mode="p2p"`` (``auto`` at two ranks): the segment pass stores each finished row straight into
      its owner's receive buffer (``pkm_bag_bwd_sharded``: the reduce-scatter
      inside the compute); after a barrier each owner sums the ``world``
      copies and stores the rows into every rank's gradient
      (``pkm_grad_shard_reduce``); a second barrier.

    The exchange after the bag backward runs on a side stream beside the
    rest of the backward (``max_blocks`` caps its grid so that the backward
    keeps most SMs).  ``wait()`` orders the caller's stream after it; the
    table's ``.grad`` is the symmetric gradient buffer itself.

    Replaces the data-parallel all-reduce of ``values.weight.grad`` that the
    reference gets from DDP around ``embedding_bag_bw_rev_indices``.
    """

    def __init__(self, weight: torch.nn.Parameter, group: Optional[dist.ProcessGroup] = None,
                 average: bool = False, max_blocks: Optional[int] = None, mode: str = "auto", chunks: int = 2):
        import torch.distributed._symmetric_memory as symm_mem

        if mode not in ("auto", "nvls", "p2p"):
            raise ValueError(mode)
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > 8:
            raise ValueError("the fused exchange spans one NVLink domain (at most 8 ranks)")
        K, D = weight.shape
        self.K, self.D = K, D
        self.shard_rows = -(-K // self.world)
        dev = weight.device
        rows = self.world * self.shard_rows
        self.full = symm_mem.empty((rows, D), dtype=weight.dtype, device=dev)
        h_full = symm_mem.rendezvous(self.full, self.group)
        handles = [h_full]
        self.mode = "p2p"
        # measured on B200s at config 2: the NVLink stores win at two ranks
        # (3.24 vs 3.99 ms per step), the in-switch reduction at eight
        # (3.92 vs 3.97 ms)
        want_nvls = mode == "nvls" or (mode == "auto" and self.world > 2)
        if want_nvls and int(h_full.multicast_ptr) != 0:
            self.local = symm_mem.empty((rows, D), dtype=weight.dtype, device=dev)
            h_local = symm_mem.rendezvous(self.local, self.group)
            handles.append(h_local)
            if int(h_local.multicast_ptr) != 0:
                self.mode = "nvls"
                self.mc_local = int(h_local.multicast_ptr) + self._offset(h_local, self.local)
                self.mc_full = int(h_full.multicast_ptr) + self._offset(h_full, self.full)
        if mode == "nvls" and self.mode != "nvls":
            raise RuntimeError("NVLink multicast (NVLS) is not available for symmetric memory here")
        if self.mode == "p2p":
            self.recv = symm_mem.empty((self.world, self.shard_rows, D), dtype=weight.dtype, device=dev)
            h_recv = symm_mem.rendezvous(self.recv, self.group)
            handles.append(h_recv)
            self.recv_ptrs = self._peers(h_recv, self.recv)
            self.full_ptrs = self._peers(h_full, self.full)
        self._handles = handles
        self.scale = 1.0 / self.world if average else 1.0
        if max_blocks is None:  # grid cap of the side-stream kernel (measured best per mode / size)
            max_blocks = 64 if (self.mode == "nvls" or self.world <= 2) else 148
        self.max_blocks = max_blocks
        # in-switch mode: the bag backward's rows are computed and exchanged in
        # `chunks` row ranges, the exchange of one beside the pass of the next
        self.chunks = max(1, int(chunks))
        self.side = torch.cuda.Stream(dev)
        self.flag = torch.zeros(1, device=dev)
        self.done = None
        self.weight = weight
        # with `timing` set, each step's side-stream exchange is bracketed by
        # CUDA events (start of its first transfer, end of the last barrier)
        self.timing = False
        self.timed = []
        self._t0 = None
        weight._pkm_grad_exchange = self

    def _offset(self, h, t) -> int:
        return _symm_offset(h, t, self.rank)

    def _peers(self, h, t):
        return _symm_peers(h, t, self.rank, self.world)

    def backward(self, indices, weight, psw, grad_out, need_dpsw: bool):
        """Bag backward of one step: returns (table gradient, psw gradient);
        the table gradient is complete after ``wait()``."""
        from . import _native

        main = torch.cuda.current_stream(weight.device)
        if self.mode == "nvls":
            ph = _native.BagBwdPhases(indices, weight, psw, grad_out, need_dpsw=need_dpsw)
            ph.sort()
            bounds = [self.K * c // self.chunks for c in range(self.chunks + 1)]
            for r0, r1 in zip(bounds[:-1], bounds[1:]):
                ph.rows(r0, r1, self.local[: self.K])
                self.side.wait_stream(main)
                self._mark_start()
                with torch.cuda.stream(self.side):
                    dist.all_reduce(self.flag, group=self.group)  # every rank's rows [r0, r1) are written
                    _native.grad_multimem_allreduce(self.mc_local, self.mc_full, weight.dtype, self.K, self.D,
                                                    self.world, self.rank, self.shard_rows, weight.device,
                                                    self.scale, self.max_blocks, r0, r1)
            dpsw = ph.dpsw
        else:
            dpsw = _native.bag_bwd_sharded(indices, weight, psw, grad_out, self.recv_ptrs, self.rank,
                                           self.shard_rows, need_dpsw=need_dpsw)
            self.side.wait_stream(main)
            self._mark_start()
            with torch.cuda.stream(self.side):
                dist.all_reduce(self.flag, group=self.group)  # every rank's rows are in the receive buffers
                _native.grad_shard_reduce(self.recv, self.K, self.rank, self.shard_rows, self.full_ptrs,
                                          self.scale, self.max_blocks)
        with torch.cuda.stream(self.side):
            dist.all_reduce(self.flag, group=self.group)  # every shard is in every rank's gradient
            self.done = torch.cuda.Event(enable_timing=self.timing)
            self.done.record(self.side)
            if self.timing and self._t0 is not None:
                self.timed.append((self._t0, self.done))
            self._t0 = None
        return self.full[: self.K], dpsw

    def _mark_start(self):
        if self.timing and self._t0 is None:
            self._t0 = torch.cuda.Event(enable_timing=True)
            self._t0.record(self.side)

    def exchange_ms(self):
        """Mean side-stream time of the timed steps' exchanges (ms), or None."""
        if not self.timed:
            return None
        return sum(a.elapsed_time(b) for a, b in self.timed) / len(self.timed)

    def wait(self):
        """Order the current stream after this step's exchange."""
        if self.done is None:
            return
        torch.cuda.current_stream(self.weight.device).wait_event(self.done)
        self.done = None
        g = self.weight.grad
        if g is not None and g.data_ptr() != self.full.data_ptr():
            # autograd copied (or accumulated into) the gradient before the
            # exchange finished: redo it from the completed buffer
            g.copy_(self.full[: self.K])

    def close(self):
        if getattr(self.weight, "_pkm_grad_exchange", None) is self:
            del self.weight._pkm_grad_exchange


class RowOwnerSGD:
    """SGD of a replicated value table with the optimizer sharded by rows:
    reduce-scatter, row-owner update, all-gather of the parameters.

    Rank ``o`` owns table rows ``[o*S, (o+1)*S)`` (``S = ceil(K / world)``).
    The table itself is moved into symmetric memory (``weight.data`` becomes
    a view of it) so that peers can write it.  In the backward the bag
    kernel stores each finished row of this rank's gradient straight into
    its owner's receive buffer (``pkm_bag_bwd_sharded``: the reduce-scatter
    inside the compute) and returns no table gradient.  ``step()`` then, on
    the current stream: a barrier; each owner sums the ``world`` copies of
    its rows, applies ``p -= lr * (g + weight_decay * p)`` to its rows only
    and stores them into every rank's table (``pkm_grad_shard_sgd``); a
    second barrier.  Against an all-reduce of the table gradient followed by
    every rank's optimizer pass over the whole table, the gradient is never
    all-gathered and each rank's optimizer touches 1/world of the rows.

    Use it in place of the table's entry in the dense optimizer and in
    ``GradReducer`` (``sharded=[...]``); call ``step()`` after the backward
    of every step, on every rank.
    """

    def __init__(self, weight: torch.nn.Parameter, lr: float, weight_decay: float = 0.0,
                 group: Optional[dist.ProcessGroup] = None, average: bool = False, max_blocks: int = 0):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > 8:
            raise ValueError("the fused exchange spans one NVLink domain (at most 8 ranks)")
        K, D = weight.shape
        self.K, self.D = K, D
        self.shard_rows = -(-K // self.world)
        dev = weight.device
        rows = self.world * self.shard_rows
        self.table = symm_mem.empty((rows, D), dtype=weight.dtype, device=dev)
        h_table = symm_mem.rendezvous(self.table, self.group)
        self.recv = symm_mem.empty((self.world, self.shard_rows, D), dtype=weight.dtype, device=dev)
        h_recv = symm_mem.rendezvous(self.recv, self.group)
        self._handles = [h_table, h_recv]
        with torch.no_grad():
            self.table[:K].copy_(weight.data)
            self.table[K:].zero_()
        weight.data = self.table[:K]
        self.table_ptrs = _symm_peers(h_table, self.table, self.rank, self.world)
        self.recv_ptrs = _symm_peers(h_recv, self.recv, self.rank, self.world)
        self.lr, self.weight_decay = float(lr), float(weight_decay)
        self.scale = 1.0 / self.world if average else 1.0
        self.max_blocks = max_blocks
        self.flag = torch.zeros(1, device=dev)
        self.pending = False
        self.weight = weight
        weight._pkm_grad_exchange = self

    def backward(self, indices, weight, psw, grad_out, need_dpsw: bool):
        """Bag backward of one step: the table gradient goes to the row
        owners (no local gradient is returned); returns (None, psw gradient)."""
        from . import _native

        dpsw = _native.bag_bwd_sharded(indices, weight, psw, grad_out, self.recv_ptrs, self.rank, self.shard_rows,
                                       need_dpsw=need_dpsw)
        self.pending = True
        return None, dpsw

    def wait(self):
        """Nothing to wait for: the table gradient never materialises
        (``GradReducer`` calls this for every sharded table)."""

    def step(self):
        """Owner update of this step's gradient, then every rank's table
        holds every updated row.  Every rank must call it."""
        from . import _native

        if not self.pending:
            raise RuntimeError("RowOwnerSGD.step() without a backward through the table")
        dist.all_reduce(self.flag, group=self.group)  # every rank's rows are in the receive buffers
        _native.grad_shard_sgd(self.recv, self.K, self.rank, self.shard_rows, self.table_ptrs, self.lr,
                               self.weight_decay, self.scale, self.max_blocks)
        dist.all_reduce(self.flag, group=self.group)  # every shard is in every rank's table
        self.pending = False

    def close(self):
        if getattr(self.weight, "_pkm_grad_exchange", None) is self:
            del self.weight._pkm_grad_exchange


class GradReducer:
    """Sum gradients of ``params`` over ``group`` (``average`` divides by the
    world size).  A gradient of at least ``bucket_bytes`` starts its
    all-reduce, asynchronously and in its own dtype, from its
    post-accumulate-grad hook, so the transfer overlaps the rest of the
    backward; smaller ones are all-reduced together in ``finish()`` as one
    coalesced NCCL launch.  Tables handled by a ``ShardedTableGrad``
    (``sharded``) are skipped here and ``finish()`` orders the caller after
    their exchange.  ``early`` names parameters whose reduction starts from
    the hook whatever their size."""

    def __init__(self, params: Iterable[torch.nn.Parameter], early: Iterable[torch.nn.Parameter] = (),
                 group: Optional[dist.ProcessGroup] = None, average: bool = False,
                 sharded: Iterable = (), bucket_bytes: int = 1 << 20):
        self.group = group
        self.average = average
        self.sharded = list(sharded)
        skip = {id(x.weight) for x in self.sharded}
        early_ids = {id(p) for p in early}
        self.params: List[torch.nn.Parameter] = [p for p in params if id(p) not in skip and p.requires_grad]
        self.hooked = [p for p in self.params
                       if id(p) in early_ids or p.numel() * p.element_size() >= bucket_bytes]
        hooked_ids = {id(p) for p in self.hooked}
        self.small = [p for p in self.params if id(p) not in hooked_ids]
        self.pending = []
        self.handles = [p.register_post_accumulate_grad_hook(self._start) for p in self.hooked]

    def world(self) -> int:
        return dist.get_world_size(self.group)

    def _start(self, p: torch.Tensor):
        if p.grad is None:
            return
        self.pending.append((p.grad, dist.all_reduce(p.grad, group=self.group, async_op=True)))

    def finish(self):
        """Reduce the small gradients and wait for every reduction of this step."""
        from torch.distributed.distributed_c10d import _coalescing_manager

        grads = [p.grad for p in self.small if p.grad is not None]
        if grads:
            with _coalescing_manager(group=self.group, async_ops=True) as cm:
                for g in grads:
                    dist.all_reduce(g, group=self.group)
            cm.wait()
            if self.average:
                for g in grads:
                    g /= self.world()
        for g, work in self.pending:
            work.wait()
            if self.average:
                g /= self.world()
        self.pending = []
        for x in self.sharded:
            x.wait()

    def remove(self):
        for h in self.handles:
            h.remove()
        self.handles = []
