"""Data-parallel gradient reduction for the PKM layers.

Tokens are independent in the memory lookup, so the layer shards over the
batch: every rank holds the full (replicated) value table and runs its own
tokens, and the gradients are summed across ranks.  The value table's
gradient is the large one (``[n_keys^2, v_dim]``, 512 MiB in bf16 at
BASELINE config 2); ``ShardedTableGrad`` fuses its exchange into the bag
backward (rows stored to their owners over NVLink while the segment pass
computes, owner-side reduction and all-gather beside the rest of the
backward).  ``GradReducer`` all-reduces every other gradient from its
post-accumulate hook as soon as it exists, and without a
``ShardedTableGrad`` the table's too (plain NCCL).  BatchNorm statistics
stay per rank, as the reference's ``nn.BatchNorm1d`` does under data
parallelism.
"""
from __future__ import annotations

from typing import Iterable, List, Optional

import torch
import torch.distributed as dist


class ShardedTableGrad:
    """Data-parallel gradient of a value table, exchanged while it is computed.

    Rank ``o`` owns table rows ``[o*S, (o+1)*S)`` (``S = ceil(K / world)``).
    In the bag backward, the segment pass stores each row's gradient straight
    into the owner's receive buffer over NVLink (``pkm_bag_bwd_sharded``:
    the reduce-scatter runs inside the compute).  On a side stream, after a
    barrier, every owner sums the ``world`` partial copies of its rows and
    stores the result into every rank's gradient buffer
    (``pkm_grad_shard_reduce``: the all-gather), beside the rest of the
    backward; a second barrier completes the exchange.  Both buffers are
    symmetric memory (peer-addressable).  ``max_blocks`` > 0 caps the owner
    kernel's grid (0: one pass over the shard with a full grid); the default
    leaves most SMs to the rest of the backward, which the kernel overlaps
    (measured best on two B200s).  ``wait()``
    orders the caller's
    stream after the exchange; the gradient is the symmetric buffer itself.

    Replaces the data-parallel all-reduce of ``values.weight.grad`` that the
    reference gets from DDP around ``embedding_bag_bw_rev_indices``.
    """

    def __init__(self, weight: torch.nn.Parameter, group: Optional[dist.ProcessGroup] = None,
                 average: bool = False, max_blocks: int = 64):
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
        self.recv = symm_mem.empty((self.world, self.shard_rows, D), dtype=weight.dtype, device=dev)
        self.full = symm_mem.empty((self.world * self.shard_rows, D), dtype=weight.dtype, device=dev)
        h_recv = symm_mem.rendezvous(self.recv, self.group)
        h_full = symm_mem.rendezvous(self.full, self.group)
        self.recv_ptrs = [int(h_recv.buffer_ptrs[i]) for i in range(self.world)]
        self.full_ptrs = [int(h_full.buffer_ptrs[i]) for i in range(self.world)]
        self._handles = (h_recv, h_full)
        self.scale = 1.0 / self.world if average else 1.0
        self.max_blocks = max_blocks
        self.side = torch.cuda.Stream(dev)
        self.flag = torch.zeros(1, device=dev)
        self.done = None
        self.weight = weight
        weight._pkm_grad_exchange = self

    def backward(self, indices, weight, psw, grad_out, need_dpsw: bool):
        """Bag backward of one step: returns (table gradient, psw gradient);
        the table gradient is complete after ``wait()``."""
        from . import _native

        dpsw = _native.bag_bwd_sharded(indices, weight, psw, grad_out, self.recv_ptrs, self.rank, self.shard_rows,
                                       need_dpsw=need_dpsw)
        self.side.wait_stream(torch.cuda.current_stream(weight.device))
        with torch.cuda.stream(self.side):
            dist.all_reduce(self.flag, group=self.group)  # every rank's rows are in the receive buffers
            _native.grad_shard_reduce(self.recv, self.K, self.rank, self.shard_rows, self.full_ptrs, self.scale,
                                      self.max_blocks)
            dist.all_reduce(self.flag, group=self.group)  # every shard is in every rank's gradient
            self.done = torch.cuda.Event()
            self.done.record(self.side)
        return self.full[: self.K], dpsw

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
                 sharded: Iterable[ShardedTableGrad] = (), bucket_bytes: int = 1 << 20):
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
