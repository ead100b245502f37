"""Embedding bag over a value table split by rows across ranks.

For tables that should not be replicated, rank ``o`` of the group keeps only
rows ``[o*S, (o+1)*S)`` of the ``[K, D]`` table (``S = ceil(K / world)``) and
serves the lookups that every rank routes to it:

forward, on every rank (its own bags ``indices [B, L]``, weights ``[B, L]``):

1. each occurrence ``(b, j)`` goes to the owner of its row; occurrences are
   partitioned by owner with a stable sort (bag order kept inside each
   owner's part; ``pkm_route_pack``) and exchanged with one NCCL all-to-all;
2. each owner sums, per (source rank, bag) segment (``pkm_route_segments``),
   the weighted rows of its shard (``pkm_segment_sum``: the bag kernel over
   ragged entry lists);
3. the partial sums go back with a second all-to-all, and each rank adds the
   partials of a bag in owner order (``pkm_route_combine``).

backward: the upstream-gradient rows of the bags go to the owners (one
all-to-all), each owner runs the sorted-segment backward over the entries it
served (``pkm_bag_bwd_ragged``: gradient of its own rows, per-entry weight
gradients), and the per-entry weight gradients come back (one all-to-all).
The table gradient is local to its owner: nothing is all-reduced.

Over a non-NCCL group (gloo) the collectives take host copies of the
device tensors; the kernels are the same.

Counterpart of the row-sharded mode planned for the reference's bag
(``pkm/xformer_embeddingbag.py:97-138, 331-386``) when the table is split
over the ranks of a data-parallel group.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist
from torch import nn

from . import _native


def _bounce(group) -> bool:
    """Collectives of a non-NCCL group (gloo) take host tensors."""
    return dist.get_backend(group) != "nccl"


def _all_to_all(t: torch.Tensor, send_counts: List[int], recv_counts: List[int], group) -> torch.Tensor:
    """Uneven all-to-all along dim 0."""
    src = t.contiguous()
    dev = src.device
    if _bounce(group) and src.is_cuda:
        src = src.cpu()
    out = torch.empty((sum(recv_counts),) + tuple(t.shape[1:]), dtype=t.dtype, device=src.device)
    dist.all_to_all_single(out, src, output_split_sizes=recv_counts, input_split_sizes=send_counts, group=group)
    return out.to(dev)


def _exchange_counts(send: torch.Tensor, group) -> torch.Tensor:
    """Per-peer counts: ``recv[r]`` = what rank r sends here."""
    src = send.cpu() if (_bounce(group) and send.is_cuda) else send
    recv = torch.empty_like(src)
    dist.all_to_all_single(recv, src, group=group)
    return recv.to(send.device)


class _RowShardedBag(torch.autograd.Function):
    @staticmethod
    def forward(ctx, indices, psw, shard, shard_rows, group):
        world = dist.get_world_size(group)
        B, L = indices.shape
        n = B * L
        # 1. pack by owner (stable), and this rank's (owner, bag) segments:
        #    the owners return one partial row per segment, in this order
        send_t, order, local_row, bag, w = _native.route_pack(indices, psw, shard_rows, world)
        _, _, my_seg_bag, back_recv_t = _native.route_segments(bag, send_t, world)
        # every peer learns its receive counts and whether each sender's
        # indices were all inside the table (so that all ranks raise together)
        valid = (send_t.sum() == n).to(torch.int64).expand(world)
        recv2 = _exchange_counts(torch.stack([send_t, valid], 1), group)
        recv_t = recv2[:, 0].contiguous()
        counts = torch.cat([send_t, recv2[:, 0], recv2[:, 1], back_recv_t]).tolist()
        send_counts, recv_counts = counts[:world], counts[world:2 * world]
        senders_ok, back_recv = counts[2 * world:3 * world], counts[3 * world:]
        if not all(senders_ok):
            if sum(send_counts) != n:
                if indices.is_cuda:
                    _native.read_device_errors(indices.device)  # consume the flag the pack raised
                raise IndexError("row index outside the sharded table")
            raise IndexError(f"row index outside the sharded table on rank(s) "
                             f"{[r for r, ok in enumerate(senders_ok) if not ok]}")
        r_row = _all_to_all(local_row, send_counts, recv_counts, group)
        r_w = _all_to_all(w, send_counts, recv_counts, group)
        r_bag = _all_to_all(bag, send_counts, recv_counts, group)
        # 2. the owner's segments: one per (source rank, bag), source order
        r_seg_of, r_seg_start, _, back_send_t = _native.route_segments(r_bag, recv_t, world)
        back_send = back_send_t.tolist()
        n_seg = sum(back_send)
        partial = _native.segment_sum(shard, r_row, r_w, r_seg_start[:n_seg + 1], out_dtype=shard.dtype)
        # 3. partial sums back to their sources, added per bag in owner order
        got = _all_to_all(partial, back_send, back_recv, group)
        my_seg_bag = my_seg_bag[:sum(back_recv)]
        out = _native.route_combine(got, my_seg_bag, back_recv_t, world, B, out_dtype=shard.dtype)
        ctx.save_for_backward(order, r_row, r_w, r_seg_of, my_seg_bag, shard)
        ctx.counts = (send_counts, recv_counts, back_send, back_recv)
        ctx.group = group
        ctx.shape = (B, L)
        ctx.psw_dtype = psw.dtype
        return out

    @staticmethod
    def backward(ctx, d_out):
        order, r_row, r_w, r_seg_of, my_seg_bag, shard = ctx.saved_tensors
        send_counts, recv_counts, back_send, back_recv = ctx.counts
        group = ctx.group
        B, L = ctx.shape
        # the upstream rows of this rank's (owner, bag) segments go to the owners
        rows_out = d_out.to(shard.dtype).contiguous().index_select(0, my_seg_bag)
        rows_in = _all_to_all(rows_out, back_recv, back_send, group)
        dW, dpsw_recv = _native.bag_bwd_ragged(r_row, r_seg_of, r_w, shard, rows_in,
                                               need_dpsw=ctx.needs_input_grad[1])
        d_psw = None
        if ctx.needs_input_grad[1]:
            back = _all_to_all(dpsw_recv, recv_counts, send_counts, group)
            d_flat = torch.empty(B * L, dtype=torch.float32, device=shard.device)
            d_flat[order.long()] = back
            d_psw = d_flat.view(B, L).to(ctx.psw_dtype)
        return None, d_psw, dW, None, None


class RowShardedEmbeddingBag(nn.Module):
    """Weighted bag sum over a ``[num_rows, dim]`` table stored by rows across
    the ranks of ``group``: this rank holds ``weight`` = rows
    ``[rank*S, rank*S + S)`` (``S = ceil(num_rows / world)``, the last shard
    padded).  ``forward(indices [B, L], per_sample_weights [B, L])`` returns
    ``[B, dim]`` like ``xFormerEmbeddingBag`` over the whole table; every
    rank of the group must call it (collectives)."""

    def __init__(self, num_rows: int, dim: int, group: Optional[dist.ProcessGroup] = None,
                 dtype: torch.dtype = torch.float32, device=None):
        super().__init__()
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.num_rows, self.dim = num_rows, dim
        self.shard_rows = -(-num_rows // self.world)
        self.weight = nn.Parameter(torch.empty((self.shard_rows, dim), dtype=dtype, device=device))

    def load_full(self, full: torch.Tensor):
        """Copy this rank's rows out of a full ``[num_rows, dim]`` table."""
        r0 = self.rank * self.shard_rows
        r1 = min(r0 + self.shard_rows, self.num_rows)
        with torch.no_grad():
            self.weight.zero_()
            if r1 > r0:
                self.weight[: r1 - r0].copy_(full[r0:r1])

    def forward(self, indices: torch.Tensor, per_sample_weights: torch.Tensor) -> torch.Tensor:
        return _RowShardedBag.apply(indices.contiguous(), per_sample_weights.contiguous(), self.weight,
                                    self.shard_rows, self.group)


# ---------------------------------------------------------------------------
# the fast-weight memory's value table, split by rows
# ---------------------------------------------------------------------------
class FwRoute:
    """The routing of one chunk's lookups ``indices [B, L]`` (weights
    ``psw [B, L]``) to the owners of their rows, built once per chunk and
    shared by the forward, the backward and the double backward of
    :func:`fw_sharded_bag`.  Every rank of ``group`` builds its route in the
    same step (collectives)."""

    def __init__(self, indices: torch.Tensor, psw: torch.Tensor, shard_rows: int, group):
        self.group = group
        world = dist.get_world_size(group)
        self.world = world
        B, L = indices.shape
        self.B, self.L = B, L
        n = B * L
        send_t, order, local_row, bag, w = _native.route_pack(indices.contiguous(), psw.detach().contiguous(),
                                                              shard_rows, world)
        _, _, my_seg_bag, back_recv_t = _native.route_segments(bag, send_t, world)
        valid = (send_t.sum() == n).to(torch.int64).expand(world)
        recv2 = _exchange_counts(torch.stack([send_t, valid], 1), group)
        recv_t = recv2[:, 0].contiguous()
        counts = torch.cat([send_t, recv2[:, 0], recv2[:, 1], back_recv_t]).tolist()
        self.send, self.recv = counts[:world], counts[world:2 * world]
        senders_ok, self.back_recv = counts[2 * world:3 * world], counts[3 * world:]
        if not all(senders_ok):
            if sum(self.send) != n:
                if indices.is_cuda:
                    _native.read_device_errors(indices.device)
                raise IndexError("row index outside the sharded table")
            raise IndexError(f"row index outside the sharded table on rank(s) "
                             f"{[r for r, ok in enumerate(senders_ok) if not ok]}")
        self.order = order.long()
        self.r_row = _all_to_all(local_row, self.send, self.recv, group)
        self.r_w = _all_to_all(w, self.send, self.recv, group)
        r_bag = _all_to_all(bag, self.send, self.recv, group)
        self.r_seg_of, r_seg_start, _, back_send_t = _native.route_segments(r_bag, recv_t, world)
        self.back_send = back_send_t.tolist()
        self.r_seg_start = r_seg_start[:sum(self.back_send) + 1]
        self.my_seg_bag = my_seg_bag[:sum(self.back_recv)]
        self.back_recv_t = back_recv_t

    def bag(self, table: torch.Tensor) -> torch.Tensor:
        """``[B, D]`` weighted bag sums over ``table`` (this rank's rows of a
        row-split table): the owners' partial sums, combined per bag."""
        partial = _native.segment_sum(table.contiguous(), self.r_row, self.r_w, self.r_seg_start,
                                      out_dtype=table.dtype)
        got = _all_to_all(partial, self.back_send, self.back_recv, self.group)
        return _native.route_combine(got, self.my_seg_bag, self.back_recv_t, self.world, self.B,
                                     out_dtype=table.dtype)

    def rows_to_owners(self, d_out: torch.Tensor, dtype) -> torch.Tensor:
        """The rows of ``d_out [B, D]`` that each owner's segments read."""
        rows = d_out.to(dtype).contiguous().index_select(0, self.my_seg_bag.long())
        return _all_to_all(rows, self.back_recv, self.back_send, self.group)

    def entries_home(self, vals: torch.Tensor) -> torch.Tensor:
        """Per-entry values computed by the owners, back in ``[B, L]`` order."""
        back = _all_to_all(vals, self.recv, self.send, self.group)
        flat = torch.empty(self.B * self.L, dtype=vals.dtype, device=vals.device)
        flat[self.order] = back
        return flat.view(self.B, self.L)


class _FwShardedBagBW(torch.autograd.Function):
    """The owner's table gradient ``dW[k] = sum psw[b,j] d_out[b]`` as a
    differentiable function of ``psw`` and ``d_out`` (the double backward
    of the sharded bag, as ``EmbeddingBagBW`` is for the whole table):
    ``d(d_out)[b] = sum_j psw[b,j] gbar[idx[b,j]]`` is the sharded bag over
    ``gbar``, ``d(psw)[b,j] = <gbar[idx[b,j]], d_out[b]>`` the owners'
    per-entry dot products."""

    @staticmethod
    def forward(ctx, psw, d_out, route, rows_in, dW):
        ctx.route = route
        ctx.save_for_backward(rows_in)
        ctx.psw_dtype, ctx.dout_dtype = psw.dtype, d_out.dtype
        return dW

    @staticmethod
    def backward(ctx, g_bar):
        (rows_in,) = ctx.saved_tensors
        route = ctx.route
        g_bar = g_bar.contiguous()
        d_psw = d_dout = None
        if ctx.needs_input_grad[1]:
            d_dout = route.bag(g_bar).to(ctx.dout_dtype)
        if ctx.needs_input_grad[0]:
            _, dots = _native.bag_bwd_ragged(route.r_row, route.r_seg_of, route.r_w, g_bar, rows_in, need_dpsw=True)
            d_psw = route.entries_home(dots).to(ctx.psw_dtype)
        return d_psw, d_dout, None, None, None


class _FwShardedBag(torch.autograd.Function):
    @staticmethod
    def forward(ctx, shard, psw, route):
        ctx.route = route
        ctx.save_for_backward(shard, psw)
        return route.bag(shard)

    @staticmethod
    def backward(ctx, d_out):
        shard, psw = ctx.saved_tensors
        route = ctx.route
        rows_in = route.rows_to_owners(d_out, shard.dtype)
        dW, dots = _native.bag_bwd_ragged(route.r_row, route.r_seg_of, route.r_w, shard.detach(), rows_in,
                                          need_dpsw=ctx.needs_input_grad[1])
        d_psw = route.entries_home(dots).to(psw.dtype) if ctx.needs_input_grad[1] else None
        grad_shard = _FwShardedBagBW.apply(psw, d_out, route, rows_in, dW) if ctx.needs_input_grad[0] else None
        return grad_shard, d_psw, None


def fw_sharded_bag(indices: torch.Tensor, shard: torch.Tensor, psw: torch.Tensor, shard_rows: int, group):
    """Weighted bag sums ``[B, D]`` of ``indices [B, L]`` over a row-split
    table of which this rank holds ``shard`` (rows ``[rank*S, rank*S + S)``),
    with a table gradient that is differentiable once more (the fast-weight
    memory's inner update).  Returns ``(out, route)``; ``route.r_row`` are
    the shard rows of the entries this rank served (its slot counts)."""
    route = FwRoute(indices, psw, shard_rows, group)
    return _FwShardedBag.apply(shard, psw, route), route
