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
