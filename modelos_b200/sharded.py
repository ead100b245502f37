"""Embedding bag over a value table split by rows across ranks.

For tables that should not be replicated, rank ``o`` of the group keeps only
rows ``[o*S, (o+1)*S)`` of the ``[K, D]`` table (``S = ceil(K / world)``) and
serves the lookups that every rank routes to it:

forward, on every rank (its own bags ``indices [B, L]``, weights ``[B, L]``):

1. each occurrence ``(b, j)`` goes to the owner of its row; occurrences are
   partitioned by owner with a stable sort (bag order kept inside each
   owner's part) and exchanged with one NCCL all-to-all;
2. each owner sums, per (source rank, bag), the weighted rows of its shard
   (``pkm_segment_sum``: the bag kernel over ragged entry lists);
3. the partial sums go back with a second all-to-all, and each rank adds the
   partials of a bag in owner order.

backward: the upstream-gradient rows of the bags go to the owners (one
all-to-all), each owner runs the sorted-segment backward over the entries it
served (``pkm_bag_bwd_ragged``: gradient of its own rows, per-entry weight
gradients), and the per-entry weight gradients come back (one all-to-all).
The table gradient is local to its owner: nothing is all-reduced.

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


def _all_to_all(t: torch.Tensor, send_counts: List[int], recv_counts: List[int], group) -> torch.Tensor:
    """Uneven all-to-all along dim 0."""
    out = torch.empty((sum(recv_counts),) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_to_all_single(out, t.contiguous(), output_split_sizes=recv_counts, input_split_sizes=send_counts,
                           group=group)
    return out


class _RowShardedBag(torch.autograd.Function):
    @staticmethod
    def forward(ctx, indices, psw, shard, shard_rows, group):
        world = dist.get_world_size(group)
        B, L = indices.shape
        dev = shard.device
        flat = indices.reshape(-1)
        owner = torch.div(flat, shard_rows, rounding_mode="floor")
        if bool(((flat < 0) | (owner >= world)).any()):
            raise IndexError("row index outside the sharded table")
        order = torch.argsort(owner, stable=True)
        send_counts_t = torch.bincount(owner, minlength=world)
        recv_counts_t = torch.empty_like(send_counts_t)
        dist.all_to_all_single(recv_counts_t, send_counts_t, group=group)
        send_counts = send_counts_t.tolist()
        recv_counts = recv_counts_t.tolist()
        o_sorted = owner[order]
        local_row = (flat[order] - o_sorted * shard_rows).to(torch.int32)
        bag = torch.div(order, L, rounding_mode="floor").to(torch.int32)
        w = psw.reshape(-1)[order].to(torch.float32)
        r_row = _all_to_all(local_row, send_counts, recv_counts, group)
        r_w = _all_to_all(w, send_counts, recv_counts, group)
        r_bag = _all_to_all(bag, send_counts, recv_counts, group)
        # segments of the received entries: one per (source rank, bag), in
        # source order and, within a source, bag order
        r_src = torch.repeat_interleave(torch.arange(world, device=dev), torch.tensor(recv_counts, device=dev))
        key = r_src.to(torch.int64) * (1 << 32) + r_bag.to(torch.int64)
        n_recv = key.numel()
        starts = torch.ones(n_recv, dtype=torch.bool, device=dev)
        if n_recv > 1:
            starts[1:] = key[1:] != key[:-1]
        seg_start = torch.nonzero(starts).reshape(-1)
        offsets = torch.cat([seg_start, torch.tensor([n_recv], device=dev)])
        seg_of = torch.cumsum(starts.to(torch.int32), 0) - 1
        partial = _native.segment_sum(shard, r_row, r_w, offsets, out_dtype=shard.dtype)
        # partials back to their source ranks: per source, one row per bag it
        # sent here, in bag order
        seg_src = r_src[seg_start]
        back_send = torch.bincount(seg_src, minlength=world).tolist()
        # this rank's bags per owner, in the order the owner returns them
        s_starts = torch.ones(flat.numel(), dtype=torch.bool, device=dev)
        skey = o_sorted * (1 << 32) + bag.to(torch.int64)
        if flat.numel() > 1:
            s_starts[1:] = skey[1:] != skey[:-1]
        my_seg_bag = bag[s_starts].to(torch.int64)
        my_seg_owner = o_sorted[s_starts]
        back_recv = torch.bincount(my_seg_owner, minlength=world).tolist()
        got = _all_to_all(partial, back_send, back_recv, group)
        out = torch.zeros((B, shard.shape[1]), dtype=torch.float32, device=dev)
        pos = 0
        for o in range(world):  # owners in order: a fixed summation order
            n = back_recv[o]
            if n:
                out.index_add_(0, my_seg_bag[pos:pos + n], got[pos:pos + n].float())
            pos += n
        ctx.save_for_backward(order, r_row, r_w, seg_of, my_seg_bag, shard)
        ctx.counts = (send_counts, recv_counts, back_send, back_recv)
        ctx.group = group
        ctx.shape = (B, L)
        ctx.psw_dtype = psw.dtype
        return out.to(shard.dtype)

    @staticmethod
    def backward(ctx, d_out):
        order, r_row, r_w, seg_of, my_seg_bag, shard = ctx.saved_tensors
        send_counts, recv_counts, back_send, back_recv = ctx.counts
        group = ctx.group
        B, L = ctx.shape
        # the upstream rows of this rank's (owner, bag) segments go to the owners
        rows_out = d_out.to(shard.dtype).contiguous()[my_seg_bag]
        rows_in = _all_to_all(rows_out, back_recv, back_send, group)
        dW, dpsw_recv = _native.bag_bwd_ragged(r_row, seg_of, r_w, shard, rows_in,
                                               need_dpsw=ctx.needs_input_grad[1])
        d_psw = None
        if ctx.needs_input_grad[1]:
            back = _all_to_all(dpsw_recv, recv_counts, send_counts, group)
            d_flat = torch.empty(B * L, dtype=torch.float32, device=shard.device)
            d_flat[order] = back
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
