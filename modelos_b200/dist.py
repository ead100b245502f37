"""Data-parallel gradient reduction for the PKM layers.

Tokens are independent in the memory lookup, so the layer shards over the
batch: every rank holds the full (replicated) value table and runs its own
tokens, and the gradients are summed across ranks.  The value table's
gradient is the large one (``[n_keys^2, v_dim]``, 512 MiB in bf16 at
BASELINE config 2) and is produced in the middle of the backward, by the bag
backward; ``GradReducer`` starts its all-reduce as soon as it is accumulated,
so the transfer overlaps the rest of the backward (scoring and query
projection), and reduces the small dense gradients together in one flattened
bucket at the end.  BatchNorm statistics stay per rank, as the reference's
``nn.BatchNorm1d`` does under data parallelism.
"""
from __future__ import annotations

from typing import Iterable, List, Optional

import torch
import torch.distributed as dist


class GradReducer:
    """Sum gradients of ``params`` over ``group`` (``average`` divides by the
    world size).  ``early`` names the parameters whose all-reduce starts from
    a post-accumulate-grad hook; the rest are flattened into one bucket by
    ``finish()``, which also waits for the early reductions."""

    def __init__(self, params: Iterable[torch.nn.Parameter], early: Iterable[torch.nn.Parameter] = (),
                 group: Optional[dist.ProcessGroup] = None, average: bool = False):
        self.group = group
        self.average = average
        early = list(early)
        early_ids = {id(p) for p in early}
        self.rest: List[torch.nn.Parameter] = [p for p in params if id(p) not in early_ids and p.requires_grad]
        self.pending = []
        self.handles = []
        for p in early:
            self.handles.append(p.register_post_accumulate_grad_hook(self._start))

    def world(self) -> int:
        return dist.get_world_size(self.group)

    def _start(self, p: torch.Tensor):
        if p.grad is None:
            return
        self.pending.append((p.grad, dist.all_reduce(p.grad, group=self.group, async_op=True)))

    def finish(self):
        """Reduce the remaining gradients and wait for everything."""
        grads = [p.grad for p in self.rest if p.grad is not None]
        if grads:
            flat = torch.cat([g.reshape(-1).to(torch.float32) for g in grads])
            dist.all_reduce(flat, group=self.group)
            if self.average:
                flat /= self.world()
            off = 0
            for g in grads:
                n = g.numel()
                g.copy_(flat[off:off + n].view_as(g))
                off += n
        for g, work in self.pending:
            work.wait()
            if self.average:
                g /= self.world()
        self.pending = []

    def remove(self):
        for h in self.handles:
            h.remove()
        self.handles = []
