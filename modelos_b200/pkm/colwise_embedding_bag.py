"""``xFormerEmbeddingBag`` module (``pkm/colwise_embedding_bag.py:28-49``).

The value table of ``HashingMemory``: one ``weight`` parameter ``[size, dim]``
read through the B200 bag kernels.  For a DTensor weight the local shard is
used and its gradient is scaled by ``1/num_shards`` exactly as the reference
does (``:38-44``).  The reference's ``ColwiseEmbeddingBag`` tensor-parallel
style (``:52-114``) is never applied in the reference and is not provided.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .xformer_embeddingbag import xformers_embedding_bag


class xFormerEmbeddingBag(nn.Module):
    def __init__(self, size, dim):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(size, dim))

    def __repr__(self):
        return f"xFormerEmbeddingBag(num_embeddings={self.weight.size(0)}, embedding_dim={self.weight.size(1)})"

    @torch.compiler.disable(recursive=True)
    def forward(self, indices, scores):
        weight = self.weight
        try:
            from torch.distributed.tensor import DTensor
        except Exception:  # pragma: no cover - torch without distributed
            DTensor = ()
        if DTensor and isinstance(weight, DTensor):
            num_shards = weight.device_mesh.size()
            weight = weight.to_local()
            if num_shards > 1:
                grad_scale = 1 / num_shards
                weight = weight * grad_scale + (weight * (1 - grad_scale)).detach()
        return xformers_embedding_bag(indices, weight, per_sample_weights=scores, mode="sum")
