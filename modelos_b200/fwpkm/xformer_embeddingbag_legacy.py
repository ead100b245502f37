"""First-order embedding-bag kernels used by the fast-weight memory.

Mirrors ``fwpkm/xformer_embeddingbag_legacy.py`` of the reference (its own
copy of the bag forward and of the reverse-index backward,
``:33-74, 170-227``) on the sm_100a kernels: ``embedding_bag_bw_rev_indices``
is the ``bw_kernel`` that ``_XEmbeddingBagFn`` calls.  CUDA tensors only.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import _native


def embedding_bag_b200(indices: torch.Tensor, weight: torch.Tensor,
                       per_sample_weights: Optional[torch.Tensor]) -> torch.Tensor:
    """``out[b] = sum_j psw[b,j] * weight[indices[b,j]]`` in the weight's dtype."""
    return _native.bag_fwd(indices.contiguous(), weight.contiguous(),
                           None if per_sample_weights is None else per_sample_weights.contiguous())


embedding_bag_triton = embedding_bag_b200


def embedding_bag_bw_rev_indices(indices: torch.Tensor, weight: torch.Tensor,
                                 per_sample_weights: Optional[torch.Tensor],
                                 gradient: torch.Tensor) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """``(weight.grad, per_sample_weights.grad)`` of the weighted bag
    (``fwpkm/xformer_embeddingbag_legacy.py:170-227``): dense weight gradient
    in the weight's dtype, per-sample gradient in its own dtype (``None``
    when there are no per-sample weights)."""
    g = gradient.contiguous()
    if g.dtype != weight.dtype:
        g = g.to(weight.dtype)
    psw = None if per_sample_weights is None else per_sample_weights.contiguous()
    dW, dpsw, _ = _native.bag_bwd(indices.contiguous(), weight.contiguous(), psw, g,
                                  need_dpsw=psw is not None)
    return dW, dpsw


class xFormersEmbeddingBag(torch.autograd.Function):
    """``fwpkm/xformer_embeddingbag_legacy.py:230-253``."""

    @staticmethod
    def forward(ctx, indices, weight, per_sample_weights):
        ctx.save_for_backward(indices, weight, per_sample_weights)
        return embedding_bag_b200(indices, weight, per_sample_weights)

    @staticmethod
    def backward(ctx, gradient):
        indices, weight, per_sample_weights = ctx.saved_tensors
        weight_g, per_sample_weights_g = embedding_bag_bw_rev_indices(indices, weight, per_sample_weights,
                                                                      gradient)
        return None, weight_g, per_sample_weights_g


def xformers_embedding_bag(indices: torch.Tensor, weight: torch.Tensor, per_sample_weights: torch.Tensor,
                           mode: str = "sum") -> torch.Tensor:
    assert mode == "sum"
    return xFormersEmbeddingBag.apply(indices, weight, per_sample_weights)
