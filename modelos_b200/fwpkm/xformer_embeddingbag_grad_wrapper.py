"""Embedding bag with a differentiable weight gradient (double-backward).

Mirrors ``fwpkm/xformer_embeddingbag_grad_wrapper.py`` of the reference.  The
fast-weight memory differentiates the memorisation loss w.r.t. the value
table with ``create_graph=True`` and then back-propagates the outer loss
through that gradient, so the bag's weight gradient must itself be a
differentiable function of ``grad_output`` and ``per_sample_weights``:

* ``_XEmbeddingBagFn`` (``:83-155``): forward gather-sum (K3), first-order
  backward by ``bw_kernel`` (K4 by default), with the weight gradient wrapped
  in ``EmbeddingBagBW``;
* ``EmbeddingBagBW`` (``:13-74``): its backward is the vector-Jacobian
  product of that gradient, ``dG[b] = sum_j a[b,j] gbar[idx[b,j]]`` and
  ``da[b,j] = <gbar[idx[b,j]], g[b]>``, computed by K5 without
  materialising the ``[B, bag, D]`` gather.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
from torch.autograd import Function

from .. import _native
from .xformer_embeddingbag_legacy import embedding_bag_bw_rev_indices


class EmbeddingBagBW(Function):
    @staticmethod
    def forward(ctx, indices: torch.Tensor, per_sample_weights: Optional[torch.Tensor], grad_output: torch.Tensor,
                num_embeddings: int, embedding_dim: int, fast_grad_weight: torch.Tensor) -> torch.Tensor:
        ctx.has_psw = per_sample_weights is not None
        ctx.save_for_backward(indices, per_sample_weights if ctx.has_psw else None, grad_output)
        ctx.num_embeddings = num_embeddings
        ctx.embedding_dim = embedding_dim
        return fast_grad_weight

    @staticmethod
    def backward(ctx, g_bar: torch.Tensor):
        idx, a, g = ctx.saved_tensors
        gb = g_bar.contiguous()
        d_go, d_a = _native.bag_bwd2(idx, a, gb, g.contiguous(), d_grad_out_dtype=g.dtype,
                                     d_a_dtype=None if a is None else a.dtype)
        return None, d_a, d_go, None, None, None


class _XEmbeddingBagFn(Function):
    @staticmethod
    def forward(ctx, weight: torch.Tensor, indices: torch.Tensor, per_sample_weights: Optional[torch.Tensor],
                bw_kernel: Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor],
                                    Tuple[torch.Tensor, torch.Tensor]]) -> torch.Tensor:
        assert indices.dtype == torch.long
        K, D = weight.shape
        # output dtype follows torch promotion of rows * weights (:99-103)
        out_dtype = weight.dtype if per_sample_weights is None else torch.promote_types(
            weight.dtype, per_sample_weights.dtype)
        out = _native.bag_fwd(indices.contiguous(), weight.contiguous(),
                              None if per_sample_weights is None else per_sample_weights.contiguous(),
                              out_dtype=out_dtype)
        ctx.save_for_backward(weight, indices, per_sample_weights)
        ctx.has_psw = per_sample_weights is not None
        ctx.K, ctx.D = K, D
        ctx.bw_kernel = bw_kernel
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        weight, indices, a = ctx.saved_tensors
        weight_grad_fast, psw_grad_fast = ctx.bw_kernel(indices, weight, a, grad_output)
        grad_weight = EmbeddingBagBW.apply(indices, a if ctx.has_psw else None, grad_output, ctx.K, ctx.D,
                                           weight_grad_fast)
        grad_psw = psw_grad_fast if ctx.has_psw else None
        return grad_weight, None, grad_psw, None


def xformers_embedding_bag(indices: torch.Tensor, weight: torch.Tensor,
                           per_sample_weights: torch.Tensor) -> torch.Tensor:
    return _XEmbeddingBagFn.apply(weight, indices, per_sample_weights, embedding_bag_bw_rev_indices)
