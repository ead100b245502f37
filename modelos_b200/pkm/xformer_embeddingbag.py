"""Weighted embedding bag on B200 kernels, with the reference's API.

Mirrors ``pkm/xformer_embeddingbag.py`` of the reference: the same function
and autograd-class names and signatures, backed by the sm_100a kernels of
``libpkm_b200.so`` instead of the Triton kernels:

* ``embedding_bag_triton`` (forward, ``:116-138``) -> K3 ``pkm_bag_fwd``
* ``embedding_bag_bw_rev_indices`` (``:331-386``) -> K4 ``pkm_bag_bwd``, a
  deterministic sorted-segment backward (the reference orders occurrences
  with atomics, ``:277-288``, so its sum order varies between runs)
* ``xFormersEmbeddingBag`` / ``xformers_embedding_bag`` (``:389-438``)

Unlike the reference there is no CPU branch (``:436-437``): CPU tensors raise.
"""
from __future__ import annotations

from typing import Tuple

import torch

from .. import _native


def embedding_bag_b200(indices: torch.Tensor, weight: torch.Tensor,
                       per_sample_weights: torch.Tensor) -> torch.Tensor:
    """``out[b] = sum_j psw[b,j] * weight[indices[b,j]]`` in the weight's dtype
    (``embedding_bag_triton``, ``pkm/xformer_embeddingbag.py:116-138``)."""
    return _native.bag_fwd(indices.contiguous(), weight.contiguous(),
                           None if per_sample_weights is None else per_sample_weights.contiguous())


# the reference's launcher name, kept for callers that import it
embedding_bag_triton = embedding_bag_b200


def embedding_bag_bw_rev_indices(indices: torch.Tensor, weight: torch.Tensor,
                                 per_sample_weights: torch.Tensor,
                                 gradient: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Returns ``(weight.grad, per_sample_weights.grad)``
    (``pkm/xformer_embeddingbag.py:331-386``): a dense weight gradient in the
    weight's dtype (zero rows where no index points) and the per-sample
    gradient in its own dtype."""
    assert indices.is_contiguous()
    assert weight.is_contiguous()
    assert per_sample_weights.is_contiguous()
    assert gradient.is_contiguous()
    B, bag = indices.shape
    assert per_sample_weights.shape == (B, bag)
    assert gradient.shape == (B, weight.shape[1])
    g = gradient if gradient.dtype == weight.dtype else gradient.to(weight.dtype)
    dW, dpsw, _ = _native.bag_bwd(indices, weight, per_sample_weights, g)
    return dW, dpsw


class xFormersEmbeddingBag(torch.autograd.Function):
    """Autograd node of the bag (``pkm/xformer_embeddingbag.py:389-425``)."""

    @staticmethod
    def forward(ctx, indices, weight, per_sample_weights, bw_algo):
        ctx.save_for_backward(indices, weight, per_sample_weights)
        ctx.bw_algo = bw_algo
        # data-parallel training may attach a fused gradient exchange to the
        # table (modelos_b200.dist.ShardedTableGrad)
        ctx.exchange = getattr(weight, "_pkm_grad_exchange", None)
        return embedding_bag_b200(indices, weight, per_sample_weights)

    @staticmethod
    def backward(ctx, gradient):
        indices, weight, per_sample_weights = ctx.saved_tensors
        # every bw_algo of the reference ("reverse_indices", "atomics", "lock")
        # computes the same gradients; all map to the sorted-segment kernel
        assert ctx.bw_algo in ("reverse_indices", "atomics", "lock")
        if ctx.exchange is not None and ctx.needs_input_grad[1]:
            g = gradient.contiguous().to(weight.dtype)
            weight_g, per_sample_weights_g = ctx.exchange.backward(
                indices, weight, per_sample_weights, g, need_dpsw=ctx.needs_input_grad[2])
            return None, weight_g, per_sample_weights_g, None
        weight_g, per_sample_weights_g = embedding_bag_bw_rev_indices(
            indices, weight, per_sample_weights, gradient.contiguous())
        return None, weight_g, per_sample_weights_g, None


def xformers_embedding_bag(indices: torch.Tensor, weight: torch.Tensor, per_sample_weights: torch.Tensor,
                           mode: str = "sum", bw_algo: str = "reverse_indices") -> torch.Tensor:
    """``pkm/xformer_embeddingbag.py:428-438`` on the B200 kernels."""
    assert mode == "sum"
    if not indices.is_cuda:
        raise RuntimeError("modelos_b200.xformers_embedding_bag needs CUDA tensors (no CPU path)")
    return xFormersEmbeddingBag.apply(indices, weight, per_sample_weights, bw_algo)
