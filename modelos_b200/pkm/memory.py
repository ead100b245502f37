"""Product-key memory layer on B200 kernels (``pkm/memory.py`` of the reference).

``HashingMemory`` keeps the reference's constructor arguments, parameter
names and shapes, ``reset_parameters``, ``forward`` and ``get_indices``
(``pkm/memory.py:37-289``), so a state dict moves between the two and
``modeling_qwen3pkm.py`` can import this class unchanged.  The memory lookup
runs on the sm_100a kernels:

* sub-key scores of both halves (K1, ``pkm_subkey_scores``),
* dual top-k, cartesian top-k and per-head softmax fused in one warp per
  (token, head) (K2, ``pkm_product_topk``),
* the weighted bag over the value table (K3/K4 via ``xFormerEmbeddingBag``),
* and, in the backward, the softmax gradient scattered onto the dense
  sub-score grid (``pkm_score_grad_dense``) followed by two batched GEMMs
  over the (head, half) groups for the query and key gradients.

The query projection, the SwiLU projection and the value projection keep
their ``nn.Linear`` modules (same parameters) and run, with their data and
weight gradients, on the library's tensor-core GEMM in bf16
(``pkm_gemm_bf16``: either operand K-major or MN-major, so no gradient
transposes a tensor); the SwiGLU gate between them and the bias gradients
run on the library's kernels (``SwiGLUProjection``), and the query batch
norm keeps ``nn.BatchNorm1d``'s parameters and buffers and runs on the
library's batch-normalisation kernels (``QueryBatchNorm``).  The scoring
backward's two GEMMs per (head, half) are one batched call each.  fp32
layers (the CPU-runnable parity configuration) use torch's fp32 GEMMs for
these dense products.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from logging import getLogger
from typing import Optional

import torch
from torch import nn
from torch.nn import functional as F

from .. import _native
from .colwise_embedding_bag import xFormerEmbeddingBag

logger = getLogger()


@dataclass
class ProductKeyArgs:
    """Configuration record of the reference (``pkm/memory.py:15-28``)."""

    is_enabled: bool = False
    layers: str = ""
    mem_n_keys: int = 1024
    mem_heads: int = 4
    mem_knn: int = 32
    mem_share_values: bool = True
    mem_k_dim: int = 512
    mem_v_dim: int = -1
    swilu_projection: bool = True
    value_fixed_lr: Optional[float] = 0.001
    mem_gated: bool = False
    peer_variant: bool = False


class AttrDict(dict):
    def __init__(self, *args, **kwargs):
        super(AttrDict, self).__init__(*args, **kwargs)
        self.__dict__ = self


# ---------------------------------------------------------------------------
# autograd nodes of the lookup
# ---------------------------------------------------------------------------
def subkey_scores(query: torch.Tensor, keys: torch.Tensor, heads: int) -> torch.Tensor:
    """All sub-key dot scores ``[N*H, 2, n]`` (``pkm/memory.py:267-268``).

    fp32 uses the sequential-sum kernel, whose scores (and therefore top-k
    indices) are bit-identical to the oracle's definition; bf16 runs the
    contraction on the tcgen05 tensor cores (fp32 accumulation, bf16 output,
    as the reference's einsum)."""
    return _native.subkey_scores(query, keys, heads, "dot")


def _score_backward(ctx, d_scores, psw):
    """Gradients of the product-key scores w.r.t. query and keys.

    The score of slot ``i1*n + i2`` is ``s1[i1] + s2[i2]``
    (``pkm/memory.py:274-281``): the kernel scatters the (softmax-)gradient
    onto the dense sub-score grid ``[N*H, 2, n]``, then two GEMMs per
    (head, half) give ``dq = dS @ keys`` and ``dkeys = dS^T @ q``, the same
    contraction the reference's einsum backward performs.
    """
    query, keys, idx = ctx.saved_tensors[:3]
    R, kd = query.shape
    half = kd // 2
    H, n = ctx.heads, ctx.n_keys
    N = R // H
    dS = _native.score_grad_dense(idx, psw, d_scores.to(query.dtype), n).view(N, H * 2, n)
    dq = dk = None
    G = H * 2
    if _tc(query, keys) and half % 8 == 0 and n % 8 == 0 and (n % 64 == 0 or G == 1):
        # batched GEMMs over the H*2 (head, half) groups on the tensor cores,
        # each group's operands addressed by coordinate offsets (no copies)
        dS2 = dS.view(N, G * n)
        if ctx.needs_input_grad[0]:
            dq = torch.empty((N, G * half), dtype=query.dtype, device=query.device)
            _native.gemm(dS2, keys.view(G * n, half), b_mn=True, batch=G, M=N, N=half, K=n, a_batch=(n, 0),
                         b_batch=(0, n), out=dq, c_batch_stride=half)
            dq = dq.view(R, kd)
        if ctx.needs_input_grad[1]:
            dk = torch.empty((G * n, half), dtype=keys.dtype, device=keys.device)
            _native.gemm(dS2, query.view(N, G * half), a_mn=True, b_mn=True, batch=G, M=n, N=half, K=N,
                         a_batch=(n, 0), b_batch=(half, 0), out=dk, c_batch_stride=n * half)
            dk = dk.view(keys.shape)
        return dq, dk
    if ctx.needs_input_grad[0]:
        # one strided batched GEMM over the H*2 (head, half) blocks, written
        # straight into the token-major [N, H, 2, half] layout of the query
        dq = torch.empty((N, H * 2, half), dtype=query.dtype, device=query.device)
        torch.bmm(dS.transpose(0, 1), keys.view(H * 2, n, half), out=dq.transpose(0, 1))
        dq = dq.view(R, kd)
    if ctx.needs_input_grad[1]:
        dk = torch.bmm(dS.permute(1, 2, 0), query.view(N, H * 2, half).transpose(0, 1)).reshape(keys.shape)
    return dq, dk


class ProductKeyTopK(torch.autograd.Function):
    """``(scores, indices)`` of ``HashingMemory.get_indices`` (``pkm/memory.py:250-289``)."""

    @staticmethod
    def forward(ctx, query, keys, heads, knn):
        scores_all = subkey_scores(query, keys, heads)
        n_keys = scores_all.shape[-1]
        idx, top, _, _, _ = _native.product_topk(scores_all, knn)
        ctx.save_for_backward(query, keys, idx)
        ctx.heads, ctx.n_keys = heads, n_keys
        ctx.mark_non_differentiable(idx)
        return top, idx

    @staticmethod
    def backward(ctx, d_top, d_idx):
        if d_top is None:
            return None, None, None, None
        dq, dk = _score_backward(ctx, d_top.contiguous(), None)
        return dq, dk, None, None


class ProductKeyLookup(torch.autograd.Function):
    """Fused lookup of ``HashingMemory.forward`` (``pkm/memory.py:204-222``):
    returns per-head softmax weights (differentiable), indices and the raw
    top-k scores (not differentiable, kept for ``last_scores``)."""

    @staticmethod
    def forward(ctx, query, keys, heads, knn):
        scores_all = subkey_scores(query, keys, heads)
        n_keys = scores_all.shape[-1]
        idx, top, psw, _, _ = _native.product_topk(scores_all, knn, want_psw=True)
        ctx.save_for_backward(query, keys, idx, psw)
        ctx.heads, ctx.n_keys = heads, n_keys
        ctx.mark_non_differentiable(idx, top)
        return psw, idx, top

    @staticmethod
    def backward(ctx, d_psw, d_idx, d_top):
        if d_psw is None:
            return None, None, None, None
        psw = ctx.saved_tensors[3]
        dq, dk = _score_backward(ctx, d_psw.contiguous(), psw)
        return dq, dk, None, None


# ---------------------------------------------------------------------------
# dense projections: bf16 on the library's tensor-core GEMM (pkm_gemm_bf16),
# other dtypes (the fp32 parity configuration) on torch's GEMMs
# ---------------------------------------------------------------------------
def _tc(*ts) -> bool:
    return all(t.dtype == torch.bfloat16 and t.is_cuda for t in ts)


def linear(x, w, b=None):
    """``x @ w.T + b`` (``F.linear``)."""
    if _tc(x, w) and w.shape[0] % 8 == 0:
        return _native.gemm(x.contiguous(), w.contiguous(), bias=b)
    return F.linear(x, w, b)


def matmul_nn(dy, w):
    """``dy @ w`` (the data gradient of ``linear``)."""
    if _tc(dy, w) and w.shape[1] % 8 == 0:
        return _native.gemm(dy.contiguous(), w.contiguous(), b_mn=True)
    return dy.mm(w)


def matmul_tn(dy, x, out_dtype=None):
    """``dy.T @ x`` (the weight gradient of ``linear``)."""
    if _tc(dy, x) and x.shape[1] % 8 == 0:
        return _native.gemm(dy.contiguous(), x.contiguous(), a_mn=True, b_mn=True, out_dtype=out_dtype or x.dtype)
    return dy.t().mm(x)


class LinearColsumBias(torch.autograd.Function):
    """``F.linear(x, w, b)`` on the library's GEMM (bf16), with the bias
    gradient reduced by the library's column-sum kernel."""

    @staticmethod
    def forward(ctx, x, w, b):
        ctx.save_for_backward(x, w)
        ctx.b_dtype = None if b is None else b.dtype
        return linear(x, w, b)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = matmul_nn(dy, w) if ctx.needs_input_grad[0] else None
        dw = matmul_tn(dy, x, w.dtype) if ctx.needs_input_grad[1] else None
        db = _native.colsum(dy, ctx.b_dtype) if ctx.b_dtype is not None and ctx.needs_input_grad[2] else None
        return dx, dw, db


class SwiGLUProjection(torch.autograd.Function):
    """``value_proj(a * silu(swilu_projection(x)))`` of ``HashingMemory.forward``
    (``pkm/memory.py:226-229``): both projections and their gradients on the
    library's GEMM (bf16); the gate as one pass each way (``pkm_swiglu_fwd``,
    ``pkm_swiglu_bwd``, the latter with the gate projection's bias gradient).

    With ``FUSE_GATE`` the gate rides in the GEMM epilogues instead (forward:
    h and z from the gate projection's GEMM; backward: da and dh from the
    value projection's data-gradient GEMM), with the same bits.  It is off by
    default: the gate's exact exp and divisions on the epilogue's eight warps
    per SM take longer than the tile's MMAs, and the HashingMemory step at
    config 2 measured 2.88 ms fused against 2.71 ms with the gate pass."""

    # whether the gate rides in the GEMM epilogues (else GEMM, then the gate
    # kernel; the two give the same bits)
    FUSE_GATE = False

    @staticmethod
    def _fused(a, x, ws, wv):
        # the gate rides in the GEMM epilogues (bf16, N a multiple of 8)
        return (SwiGLUProjection.FUSE_GATE and _tc(a, x, ws, wv) and ws.shape[0] % 8 == 0
                and a.shape == (x.shape[0], ws.shape[0]))

    @staticmethod
    def forward(ctx, a, x, ws, bs, wv, bv):
        if SwiGLUProjection._fused(a, x, ws, wv):
            h, z = _native.gemm_swiglu_fwd(x, ws, bs, a)
        else:
            h = linear(x, ws, bs)
            z = _native.swiglu_fwd(a, h)
        ctx.save_for_backward(a, x, h, z, ws, wv)
        ctx.bias_dtypes = (None if bs is None else bs.dtype, None if bv is None else bv.dtype)
        return linear(z, wv, bv)

    @staticmethod
    def backward(ctx, dy):
        a, x, h, z, ws, wv = ctx.saved_tensors
        need_a, need_x, need_ws, need_bs, need_wv, need_bv = ctx.needs_input_grad
        dy = dy.contiguous()
        dbv = _native.colsum(dy, ctx.bias_dtypes[1]) if need_bv else None
        dwv = matmul_tn(dy, z, wv.dtype) if need_wv else None
        if SwiGLUProjection._fused(a, x, ws, wv):
            da, dh = _native.gemm_swiglu_bwd(dy, wv, a, h, need_da=need_a)
            dbs = _native.colsum(dh, ctx.bias_dtypes[0]) if need_bs and ctx.bias_dtypes[0] is not None else None
        else:
            dz = matmul_nn(dy, wv)
            da, dh, dbs = _native.swiglu_bwd(dz, a, h, need_da=need_a,
                                             bias_dtype=ctx.bias_dtypes[0] if need_bs else None)
        dws = matmul_tn(dh, x, ws.dtype) if need_ws else None
        dx = matmul_nn(dh, ws) if need_x else None
        return da, dx, dws, dbs, dwv, dbv


# ---------------------------------------------------------------------------
# the layer
# ---------------------------------------------------------------------------
class HashingMemory(nn.Module):
    VALUES = None
    EVAL_MEMORY = True

    def __init__(
        self,
        input_dim,
        output_dim,
        value_fixed_lr=0.001,
        mem_k_dim=512,
        mem_v_dim=-1,
        mem_heads=4,
        mem_knn=32,
        mem_share_values=True,
        mem_n_keys=1024,
        mem_query_bias=True,
        mem_query_batchnorm=False,
        mem_query_rmsnorm=True,
        mem_gated=False,
        mem_input_dropout=0.0,
        mem_query_dropout=0.0,
        mem_value_dropout=0.0,
        peer_variant=False,
        swilu_projection=True,
    ):
        assert mem_k_dim >= 2
        assert 0 <= mem_input_dropout < 1
        assert 0 <= mem_query_dropout < 1
        assert 0 <= mem_value_dropout < 1
        assert not (peer_variant and mem_v_dim > 0), (
            "Cannot use PEER variant with a value dimension different from the input dimension (mem_v_dim=-1)"
        )
        assert mem_k_dim % 2 == 0
        assert mem_heads >= 2
        if peer_variant:
            raise NotImplementedError("the PEER variant is not part of the B200 product-key path")
        if mem_query_batchnorm:
            logger.warning(
                "WARNING: if you use batch normalization, be sure that you use batches of sentences with the same "
                "size at training time. Otherwise, the padding token will result in incorrect mean/variance "
                "estimations in the BatchNorm layer."
            )
        assert not (mem_query_batchnorm and mem_query_rmsnorm), "Cannot use both batchnorm and rmsnorm"

        super().__init__()
        self.use_peer_variant = peer_variant
        self.input_dim = input_dim
        self.output_dim = output_dim
        self.size = mem_n_keys**2
        self.k_dim = mem_k_dim
        self.v_dim = mem_v_dim if mem_v_dim > 0 else output_dim
        self.swilu_proj = swilu_projection
        self.v_proj = mem_v_dim > 0 or self.swilu_proj
        self.heads = mem_heads
        self.knn = mem_knn
        self.n_keys = mem_n_keys
        self.input_dropout = mem_input_dropout
        self.query_dropout = mem_query_dropout
        self.value_dropout = mem_value_dropout

        self.keys = nn.Parameter(torch.zeros(2 * self.heads * int(self.size**0.5), self.k_dim // 2))
        self.mem_share_values = mem_share_values
        self.original = not self.mem_share_values or HashingMemory.VALUES is None
        if self.original:
            self.values = xFormerEmbeddingBag(self.size, self.v_dim)
        else:
            self.values = None
        self.value_fixed_lr = value_fixed_lr

        if self.v_proj:
            proj_input = mem_v_dim
            if self.swilu_proj and proj_input < 0:
                proj_input = output_dim
            self.value_proj = torch.nn.Linear(proj_input, output_dim)
        if self.swilu_proj:
            self.swilu_projection = torch.nn.Linear(self.input_dim, proj_input)
        self.gating = None
        if mem_gated:
            self.gating = torch.nn.Linear(input_dim, 1)

        l_sizes = (self.input_dim, self.heads * self.k_dim)
        self.query_proj = QueryMLP(
            self.input_dim,
            self.heads,
            self.k_dim,
            l_sizes,
            bias=mem_query_bias,
            batchnorm=mem_query_batchnorm,
            rmsnorm=mem_query_rmsnorm,
        )
        self._last_indices_dev = None
        self._last_scores_dev = None

    # eval-mode usage statistics (pkm/memory.py:213-215); the host copy is
    # made when the attribute is read instead of on every forward
    @property
    def last_indices(self):
        t = self._last_indices_dev
        return None if t is None else t.cpu()

    @last_indices.setter
    def last_indices(self, v):
        self._last_indices_dev = v

    @property
    def last_scores(self):
        t = self._last_scores_dev
        return None if t is None else t.cpu().float()

    @last_scores.setter
    def last_scores(self, v):
        self._last_scores_dev = v

    def reset_parameters(self, init_std=None, factor=1.0):
        bound = 1 / math.sqrt(self.k_dim)
        nn.init.uniform_(self.keys, a=-bound, b=bound)
        if self.original:
            nn.init.normal_(self.values.weight, mean=0, std=self.v_dim**-0.5)
        nn.init.xavier_uniform_(self.query_proj.query_mlps[0].weight)
        if self.v_proj:
            nn.init.normal_(self.value_proj.weight, mean=0, std=self.output_dim**-0.5)
        if self.swilu_proj:
            nn.init.normal_(self.swilu_projection.weight, mean=0, std=self.output_dim**-0.5)
        if self.gating is not None:
            nn.init.normal_(self.gating.weight, mean=0, std=self.input_dim**-0.5)

    def forward(self, input):
        """Read from the memory: ``(out [B,T,output_dim], indices [B,T,H*knn])``."""
        B, T, C = input.shape
        input = input.view(-1, self.input_dim)
        assert input.shape[-1] == self.input_dim
        bs = input.shape[0]
        input = F.dropout(input, p=self.input_dropout, training=self.training)
        query = self.query_proj(input)
        query = F.dropout(query, p=self.query_dropout, training=self.training)
        assert query.shape == (bs * self.heads, self.k_dim)

        knn = self.knn
        psw, indices, scores = ProductKeyLookup.apply(query.contiguous(), self.keys, self.heads, knn)
        if not self.training and HashingMemory.EVAL_MEMORY:
            self.last_indices = indices.view(bs, self.heads, knn).detach()
            self.last_scores = scores.view(bs, self.heads, knn).detach()

        indices = indices.view(bs, self.heads * knn)
        psw = psw.view(bs, self.heads * knn)
        output = self.values(indices, psw)
        if self.v_proj and not self.swilu_proj:
            output = self.value_proj(output)
        if self.swilu_proj:
            output = SwiGLUProjection.apply(output, input, self.swilu_projection.weight, self.swilu_projection.bias,
                                            self.value_proj.weight, self.value_proj.bias)
        output = F.dropout(output, p=self.value_dropout, training=self.training)
        if self.gating:
            output = F.sigmoid(self.gating(input)) * output
        output = output.view(B, T, -1)
        indices = indices.view(B, T, -1)
        return output, indices

    def get_indices(self, query, knn):
        """``(scores [bs*H, knn], indices [bs*H, knn])`` (``pkm/memory.py:250-289``)."""
        assert query.dim() == 2 and query.size(1) == self.k_dim
        bs = len(query) // self.heads
        scores, indices = ProductKeyTopK.apply(query.contiguous(), self.keys, self.heads, knn)
        assert scores.shape == indices.shape == (bs * self.heads, knn)
        return scores, indices


class _QueryBatchNormFn(torch.autograd.Function):
    """Training/evaluation batch normalisation of a [n, c] tensor on the
    library's kernels (``F.batch_norm`` semantics)."""

    @staticmethod
    def forward(ctx, x, weight, bias, running_mean, running_var, training, momentum, eps):
        out, mean, rstd = _native.batchnorm_fwd(x, weight, bias, running_mean, running_var, training, momentum, eps)
        ctx.training = training
        ctx.save_for_backward(x, weight, mean, rstd)
        ctx.param_dtype = weight.dtype if weight is not None else (bias.dtype if bias is not None else x.dtype)
        return out

    @staticmethod
    def backward(ctx, d_out):
        x, weight, mean, rstd = ctx.saved_tensors
        if not ctx.training:
            # evaluation: an affine map of x with the running statistics
            scale = rstd * (weight.float() if weight is not None else 1.0)
            dx = (d_out.float() * scale).to(x.dtype) if ctx.needs_input_grad[0] else None
            dw = (d_out.float() * (x.float() - mean) * rstd).sum(0).to(ctx.param_dtype) \
                if ctx.needs_input_grad[1] else None
            db = d_out.float().sum(0).to(ctx.param_dtype) if ctx.needs_input_grad[2] else None
            return dx, dw, db, None, None, None, None, None
        dx, dw, db = _native.batchnorm_bwd(d_out, x, mean, rstd, weight, need_dx=ctx.needs_input_grad[0],
                                           need_dw=ctx.needs_input_grad[1], need_db=ctx.needs_input_grad[2],
                                           param_dtype=ctx.param_dtype)
        return dx, dw, db, None, None, None, None, None


class QueryBatchNorm(nn.BatchNorm1d):
    """``nn.BatchNorm1d`` of the query network (``pkm/memory.py:308-309``)
    with the same parameters, buffers and running-statistics rule
    (``torch.nn.modules.batchnorm._BatchNorm.forward``), computed by the
    library's batch-normalisation kernels.  Inputs are [n, c] CUDA tensors."""

    def forward(self, input):
        self._check_input_dim(input)
        if not input.is_cuda:
            raise RuntimeError("modelos_b200 QueryBatchNorm needs CUDA tensors (no CPU path)")
        if input.dim() != 2:
            raise NotImplementedError("QueryBatchNorm takes [n, c] inputs")
        factor = 0.0 if self.momentum is None else self.momentum
        if self.training and self.track_running_stats and self.num_batches_tracked is not None:
            self.num_batches_tracked.add_(1)
            factor = 1.0 / float(self.num_batches_tracked) if self.momentum is None else self.momentum
        bn_training = self.training or (self.running_mean is None and self.running_var is None)
        use_running = not self.training or self.track_running_stats
        return _QueryBatchNormFn.apply(input.contiguous(), self.weight, self.bias,
                                       self.running_mean if use_running else None,
                                       self.running_var if use_running else None, bn_training, factor, self.eps)


class QueryMLP(nn.Module):
    """Query network (``pkm/memory.py:292-349``)."""

    def __init__(self, input_dim, heads, k_dim, sizes, bias=False, batchnorm=False, rmsnorm=False):
        super().__init__()
        self.input_dim = input_dim
        self.heads = heads
        self.k_dim = k_dim
        self.sizes = sizes
        assert sizes[0] == input_dim
        assert sizes[-1] == (heads * k_dim)
        sizes_ = list(sizes)
        self.query_mlps = QueryMLP.mlp(sizes_, bias=bias)
        if batchnorm:
            self.norm = QueryBatchNorm(sizes_[-1], affine=True, eps=1e-6, momentum=0.1)
        elif rmsnorm:
            from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm

            self.norm = Qwen3RMSNorm(sizes_[-1], eps=1e-6)
        else:
            self.norm = None

    @staticmethod
    def mlp(sizes, bias=True):
        assert len(sizes) >= 2
        pairs = [(sizes[i], sizes[i + 1]) for i in range(len(sizes) - 1)]
        layers = []
        for i, (dim_in, dim_out) in enumerate(pairs):
            layers.append(nn.Linear(dim_in, dim_out, bias=bias))
            if i < len(pairs) - 1:
                layers.append(nn.ReLU())
        return nn.Sequential(*layers)

    def forward(self, input):
        assert input.shape[-1] == self.input_dim
        input = input.contiguous().view(-1, self.input_dim) if input.dim() > 2 else input
        bs = len(input)
        mlp = self.query_mlps
        if len(mlp) == 1 and isinstance(mlp[0], nn.Linear):
            # single projection: the library's GEMM, bias gradient by column sum
            query = LinearColsumBias.apply(input, mlp[0].weight, mlp[0].bias)
        else:
            query = mlp(input)
        if self.norm is not None:
            query = self.norm(query)
        assert query.shape == (bs, self.heads * self.k_dim)
        return query.view(bs * self.heads, self.k_dim)
