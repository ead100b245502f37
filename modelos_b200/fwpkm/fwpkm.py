"""Fast-weight product-key memory on B200 kernels (``fwpkm/fwpkm.py`` of the reference).

``FastWeightProductKeyMemory`` keeps the reference's constructor arguments,
parameters (``keys``, ``values``), ``forward`` signature and returned dict,
so ``modeling_qwen3pkm.py`` imports it unchanged (``modeling_qwen3pkm.py:23``).
Per chunk of the sequence it reads the memory with the current fast weights,
scores the read against a target (MSE memorisation loss plus the
marginal-entropy addressing loss), differentiates with
``create_graph=True`` and takes one SGD step on the fast weights, so the outer
loss back-propagates through every update (``forward_wo_past``, ``:395-558``).

Kernel mapping:

* sub-key scores, dot or idw (K1, ``pkm_subkey_scores``; idw is built from
  the distance mode), bit-exact in fp32; their backward's grouped products
  run on the library's fp32 GEMM (``pkm_gemm_f32``) inside an autograd node
  that is differentiable once more (second derivatives for the inner
  updates), reading the same saved tensors as the reference's autograd;
* the score transform (joint softmax over H*knn, ``pkm_score_transform``);
* dual / cartesian top-k (K2, ``pkm_product_topk``), ties to the lowest index;
* the bag forward, its sorted-segment backward and the double-backward
  (K3 / K4 / K5, through ``xformer_embeddingbag_grad_wrapper``).
"""
from __future__ import annotations

import math
from collections import OrderedDict, defaultdict
from logging import getLogger

import torch
from torch import nn
from torch.nn import functional as F

from .. import _native
from .xformer_embeddingbag_grad_wrapper import xformers_embedding_bag

logger = getLogger()


def l2norm(x: torch.FloatTensor, dim: int = -1, eps: float = 1e-6):
    """``x / sqrt(sum(x^2) + eps)`` (``fwpkm/fwpkm.py:16-19``)."""
    inv_norm = torch.rsqrt((x * x).sum(dim=dim, keepdim=True) + eps)
    return x * inv_norm


def _group_mm(dS, q, k, H, want_dq=True, want_dk=True):
    """Per (head, half) group g: ``dS_g @ K_g`` and ``dS_g^T @ Q_g``, for
    sub-key scores ``S_g = Q_g @ K_g^T`` (``fwpkm/fwpkm.py:861``).  dS [R, 2, n]
    (row = token*H + head), q [R, k_dim], k [2*H*n, k_dim/2]; the groups are
    addressed as column / row offsets of the 2-D views, no copies.  fp32 on
    the library's fp32 GEMM; other dtypes as the einsums."""
    R, kd = q.shape
    half, G = kd // 2, 2 * H
    T = R // H
    n = k.shape[0] // G
    if not (dS.dtype == q.dtype == k.dtype == torch.float32 and dS.is_cuda):
        d = dS.view(T, H, 2, n)
        dq = torch.einsum("thpn,hpnd->thpd", d, k.view(H, 2, n, half)).reshape(R, kd) if want_dq else None
        dk = torch.einsum("thpn,thpd->hpnd", d, q.view(T, H, 2, half)).reshape(k.shape) if want_dk else None
        return dq, dk
    dS2 = dS.contiguous().view(T, G * n)
    q2 = q.contiguous().view(T, G * half)
    k2 = k.contiguous().view(G * n, half)
    dq = dk = None
    if want_dq:
        dq = torch.empty((T, G * half), dtype=q.dtype, device=q.device)
        _native.gemm_f32(dS2, k2, b_mn=True, batch=G, M=T, N=half, K=n, a_batch=(n, 0), b_batch=(0, n), out=dq,
                         c_batch_stride=half)
        dq = dq.view(R, kd)
    if want_dk:
        dk = torch.empty((G * n, half), dtype=k.dtype, device=k.device)
        _native.gemm_f32(dS2, q2, a_mn=True, b_mn=True, batch=G, M=n, N=half, K=T, a_batch=(n, 0),
                         b_batch=(half, 0), out=dk, c_batch_stride=n * half)
        dk = dk.view(k.shape)
    return dq, dk


def _group_scores(a, k, H):
    """``S_g = A_g @ K_g^T`` per (head, half) group for a query-shaped a
    [R, k_dim] and key-shaped k: [R, 2, n] (the scoring product itself, as a
    GEMM; used for second derivatives)."""
    R, kd = a.shape
    half, G = kd // 2, 2 * H
    T = R // H
    n = k.shape[0] // G
    if not (a.dtype == k.dtype == torch.float32 and a.is_cuda):
        return torch.einsum("thpd,hpnd->thpn", a.view(T, H, 2, half), k.view(H, 2, n, half)).reshape(R, 2, n)
    out = torch.empty((T, G * n), dtype=a.dtype, device=a.device)
    _native.gemm_f32(a.contiguous().view(T, G * half), k.contiguous().view(G * n, half), batch=G, M=T, N=n, K=half,
                     a_batch=(half, 0), b_batch=(0, n), out=out, c_batch_stride=n)
    return out.view(R, 2, n)


class GroupMM(torch.autograd.Function):
    """``(dS_g @ K_g, dS_g^T @ Q_g)`` over the (head, half) groups: the
    gradients of the sub-key products, differentiable once more in
    (dS, q, k) for the inner updates' ``create_graph`` (the outer backward
    takes the second derivative through them)."""

    @staticmethod
    def forward(ctx, dS, q, k, H):
        ctx.save_for_backward(dS, q, k)
        ctx.H = H
        dq, dk = _group_mm(dS, q, k, H)
        return dq, dk

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, g_dq, g_dk):
        dS, q, k = ctx.saved_tensors
        H = ctx.H
        d_dS = d_q = d_k = None
        # dq = dS @ K:  d(dS) += g_dq @ K^T,  dK += dS^T @ g_dq
        # dk = dS^T @ Q: d(dS) += Q @ g_dk^T,  dQ += dS @ g_dk
        if g_dq is not None:
            d_dS = _group_scores(g_dq.contiguous(), k, H)
            _, d_k = _group_mm(dS, g_dq.contiguous(), k, H, want_dq=False)
        if g_dk is not None:
            t = _group_scores(q, g_dk.contiguous(), H)
            d_dS = t if d_dS is None else d_dS + t
            d_q, _ = _group_mm(dS, q, g_dk.contiguous(), H, want_dk=False)
        return d_dS, d_q, d_k, None


class SubkeyScores(torch.autograd.Function):
    """Dot-product sub-key scores ``[R, 2, n]`` of queries ``[R, k_dim]``
    (``fwpkm/fwpkm.py:861``).

    Forward: the sequential-sum kernel.  Backward: the grouped products
    ``dS @ K`` and ``dS^T @ Q`` on the saved query and keys (as the
    reference's einsum backward reads them), through ``GroupMM`` so that
    they are differentiable again (the inner updates take gradients with
    ``create_graph=True``)."""

    @staticmethod
    def forward(ctx, query, keys, heads):
        s = _native.subkey_scores(query.contiguous(), keys.contiguous(), heads, "dot")
        ctx.save_for_backward(query, keys)
        ctx.heads = heads
        return s

    @staticmethod
    def backward(ctx, dS):
        q, k = ctx.saved_tensors
        dq, dk = GroupMM.apply(dS.contiguous(), q, k, ctx.heads)
        return dq, dk, None


class SubkeyDist(torch.autograd.Function):
    """Euclidean distances ``[R, 2, n]`` between query halves and sub-keys,
    ``sqrt(max(|q|^2 - 2 q.k + |k|^2, 1e-30))`` as torch's ``cdist`` with
    ``use_mm_for_euclid_dist`` (``fwpkm/fwpkm.py:864``).

    Backward follows that op's own derivative: with ``ratio = grad / dist``,
    ``dq = q * sum(ratio) - ratio @ k`` and ``dk = k * sum(ratio) - ratio^T @ q``,
    using the saved distances and the saved query/keys tensors, so it reads
    exactly what the reference's autograd reads."""

    @staticmethod
    def forward(ctx, query, keys, heads):
        dist = _native.subkey_scores(query.contiguous(), keys.contiguous(), heads, "dist")
        ctx.save_for_backward(query, keys, dist)
        ctx.heads = heads
        return dist

    @staticmethod
    def backward(ctx, grad):
        q, k, dist = ctx.saved_tensors
        H = ctx.heads
        R, kd = q.shape
        half = kd // 2
        n = k.shape[0] // (2 * H)
        ratio = grad / dist
        rk, rq = GroupMM.apply(ratio.contiguous(), q, k, H)  # ratio @ K, ratio^T @ Q per group
        r4 = ratio.view(R // H, H, 2, n)
        qv = q.view(R // H, H, 2, half)
        kv = k.view(H, 2, n, half)
        dq = qv * r4.sum(-1, keepdim=True) - rk.view(R // H, H, 2, half)
        dk = kv * r4.sum(0).unsqueeze(-1) - rq.view(H, 2, n, half)
        return dq.reshape(R, kd), dk.reshape(k.shape), None


class IdwScore(torch.autograd.Function):
    """``-log(1e-3 + dist^2)`` (``fwpkm/fwpkm.py:866``); the log is taken in
    fp64 and rounded, the oracle's definition, and the backward is
    ``-grad / (1e-3 + dist^2) * 2 dist`` in differentiable tensor ops."""

    @staticmethod
    def forward(ctx, dist):
        t = 1e-3 + dist * dist
        ctx.save_for_backward(dist)
        return (-torch.log(t.double())).to(dist.dtype)

    @staticmethod
    def backward(ctx, grad):
        (dist,) = ctx.saved_tensors
        return (-grad / (1e-3 + dist.pow(2))) * (2 * dist)


class ScoreTransform(torch.autograd.Function):
    """``score_transform`` (``fwpkm/fwpkm.py:105-115``) on the library's
    kernel: softmax / silu / relu of ``scores / temperature`` over each row
    of ``[tokens, H*knn]`` (jointly over the heads), in the scores' dtype.
    The backward is one kernel.  When it runs under ``create_graph`` (an
    inner update whose loss reaches the keys through the weights:
    ``mem_grad_to_values_only=False``) it is the same derivative in tensor
    ops instead, so that the outer backward can differentiate it again, as
    torch's own softmax backward can be."""

    @staticmethod
    def forward(ctx, scores, temperature, mode):
        s = scores.contiguous()
        y = _native.score_transform_fwd(s, temperature, mode)
        ctx.save_for_backward(s if mode != "softmax" else None, y if mode == "softmax" else None)
        ctx.args = (temperature, mode)
        return y

    @staticmethod
    def backward(ctx, dy):
        s, y = ctx.saved_tensors
        temperature, mode = ctx.args
        if not torch.is_grad_enabled():
            return _native.score_transform_bwd(s, y, dy, temperature, mode), None, None
        if mode == "softmax":
            dx = y * (dy - (dy * y).sum(-1, keepdim=True)) / temperature
        else:
            z = s / temperature
            if mode == "silu":
                sg = torch.sigmoid(z)
                dx = dy * sg * (1 + z * (1 - sg)) / temperature
            else:
                dx = dy * (z > 0).to(dy.dtype) / temperature
        return dx, None, None


class FusedValueUpdate(torch.autograd.Function):
    """Value branch of ``update_fw`` (``fwpkm/fwpkm.py:274-367``) as one
    kernel pass: ``scaled = grad * scale / max(bincount(indices), 1)``,
    ``new = values - lr * (clamp?(scaled) + wd * values)``.  Returns
    ``(new, scaled)``; differentiable in ``values`` and ``grad`` for the
    outer backward through the inner update."""

    @staticmethod
    def forward(ctx, values, grad, indices, scale, lr, weight_decay, grad_clip):
        new, scaled, counts = _native.fw_update(values, grad, indices, scale, lr, weight_decay, grad_clip)
        ctx.save_for_backward(scaled if grad_clip else None, counts)
        ctx.args = (scale, lr, weight_decay, grad_clip)
        return new, scaled

    @staticmethod
    def backward(ctx, d_new, d_scaled):
        scaled, counts = ctx.saved_tensors
        scale, lr, wd, clip = ctx.args
        if d_new is None:
            d_new = torch.zeros_like(d_scaled)
        # d_values = d_new * (1 - lr * wd): without weight decay that is
        # d_new itself, passed on rather than copied (1 GiB at config 4)
        pass_through = ctx.needs_input_grad[0] and wd == 0.0
        dv = dg = None
        if (ctx.needs_input_grad[0] and not pass_through) or ctx.needs_input_grad[1]:
            dv, dg = _native.fw_update_bwd(d_new, d_scaled, scaled, counts, scale, lr, wd, clip,
                                           need_values=ctx.needs_input_grad[0] and not pass_through,
                                           need_grad=ctx.needs_input_grad[1])
        if pass_through:
            dv = d_new
        return dv, dg, None, None, None, None, None


class FastWeightProductKeyMemory(nn.Module):
    def __init__(
        self,
        mem_k_dim=512,
        mem_v_dim=512,
        mem_heads=1,
        mem_topk=8,
        mem_n_subkeys=512,
        lookahead=1,
        qk_score_type="idw",
        score_nonlinear="softmax",
        score_temperature=1.0,
        optimizer_type="sgd",
        learning_rate=1.0,
        weight_decay=0.0,
        loss_type="mse",
        mem_grad_to_values_only=True,
        grad_clip=False,
        addr_loss="me",
        addr_loss_weight=1.0,
        fp32_fw=True,
    ):
        assert mem_k_dim >= 2
        assert mem_k_dim % 2 == 0
        super().__init__()
        self.subsize = mem_n_subkeys
        self.size = mem_n_subkeys**2
        self.k_dim = mem_k_dim
        self.v_dim = mem_v_dim
        self.heads = mem_heads
        self.topk = mem_topk
        self.lookahead = lookahead
        self.qk_score_type = qk_score_type
        self.score_nonlinear = score_nonlinear
        self.score_temperature = score_temperature
        self.optimizer_type = optimizer_type
        self.learning_rate = learning_rate
        self.weight_decay = weight_decay
        self.loss_type = loss_type
        self.mem_grad_to_values_only = mem_grad_to_values_only
        self.grad_clip = grad_clip
        self.addr_loss = addr_loss
        self.addr_loss_weight = addr_loss_weight
        self.fp32_fw = fp32_fw
        self.ob_mode = None
        self.ob_idx2log = defaultdict(list)
        self.keys = nn.Parameter(torch.zeros(2 * self.heads * self.subsize, self.k_dim // 2))
        self.values = nn.Parameter(torch.zeros(self.size, self.v_dim))

    def reset_parameters(self):
        bound = 1 / math.sqrt(self.k_dim)
        nn.init.uniform_(self.keys, a=-bound, b=bound)
        nn.init.normal_(self.values, mean=0, std=self.v_dim**-0.5)

    # ------------------------------------------------------------------
    # pieces of one read / update (fwpkm/fwpkm.py:97-367)
    # ------------------------------------------------------------------
    def get_fw_named_params(self):
        out = OrderedDict()
        for name, p in self.named_parameters():
            out[name] = p.float() if self.fp32_fw else p
        return out

    def score_transform(self, scores):
        """Normalise each row of ``scores`` [tokens, H*knn] (``fwpkm/fwpkm.py:105-115``)."""
        if self.score_nonlinear not in ("softmax", "silu", "relu"):
            raise NotImplementedError(f"Non-linear {self.score_nonlinear} not implemented for scores.")
        rows = scores.reshape(-1, scores.shape[-1])
        return ScoreTransform.apply(rows, float(self.score_temperature), self.score_nonlinear).view(scores.shape)

    def compute_marginal_entropy(self, M, epsilon=1e-8, sorted_idx=None):
        """Entropy of the batch-mean of a top-k-thresholded softmax of M [N, K].
        Split over data-parallel ranks, the batch mean is over every rank's
        rows (a differentiable all-reduce of the row sums).  ``sorted_idx``
        [N, topk], when given, are each row's topk best columns, best first
        (the product top-k's stage-1 lists of these very scores): the
        threshold, the topk-th largest value, is then read at its last
        column instead of running a top-k again (equal values tie, so the
        value is the same whichever tied column holds it)."""
        in_dtype = M.dtype
        if self.addr_loss_weight == 0.0:
            return torch.tensor(0.0, device=M.device, dtype=in_dtype)
        if sorted_idx is not None:
            kth = M.gather(1, sorted_idx.reshape(M.shape[0], -1)[:, self.topk - 1:self.topk].long())
        else:
            kth = torch.topk(M, self.topk, dim=1).values[:, -1:]
        M = torch.where(M >= kth, M, torch.full_like(M, float("-inf"))).float()
        world, group = self._dp()
        if world == 1:
            P_bar = F.softmax(M, dim=1).mean(dim=0)
        else:
            from torch.distributed.nn.functional import all_reduce
            P_bar = all_reduce(F.softmax(M, dim=1).sum(dim=0), group=group) / (M.shape[0] * world)
        return (-(P_bar * torch.log(P_bar + epsilon)).sum()).to(in_dtype)

    # ------------------------------------------------------------------
    # data parallelism over the batch (replicated fast weights)
    # ------------------------------------------------------------------
    def data_parallel(self, group=None):
        """Split the batch over the ranks of ``group`` (every rank passes the
        same number of sequences and the same parameters).  The fast weights
        stay replicated and every inner update uses the gradient of the whole
        batch: per chunk the memorisation loss is each rank's share of the
        global mean, the value and key gradients are summed over the ranks
        with differentiable all-reduces (so the outer backward, second
        derivatives included, is the single-process one), the slot counts
        come from every rank's indices, and the addressing loss's batch mean
        covers every rank's rows.  After the outer backward, ``reduce_grads``
        sums the parameters' gradients over the ranks."""
        self.dp_group = group
        return self

    def row_sharded(self, group=None):
        """Split the batch over the ranks of ``group`` as ``data_parallel``
        does, and split the value table by rows instead of replicating it:
        this rank keeps rows ``[rank*S, rank*S + S)`` (``S = ceil(n^2 /
        world)``, the last shard zero-padded) of the current ``values``.
        Lookups go to the rows' owners and come back as partial bag sums;
        each owner computes the value gradient of its rows from every rank's
        lookups (nothing of the table is all-reduced), updates its rows with
        the slot counts of the lookups it served, and carries the double
        backward of its rows.  The keys stay replicated; their gradients are
        summed over the ranks.  Every rank must call it, with the same
        parameters."""
        import torch.distributed as dist
        self.dp_group = group if group is not None else dist.group.WORLD
        world = dist.get_world_size(self.dp_group)
        rank = dist.get_rank(self.dp_group)
        S = -(-self.size // world)
        self.shard_rows = S
        with torch.no_grad():
            full = self.values.detach()
            shard = torch.zeros((S, full.shape[1]), dtype=full.dtype, device=full.device)
            r0, r1 = rank * S, min((rank + 1) * S, self.size)
            if r1 > r0:
                shard[: r1 - r0].copy_(full[r0:r1])
        self.values = nn.Parameter(shard)
        return self

    def _sharded(self) -> bool:
        return getattr(self, "shard_rows", None) is not None and self._dp()[0] > 1

    def _dp(self):
        group = getattr(self, "dp_group", None)
        if group is None:
            return 1, None
        import torch.distributed as dist
        if not dist.is_initialized():
            return 1, None
        return dist.get_world_size(group), group

    def reduce_grads(self):
        """Sum the fast-weight parameters' gradients over the data-parallel ranks."""
        world, group = self._dp()
        if world == 1:
            return
        import torch.distributed as dist
        for p in (self.keys,) if self._sharded() else (self.keys, self.values):
            if p.grad is not None:
                dist.all_reduce(p.grad, group=group)

    def _all_indices(self, indices):
        """Every rank's slot indices of this chunk (for the global bincount)."""
        world, group = self._dp()
        if world == 1:
            return indices
        import torch.distributed as dist
        parts = [torch.empty_like(indices) for _ in range(world)]
        dist.all_gather(parts, indices.contiguous(), group=group)
        return torch.cat([t.reshape(-1) for t in parts])

    def retrieve_values(self, query: torch.Tensor, fw_named_params: OrderedDict):
        B, T = query.shape[:2]
        scores, indices, indices1, indices2, all_scores1, all_scores2 = self.get_indices(
            query.view(B * T, self.heads, self.k_dim), fw_named_params["keys"])
        normed_scores = self.score_transform(scores.view(B * T, self.heads * self.topk))
        route = None
        if self._sharded():
            from ..sharded import fw_sharded_bag
            vals, route = fw_sharded_bag(indices.view(B * T, self.heads * self.topk), fw_named_params["values"],
                                         normed_scores, self.shard_rows, self._dp()[1])
        else:
            vals = xformers_embedding_bag(
                indices=indices.view(B * T, self.heads * self.topk),
                weight=fw_named_params["values"],
                per_sample_weights=normed_scores,
            )
        return {
            "route": route,
            "retireved_values": vals,
            "scores": scores,
            "normed_scores": normed_scores,
            "indices": indices,
            "sub_indices1": indices1,
            "sub_indices2": indices2,
            "all_sub_scores1": all_scores1,
            "all_sub_scores2": all_scores2,
        }

    def compute_mem_loss(self, hyp_values, ref_values, loss_mask=None, loss_weights=None):
        if self.loss_type != "mse":
            raise NotImplementedError(f"Loss type {self.loss_type} not implemented.")
        mem_losses = F.mse_loss(hyp_values, ref_values, reduction="none").mean(dim=-1)
        if loss_mask is not None:
            mem_losses = mem_losses * loss_mask
        if loss_weights is not None:
            mem_losses = mem_losses * loss_weights
        return mem_losses

    def compute_addr_loss(self, sub_indices1, sub_indices2, all_sub_scores1, all_sub_scores2):
        if self.addr_loss is None:
            return None
        if self.addr_loss != "me":
            raise NotImplementedError(f"Addressing loss {self.addr_loss} not implemented.")
        s1 = all_sub_scores1.reshape(-1, self.subsize)
        s2 = all_sub_scores2.reshape(-1, self.subsize)
        i1 = sub_indices1.reshape(s1.shape[0], -1) if sub_indices1 is not None else None
        i2 = sub_indices2.reshape(s2.shape[0], -1) if sub_indices2 is not None else None
        if i1 is not None and (i1.shape[1] != self.topk or i2 is None or i2.shape[1] != self.topk):
            i1 = i2 = None
        return self.addr_loss_weight * (-self.compute_marginal_entropy(s1, sorted_idx=i1)
                                        - self.compute_marginal_entropy(s2, sorted_idx=i2))

    def update_fw_param(self, p, g, lr, wd):
        if self.optimizer_type != "sgd":
            raise NotImplementedError(f"Optimizer {self.optimizer_type} not implemented.")
        return p - lr * (g + wd * p)

    def update_fw(self, fw_named_params, num_samples, indices, mem_loss, addr_loss=None, route=None):
        """One SGD step on the fast weights (``fwpkm/fwpkm.py:274-367``).
        With a row-split table (``route`` of the chunk's lookups) the value
        gradient is already this rank's rows' sum over every rank, and the
        slot counts are those of the lookups this rank served."""
        mem_loss = mem_loss * 0.5
        names = list(fw_named_params.keys())
        params = tuple(fw_named_params.values())
        if self.mem_grad_to_values_only:
            if addr_loss is not None:
                addr_grads = torch.autograd.grad(addr_loss, params, create_graph=self.training, allow_unused=True)
            else:
                addr_grads = [None] * len(params)
            (mem_grad,) = torch.autograd.grad(mem_loss, fw_named_params["values"], create_graph=self.training)
            grads = [mem_grad if n == "values" else addr_grads[i] for i, n in enumerate(names)]
        else:
            loss = mem_loss if addr_loss is None else mem_loss + addr_loss
            grads = list(torch.autograd.grad(loss, params, create_graph=self.training))
        world, group = self._dp()
        sharded = route is not None
        if world > 1:
            # each rank holds its batch share's gradient: sum them (the
            # all-reduce is differentiable, so the outer backward sees the sum);
            # a row-split value table's gradient is complete on its owner
            from torch.distributed.nn.functional import all_reduce
            grads = [g if g is None or (sharded and n == "values") else all_reduce(g, group=group)
                     for n, g in zip(names, grads)]
            indices = route.r_row.long() if sharded else self._all_indices(indices)
        # the value gradient is a sum over samples, features, heads and top-k,
        # shared out over the times each slot was read; its scaling, the
        # bincount, the clamp and the SGD step run as one fused kernel pass
        fused = {}
        for i, n in enumerate(names):
            if n == "values" and grads[i] is not None:
                scale = num_samples * self.v_dim * self.topk * self.heads
                new_v, grads[i] = FusedValueUpdate.apply(params[i], grads[i], indices, scale, self.learning_rate,
                                                         self.weight_decay, self.grad_clip)
                fused[n] = new_v
        used = [None if g is None else (torch.clamp(g, min=-1.0, max=1.0) if self.grad_clip else g) for g in grads]
        # a parameter without a gradient (keys when there is no addressing
        # loss) is left as it is; the reference fails with a TypeError there
        updated = OrderedDict(
            (n, fused[n] if n in fused else params[i] if used[i] is None else
             self.update_fw_param(params[i], used[i], self.learning_rate, self.weight_decay))
            for i, n in enumerate(names))
        return updated, grads

    def write_ob_log(self, token_ids, indices, scores):
        """Per-slot observation log (``fwpkm/fwpkm.py:369-393``), host-side."""
        assert self.ob_mode
        B, T = token_ids.shape
        ids = token_ids.tolist()
        for b in range(B):
            for t in range(T - self.lookahead):
                q_id = ids[b][t]
                v_id = ids[b][t + self.lookahead]
                lo = max(0, t + self.lookahead - 10)
                hi = min(T, t + self.lookahead + 10)
                prev = ids[b][lo:t + self.lookahead]
                nxt = ids[b][t + self.lookahead + 1:hi]
                for htk in range(self.heads * self.topk):
                    entry = (q_id, v_id, prev, nxt, scores[b, t, htk].item())
                    self.ob_idx2log[indices[b, t, htk].item()].append(entry)

    # ------------------------------------------------------------------
    # chunked forward
    # ------------------------------------------------------------------
    def _lookahead_target(self, ref):
        """Targets shifted by ``lookahead`` tokens (``fwpkm/fwpkm.py:472-480``)."""
        return ref if self.lookahead == 0 else ref[:, self.lookahead:]

    def _global_count(self, n: int) -> int:
        world, group = self._dp()
        if world == 1:
            return n
        import torch.distributed as dist
        t = torch.tensor([n], dtype=torch.int64, device=self.keys.device)
        dist.all_reduce(t, group=group)
        return int(t.item())

    def forward_wo_past(self, q, ref_v, chunk_size, gates=None, loss_mask=None, token_ids=None):
        B, T = q.shape[:2]
        world, _ = self._dp()
        input_dtype = q.dtype
        if self.fp32_fw:
            q = q.float()
            ref_v = ref_v.float()
        cut = None if self.lookahead == 0 else -self.lookahead
        all_grads, output, losses, indices, scores = [], [], [], [], []
        addr_losses = [] if self.addr_loss is not None else None
        with torch.enable_grad():
            fw_params = [self.get_fw_named_params()]
            for c0 in range(0, T, chunk_size):
                c1 = min(c0 + chunk_size, T)
                cT = c1 - c0
                cq = q[:, c0:c1].contiguous()
                cref = ref_v[:, c0:c1].contiguous()
                cgates = gates[:, c0:c1].contiguous() if gates is not None else None
                cmask = loss_mask[:, c0:c1].contiguous() if loss_mask is not None else None
                cids = token_ids[:, c0:c1].contiguous() if token_ids is not None else None
                cur = fw_params[-1]
                r = self.retrieve_values(cq, cur)
                hyp = r["retireved_values"].view(B, cT, -1)
                output.append(hyp)
                indices.append(r["indices"].view(B, cT, -1))
                scores.append(r["normed_scores"].view(B, cT, -1))
                upd_hyp = hyp[:, :cut].contiguous()
                upd_w = cgates[:, :cut].contiguous() if cgates is not None else None
                upd_mask = cmask[:, :cut].contiguous() if cmask is not None else None
                upd_ref = self._lookahead_target(cref).contiguous()
                mem_losses = self.compute_mem_loss(
                    upd_hyp.view(-1, upd_hyp.size(-1)), upd_ref.view(-1, upd_ref.size(-1)),
                    loss_mask=upd_mask.view(-1) if upd_mask is not None else None,
                    loss_weights=upd_w.view(-1) if upd_w is not None else None)
                addr_loss = self.compute_addr_loss(r["sub_indices1"], r["sub_indices2"], r["all_sub_scores1"],
                                                   r["all_sub_scores2"])
                num_samples = (upd_mask > 0).sum().item() if upd_mask is not None else B * cT
                mem_loss = mem_losses.mean()
                if world > 1:
                    # this rank's share of the batch mean and of the batch's samples
                    mem_loss = mem_loss / world
                    num_samples = self._global_count(num_samples)
                    addr_loss = None if addr_loss is None else addr_loss / world
                new_params, grads = self.update_fw(cur, num_samples, r["indices"], mem_loss, addr_loss,
                                                   route=r["route"])
                if world > 1 and addr_loss is not None:
                    addr_loss = addr_loss * world
                if self.ob_mode:
                    self.write_ob_log(cids.view(B, cT), r["indices"].view(B, cT, -1), cgates.view(B, cT, -1))
                all_grads.append([None if g is None else g.detach() for g in grads])
                fw_params.append(new_params)
                losses.append(mem_losses.view(B, -1).detach())
                if addr_losses is not None:
                    addr_losses.append(addr_loss.detach())
        output = torch.cat(output, dim=1)
        indices = torch.cat(indices, dim=1).view(B, T, self.heads, self.topk)
        scores = torch.cat(scores, dim=1).view(B, T, self.heads, self.topk)
        losses = torch.cat(losses, dim=1)
        addr_loss = torch.stack(addr_losses).mean() if addr_losses is not None else None
        with torch.no_grad():
            names0 = list(fw_params[0].keys())

            def _norm(g, n):
                if g is None:
                    return torch.zeros((), device=q.device)
                if n == "values" and self._sharded():
                    # the norm of the whole table's gradient from the shards'
                    import torch.distributed as dist
                    sq = g.double().pow(2).sum()
                    dist.all_reduce(sq, group=self._dp()[1])
                    return sq.sqrt().to(g.dtype)
                return g.norm()
            grad_norms = [torch.stack([_norm(g[i], names0[i]) for g in all_grads]).mean()
                          for i in range(len(fw_params[0]))]
            final = fw_params[-1]
            for n, p in self.named_parameters():
                if n in final:
                    p.data.copy_(final[n].data.to(p.dtype))
        return {
            "output": output.to(input_dtype),
            "indices": indices,
            "scores": scores,
            "losses": losses,
            "addr_loss": addr_loss,
            "grad_norms": grad_norms,
            "past_key_values": None,
        }

    def forward_w_past(self, q, ref_v, gates, chunk_size, loss_mask=None, past_key_values=None, token_ids=None):
        """Streaming read/update with a carried signal queue (``fwpkm/fwpkm.py:560-820``)."""
        if self._sharded():
            raise NotImplementedError("forward_w_past with a row-split value table")
        B, T = q.shape[:2]
        input_dtype = q.dtype
        if self.fp32_fw:
            q = q.float()
            ref_v = ref_v.float()
        dev, dt = ref_v.device, ref_v.dtype

        def empty(width=None, dtype=dt):
            return torch.zeros(B, 0, width, device=dev, dtype=dtype) if width else torch.zeros(B, 0, device=dev,
                                                                                               dtype=dtype)

        q_queue, hyp_queue, ref_queue = empty(q.size(-1)), empty(ref_v.size(-1)), empty(ref_v.size(-1))
        gates_queue = empty() if gates is not None else None
        mask_queue = empty() if loss_mask is not None else None
        ids_queue = empty(dtype=torch.long) if token_ids is not None else None
        if past_key_values is not None:
            pq, ph, pr, pg, pm, pi = past_key_values
            if ph is not None:
                assert ph.size(1) < chunk_size + self.lookahead, (
                    f"Past key values length {ph.size(1)} longer than chunk size + lookahead "
                    f"({chunk_size} + {self.lookahead}).")
                q_queue = torch.cat([pq, q_queue], 1)
                hyp_queue = torch.cat([ph, hyp_queue], 1)
                ref_queue = torch.cat([pr, ref_queue], 1)
                gates_queue = torch.cat([pg, gates_queue], 1) if gates is not None else None
                mask_queue = torch.cat([pm, mask_queue], 1) if loss_mask is not None else None
                ids_queue = torch.cat([pi, ids_queue], 1) if token_ids is not None else None
        first_end = min(chunk_size + self.lookahead - ref_queue.size(1), T)
        bounds = [(0, first_end)] + [(s, min(s + chunk_size, T)) for s in range(first_end, T, chunk_size)]
        cut = None if self.lookahead == 0 else -self.lookahead
        updated = False
        cur = self.get_fw_named_params()
        output, losses, indices, scores = [], [], [], []
        addr_losses = [] if self.addr_loss is not None else None
        mem_losses = addr_loss = update_mask = None
        for c0, c1 in bounds:
            cT = c1 - c0
            cq = q[:, c0:c1].contiguous()
            cref = ref_v[:, c0:c1].contiguous()
            cgates = gates[:, c0:c1].contiguous() if gates is not None else None
            cmask = loss_mask[:, c0:c1].contiguous() if loss_mask is not None else None
            cids = token_ids[:, c0:c1].contiguous() if token_ids is not None else None
            r = self.retrieve_values(cq, cur)
            hyp = r["retireved_values"].view(B, cT, -1)
            chunk_indices = r["indices"]
            output.append(hyp)
            indices.append(chunk_indices.view(B, cT, -1))
            scores.append(r["normed_scores"].view(B, cT, -1))
            q_queue = torch.cat([q_queue, cq], 1)
            hyp_queue = torch.cat([hyp_queue, hyp], 1)
            ref_queue = torch.cat([ref_queue, cref], 1)
            gates_queue = torch.cat([gates_queue, cgates], 1) if gates is not None else None
            mask_queue = torch.cat([mask_queue, cmask], 1) if loss_mask is not None else None
            ids_queue = torch.cat([ids_queue, cids], 1) if token_ids is not None else None
            if past_key_values and hyp_queue.size(1) < chunk_size:
                continue
            updated = True
            with torch.enable_grad():
                cur = {n: p.detach() for n, p in cur.items()}
                for p in cur.values():
                    p.requires_grad = True
                rb = self.retrieve_values(q_queue[:, :cut].contiguous(), cur)
                update_hyp = rb["retireved_values"].contiguous()
                update_w = gates_queue[:, :cut].contiguous() if gates_queue is not None else None
                update_mask = mask_queue[:, :cut].contiguous() if mask_queue is not None else None
                update_ref = self._lookahead_target(ref_queue).contiguous()
                mem_losses = self.compute_mem_loss(
                    update_hyp.view(-1, update_hyp.size(-1)), update_ref.view(-1, update_ref.size(-1)),
                    loss_mask=update_mask.view(-1) if update_mask is not None else None,
                    loss_weights=update_w.view(-1) if update_w is not None else None)
                addr_loss = self.compute_addr_loss(rb["sub_indices1"], rb["sub_indices2"], rb["all_sub_scores1"],
                                                   rb["all_sub_scores2"])
                num_samples = (update_mask > 0).sum().item() if update_mask is not None else B * cT
                cur, _ = self.update_fw(cur, num_samples, chunk_indices, mem_losses.mean(), addr_loss)
                if self.ob_mode:
                    pad = torch.zeros(B, self.lookahead, self.heads * self.topk, device=dev,
                                      dtype=rb["indices"].dtype)
                    idx_p = torch.cat([rb["indices"].view(B, ids_queue.size(1) - self.lookahead, -1), pad], 1)
                    sc_p = torch.cat([rb["scores"].view(B, ids_queue.size(1) - self.lookahead, -1),
                                      pad.to(rb["scores"].dtype)], 1)
                    self.write_ob_log(ids_queue, idx_p, sc_p)
            if self.lookahead == 0:
                q_queue, hyp_queue, ref_queue = empty(q.size(-1)), empty(ref_v.size(-1)), empty(ref_v.size(-1))
                gates_queue = empty() if gates is not None else None
                mask_queue = empty() if loss_mask is not None else None
                ids_queue = empty(dtype=torch.long)
            else:
                keep = slice(-self.lookahead, None)
                q_queue = q_queue[:, keep].contiguous()
                hyp_queue = hyp_queue[:, keep].contiguous()
                ref_queue = ref_queue[:, keep].contiguous()
                gates_queue = gates_queue[:, keep].contiguous() if gates is not None else None
                mask_queue = mask_queue[:, keep].contiguous() if update_mask is not None else None
                ids_queue = ids_queue[:, keep].contiguous() if ids_queue is not None else None
            losses.append(mem_losses.view(B, -1).detach())
            if addr_losses is not None:
                addr_losses.append(addr_loss.detach())
        output = torch.cat(output, 1)
        indices = torch.cat(indices, 1).view(B, T, self.heads, self.topk)
        scores = torch.cat(scores, 1).view(B, T, self.heads, self.topk)
        past = (q_queue, hyp_queue, ref_queue, gates_queue, mask_queue, ids_queue)
        if updated:
            losses = torch.cat(losses, 1)
            addr_out = torch.stack(addr_losses).mean() if addr_losses is not None else None
            with torch.no_grad():
                for n, p in self.named_parameters():
                    if n in cur:
                        p.data.copy_(cur[n].data.to(p.dtype))
        else:
            losses = None
            addr_out = None
        return {
            "output": output.to(input_dtype),
            "indices": indices,
            "scores": scores,
            "losses": losses,
            "addr_loss": addr_out,
            "grad_norms": None,
            "past_key_values": past,
        }

    @torch.compiler.disable(recursive=True)
    def forward(self, q, ref_v, gates, chunk_size, loss_mask=None, past_key_values=None, token_ids=None):
        if past_key_values is None:
            return self.forward_wo_past(q=q, ref_v=ref_v, gates=gates, chunk_size=chunk_size, loss_mask=loss_mask,
                                        token_ids=token_ids)
        return self.forward_w_past(q=q, ref_v=ref_v, gates=gates, chunk_size=chunk_size, loss_mask=loss_mask,
                                   past_key_values=past_key_values, token_ids=token_ids)

    def compute_qk_scores(self, q, k):
        """Scores ``(batch, heads, n_keys)`` of queries ``(batch, heads, d)``
        against keys ``(heads, n_keys, d)`` (``fwpkm/fwpkm.py:853-869``)."""
        if self.qk_score_type == "dot_product":
            return torch.einsum("bhd,hnd->bhn", q, k)
        if self.qk_score_type == "idw":
            d = torch.cdist(q.permute(1, 0, 2), k, p=2, compute_mode="use_mm_for_euclid_dist").permute(1, 0, 2)
            return -torch.log(1e-3 + d.pow(2))
        raise NotImplementedError(f"QK score type {self.qk_score_type} not implemented.")

    def get_indices(self, query: torch.Tensor, keys: torch.Tensor):
        """``(scores, indices, topk_indices1, topk_indices2, scores1, scores2)``
        for queries ``(BT, heads, k_dim)`` (``fwpkm/fwpkm.py:871-934``)."""
        if self.qk_score_type not in ("dot_product", "idw"):
            raise NotImplementedError(f"QK score type {self.qk_score_type} not implemented.")
        topk, H, n = self.topk, self.heads, self.subsize
        BT = query.size(0)
        q2 = query.reshape(BT * H, self.k_dim)
        if keys.dtype != q2.dtype:
            keys = keys.to(q2.dtype)
        if self.qk_score_type == "dot_product":
            s_all = SubkeyScores.apply(q2, keys, H)  # [BT*H, 2, n]
        else:
            # The reference's cdist backward works on its own copy of the keys,
            # so an in-place overwrite of the key parameter after the forward
            # (the write-back at the end of ``forward_wo_past``, which aliases
            # the first chunk's fast weights when they are fp32) does not reach
            # it; the clone gives the same behaviour.
            s_all = IdwScore.apply(SubkeyDist.apply(q2, keys.clone(), H))
        with torch.no_grad():
            idx, _, _, sub1, sub2 = _native.product_topk(s_all.detach(), topk, want_sub=True)
        scores1 = s_all[:, 0].view(BT, H, n)
        scores2 = s_all[:, 1].view(BT, H, n)
        iv = idx.view(BT, H, topk)
        scores = scores1.gather(2, iv // n) + scores2.gather(2, iv % n)
        assert scores.shape == iv.shape == (BT, H, topk)
        return (scores.contiguous(), iv.contiguous(), sub1.view(BT, H, topk), sub2.view(BT, H, topk),
                scores1.contiguous(), scores2.contiguous())
