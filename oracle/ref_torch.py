"""The reference's product-key layer step on torch's CPU operators.

TEST AND BASELINE INFRASTRUCTURE ONLY.  Nothing in ``modelos_b200`` imports
this module.  ``bench.py`` times it as the reference arm and the CPU baseline
(the reference is a Python package with no build or install recipe, so its
own files cannot travel to the benchmark machine), and ``tests/`` pin it to
the fixtures that the reference itself wrote.

It restates one training step of ``HashingMemory`` (APamplonat/Modelos
``pkm/memory.py:190-289``, query network ``:292-349``) on the CPU path the
reference takes when its tensors are not on a GPU: the query projection and
``BatchNorm1d`` (or RMSNorm) in the layer's dtype, two sub-key einsums per
head, ``torch.topk`` twice, the cartesian sums and a third ``torch.topk``,
the per-head softmax in fp32, ``F.embedding_bag`` for the weighted bag
(``pkm/xformer_embeddingbag.py:436-437``), the SwiLU-gated value projection
(``pkm/memory.py:226-229``), and autograd for the backward.  Because it runs
the same torch operators in the same order on the same dtypes, its indices,
outputs and gradients equal the reference's bit for bit on the fixtures
(``tests/test_oracle_golden.py``), and its speed is the reference's.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def make_params(cfg: dict, seed: int = 0, dtype=torch.bfloat16) -> dict:
    """Leaf tensors of one layer, drawn like ``HashingMemory.reset_parameters``
    (``pkm/memory.py:169-188``): keys U(+-1/sqrt(k_dim)), values
    N(0, v_dim^-1/2), query weight xavier-uniform, SwiLU and value
    projections N(0, output_dim^-1/2), biases nn.Linear's default U(+-1/sqrt(fan_in))."""
    g = torch.Generator().manual_seed(seed)
    C, O = cfg["input_dim"], cfg["output_dim"]
    kd, H, n = cfg["mem_k_dim"], cfg["mem_heads"], cfg["mem_n_keys"]
    v = cfg["mem_v_dim"] if cfg.get("mem_v_dim", -1) > 0 else O

    def u(shape, b):
        return (torch.rand(shape, generator=g) * 2 - 1) * b

    def nrm(shape, std):
        return torch.randn(shape, generator=g) * std

    xav = math.sqrt(6.0 / (C + H * kd))
    P = {
        "keys": u((2 * H * n, kd // 2), 1 / math.sqrt(kd)),
        "values": nrm((n * n, v), v ** -0.5),
        "wq": u((H * kd, C), xav), "bq": u((H * kd,), 1 / math.sqrt(C)),
        "ws": nrm((v, C), O ** -0.5), "bs": u((v,), 1 / math.sqrt(C)),
        "wv": nrm((O, v), O ** -0.5), "bv": u((O,), 1 / math.sqrt(v)),
    }
    if cfg.get("mem_query_batchnorm", False):
        P["bn_w"] = torch.ones(H * kd)
        P["bn_b"] = torch.zeros(H * kd)
    P = {k: t.to(dtype).requires_grad_(True) for k, t in P.items()}
    if cfg.get("mem_query_batchnorm", False):
        P["bn_mean"] = torch.zeros(H * kd, dtype=dtype)
        P["bn_var"] = torch.ones(H * kd, dtype=dtype)
    return P


def params_from_state(st: dict, dtype) -> dict:
    """The same leaves from a ``HashingMemory`` state dict."""
    names = {"keys": "keys", "values": "values.weight", "wq": "query_proj.query_mlps.0.weight",
             "bq": "query_proj.query_mlps.0.bias", "ws": "swilu_projection.weight", "bs": "swilu_projection.bias",
             "wv": "value_proj.weight", "bv": "value_proj.bias", "bn_w": "query_proj.norm.weight",
             "bn_b": "query_proj.norm.bias"}
    P = {k: st[v].to(dtype).clone().requires_grad_(True) for k, v in names.items() if v in st}
    if "query_proj.norm.running_mean" in st:
        P["bn_mean"] = st["query_proj.norm.running_mean"].to(dtype).clone()
        P["bn_var"] = st["query_proj.norm.running_var"].to(dtype).clone()
    return P


def query(P: dict, x: torch.Tensor, heads: int, k_dim: int, norm: str = "bn") -> torch.Tensor:
    """``QueryMLP.forward`` (``pkm/memory.py:333-349``): [N, C] -> [N*H, k_dim]."""
    q = F.linear(x, P["wq"], P["bq"])
    if norm == "bn":
        q = F.batch_norm(q, P["bn_mean"], P["bn_var"], P["bn_w"], P["bn_b"], True, 0.1, 1e-6)
    return q.view(-1, k_dim)


def get_indices(q: torch.Tensor, keys: torch.Tensor, heads: int, knn: int):
    """``HashingMemory.get_indices`` (``pkm/memory.py:250-289``): scores and
    slots ``[N*H, knn]``, best first."""
    k_dim = q.shape[1]
    half = k_dim // 2
    qv = q.view(-1, heads, k_dim)
    bs = qv.shape[0]
    kv = keys.view(heads, 2, -1, half)
    n = kv.shape[2]
    s1 = torch.einsum("blh, lkh->blk", qv[:, :, :half], kv[:, 0])
    s2 = torch.einsum("blh, lkh->blk", qv[:, :, half:], kv[:, 1])
    s1, i1 = s1.topk(knn, dim=2, largest=True)
    s2, i2 = s2.topk(knn, dim=2, largest=True)
    pair_s = (s1.view(bs, heads, knn, 1).expand(bs, heads, knn, knn)
              + s2.view(bs, heads, 1, knn).expand(bs, heads, knn, knn)).view(bs, heads, -1)
    pair_i = (i1.view(bs, heads, knn, 1).expand(bs, heads, knn, knn) * n
              + i2.view(bs, heads, 1, knn).expand(bs, heads, knn, knn)).view(bs, heads, -1)
    top, best = torch.topk(pair_s, k=knn, dim=2, largest=True, sorted=True)
    slots = pair_i.gather(2, best)
    return top.view(bs * heads, knn), slots.view(bs * heads, knn)


def layer_forward(P: dict, x: torch.Tensor, heads: int, knn: int, k_dim: int, norm: str = "bn"):
    """``HashingMemory.forward`` for x [B, T, C]: (out [B, T, O], slots [B, T, H*knn])."""
    B, T, C = x.shape
    xf = x.view(-1, C)
    q = query(P, xf, heads, k_dim, norm)
    top, slots = get_indices(q, P["keys"], heads, knn)
    w = F.softmax(top.float(), dim=-1).type_as(top)
    slots = slots.view(-1, heads * knn)
    w = w.view(-1, heads * knn)
    bag = F.embedding_bag(slots, P["values"], per_sample_weights=w, mode="sum")
    out = F.linear(bag * F.silu(F.linear(xf, P["ws"], P["bs"])), P["wv"], P["bv"])
    return out.view(B, T, -1), slots.view(B, T, -1)


def layer_step(P: dict, x: torch.Tensor, heads: int, knn: int, k_dim: int, norm: str = "bn"):
    """Forward, loss ``sum(out^2)`` in fp32, backward into the leaves' ``.grad``."""
    for t in P.values():
        if t.requires_grad:
            t.grad = None
    out, slots = layer_forward(P, x, heads, knn, k_dim, norm)
    loss = (out.float() ** 2).sum()
    loss.backward()
    return out, slots, loss


# ---------------------------------------------------------------------------
# the fast-weight memory (fwpkm/fwpkm.py) on the same CPU operators
# ---------------------------------------------------------------------------
class _BagGradWrap(torch.autograd.Function):
    """The weight gradient of the fast-weight bag, exposed so the outer
    backward can differentiate it (fwpkm/xformer_embeddingbag_grad_wrapper.py
    :13-74): forward passes the first-order gradient through; backward is the
    bag's VJP, gathered rows weighted and dotted."""

    @staticmethod
    def forward(ctx, idx, psw, g, grad_weight):
        ctx.save_for_backward(idx, psw, g)
        return grad_weight

    @staticmethod
    def backward(ctx, g_bar):
        idx, a, g = ctx.saved_tensors
        B, L = idx.shape
        rows = g_bar.index_select(0, idx.reshape(-1)).view(B, L, -1)
        return None, (rows * g.unsqueeze(1)).sum(dim=-1), (a.unsqueeze(-1) * rows).sum(dim=1), None


class _FwBag(torch.autograd.Function):
    """``out[b] = sum_j psw[b,j] W[idx[b,j]]`` as the fast-weight memory runs it
    on CPU (fwpkm/xformer_embeddingbag_grad_wrapper.py:83-155): gather and
    weighted sum forward; the first-order backward of
    fwpkm/xformer_embeddingbag_legacy.py:147-167 wrapped for double backward."""

    @staticmethod
    def forward(ctx, W, idx, psw):
        B, L = idx.shape
        rows = W.index_select(0, idx.reshape(-1)).view(B, L, -1)
        ctx.save_for_backward(W, idx, psw)
        return (rows * psw.unsqueeze(-1)).sum(dim=1)

    @staticmethod
    def backward(ctx, g):
        W, idx, psw = ctx.saved_tensors
        B, L = idx.shape
        K, D = W.shape
        with torch.no_grad():
            rows = W.index_select(0, idx.reshape(-1)).view(B, L, D)
            d_psw = (rows.float() * g.unsqueeze(1).float()).sum(-1).to(psw.dtype)
            contrib = g.unsqueeze(1).float() * psw.unsqueeze(-1).float()
            dW = torch.zeros(K, D, dtype=torch.float32)
            dW.index_add_(0, idx.reshape(-1), contrib.reshape(-1, D))
            dW = dW.to(W.dtype)
        return _BagGradWrap.apply(idx, psw, g, dW), None, d_psw


def fw_make_params(cfg: dict, seed: int = 0) -> dict:
    """Fast weights drawn like ``reset_parameters`` (fwpkm/fwpkm.py:91-96), fp32 leaves."""
    g = torch.Generator().manual_seed(seed)
    H, kd, D, n = cfg["mem_heads"], cfg["mem_k_dim"], cfg["mem_v_dim"], cfg["mem_n_subkeys"]
    keys = (torch.rand((2 * H * n, kd // 2), generator=g) * 2 - 1) / math.sqrt(kd)
    values = torch.randn((n * n, D), generator=g) * D ** -0.5
    return {"keys": keys.requires_grad_(True), "values": values.requires_grad_(True)}


def _fw_scores(q, k, mode):
    if mode == "dot_product":
        return torch.einsum("bhd,hnd->bhn", q, k)
    d = torch.cdist(q.permute(1, 0, 2), k, p=2, compute_mode="use_mm_for_euclid_dist").permute(1, 0, 2)
    return -torch.log(1e-3 + d.pow(2))


def _fw_marginal_entropy(M, topk, eps=1e-8):
    kth = torch.topk(M, topk, dim=1)[0][:, -1].unsqueeze(1)
    M = torch.where(M >= kth, M, torch.full_like(M, float("-inf"))).float()
    P_bar = torch.mean(F.softmax(M, dim=1), dim=0)
    return -torch.sum(P_bar * torch.log(P_bar + eps))


def fw_forward(P: dict, q: torch.Tensor, ref_v: torch.Tensor, cfg: dict, chunk: int, mode: str = "idw"):
    """``forward_wo_past`` (fwpkm/fwpkm.py:395-558) with the module defaults
    (lookahead 1, softmax at temperature 1, SGD without weight decay, MSE
    memorisation loss on the values only, addressing loss "me" of weight 1,
    fp32 fast weights): returns (output [B, T, D], indices, addr_loss).  As
    in the reference, the first chunk's fast weights are the parameters
    themselves and the final weights are copied into them at the end."""
    H, kd, topk, n = cfg["mem_heads"], cfg["mem_k_dim"], cfg["mem_topk"], cfg["mem_n_subkeys"]
    lr = cfg.get("learning_rate", 1.0)
    in_dtype = q.dtype
    q, ref_v = q.float(), ref_v.float()
    B, T = q.shape[:2]
    half = kd // 2
    outs, idxs, addr = [], [], []
    fw = {"keys": P["keys"].float(), "values": P["values"].float()}
    with torch.enable_grad():
        for c0 in range(0, T, chunk):
            c1 = min(c0 + chunk, T)
            cT = c1 - c0
            cq = q[:, c0:c1].contiguous().view(B * cT, H, kd)
            cref = ref_v[:, c0:c1].contiguous()
            kv = fw["keys"].view(H, 2, -1, half)
            s1 = _fw_scores(cq[:, :, :half], kv[:, 0], mode)
            s2 = _fw_scores(cq[:, :, half:], kv[:, 1], mode)
            t1, i1 = s1.topk(topk, dim=2, largest=True)
            t2, i2 = s2.topk(topk, dim=2, largest=True)
            BT = B * cT
            pair_s = (t1.view(BT, H, topk, 1).expand(BT, H, topk, topk)
                      + t2.view(BT, H, 1, topk).expand(BT, H, topk, topk)).view(BT, H, topk ** 2)
            pair_i = (i1.view(BT, H, topk, 1).expand(BT, H, topk, topk) * n
                      + i2.view(BT, H, 1, topk).expand(BT, H, topk, topk)).view(BT, H, topk ** 2)
            top, best = torch.topk(pair_s, k=topk, dim=2, largest=True, sorted=True)
            slots = pair_i.gather(2, best).contiguous()
            w = F.softmax(top.contiguous().view(BT, H * topk) / 1.0, dim=-1).type_as(top)
            hyp = _FwBag.apply(fw["values"], slots.view(BT, H * topk), w).view(B, cT, -1)
            outs.append(hyp)
            idxs.append(slots.view(B, cT, -1))
            mem = F.mse_loss(hyp[:, :-1].contiguous().view(-1, hyp.size(-1)),
                             cref[:, 1:].contiguous().view(-1, hyp.size(-1)), reduction="none").mean(dim=-1)
            a_loss = 1.0 * (-1.0 * _fw_marginal_entropy(s1.contiguous().view(-1, n), topk)
                            + -1.0 * _fw_marginal_entropy(s2.contiguous().view(-1, n), topk))
            params = (fw["keys"], fw["values"])
            g_addr = torch.autograd.grad(a_loss, params, create_graph=True, allow_unused=True)
            (g_mem,) = torch.autograd.grad(mem.mean() * 0.5, fw["values"], create_graph=True)
            g_v = g_mem * (B * cT * cfg["mem_v_dim"] * topk * H)
            cnt = torch.bincount(slots.view(-1), minlength=n * n).to(g_v.dtype)
            cnt[cnt == 0] = 1.0
            g_v = g_v / cnt.unsqueeze(-1)
            fw = {"keys": fw["keys"] - lr * (g_addr[0] + 0.0 * fw["keys"]),
                  "values": fw["values"] - lr * (g_v + 0.0 * fw["values"])}
            addr.append(a_loss.detach())
    with torch.no_grad():
        P["keys"].data.copy_(fw["keys"].data)
        P["values"].data.copy_(fw["values"].data)
    out = torch.cat(outs, dim=1).to(in_dtype)
    return out, torch.cat(idxs, dim=1), torch.stack(addr).mean()


def fw_step(P: dict, q: torch.Tensor, ref_v: torch.Tensor, cfg: dict, chunk: int, mode: str = "idw"):
    """One training step of the fast-weight layer: forward, loss
    ``sum(out^2)``, outer backward into the leaves' and inputs' ``.grad``."""
    for t in list(P.values()) + [q, ref_v]:
        if t.requires_grad:
            t.grad = None
    out, idx, addr = fw_forward(P, q, ref_v, cfg, chunk, mode)
    loss = (out.float() ** 2).sum()
    loss.backward()
    return out, idx, loss
