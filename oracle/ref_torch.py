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
