"""CPU stand-in for ``modelos_b200._native`` (test infrastructure only).

Implements the tensor-level wrappers with torch CPU ops and the numpy oracle
so the host-side module logic (autograd wiring, chunk loop, update rule) can
be exercised without a GPU.  Tests install it with ``monkeypatch``; the
product package never imports it.
"""
from __future__ import annotations

import functools

import numpy as np
import torch

from oracle import pkm_oracle as po

DEVERR_INDEX = 1
DEVERR_TIMEOUT = 2


def bag_fwd(indices, weight, psw, out_dtype=None):
    rows = weight.double()[indices]
    w = torch.ones(indices.shape, dtype=torch.float64) if psw is None else psw.double()
    return (w[..., None] * rows).sum(1).to(out_dtype or weight.dtype)


def bag_bwd(indices, weight, psw, grad_out, *, num_rows=None, need_dpsw=True, want_counts=False,
            grad_weight_dtype=None):
    K = weight.shape[0] if weight is not None else num_rows
    D = grad_out.shape[1]
    g = grad_out.double()
    w = torch.ones(indices.shape, dtype=torch.float64) if psw is None else psw.double()
    dW = torch.zeros(K, D, dtype=torch.float64)
    dW.index_add_(0, indices.reshape(-1), (w[..., None] * g[:, None, :]).reshape(-1, D))
    dpsw = None
    if need_dpsw and psw is not None:
        dpsw = (weight.double()[indices] * g[:, None, :]).sum(-1).to(psw.dtype)
    counts = torch.bincount(indices.reshape(-1), minlength=K).int() if want_counts else None
    dt = grad_weight_dtype or (weight.dtype if weight is not None else grad_out.dtype)
    return dW.to(dt), dpsw, counts


def bag_bwd2(indices, a, gbar, grad_out, *, d_grad_out_dtype=None, d_a_dtype=None):
    rows = gbar.double()[indices]
    w = torch.ones(indices.shape, dtype=torch.float64) if a is None else a.double()
    dgo = (w[..., None] * rows).sum(1).to(d_grad_out_dtype or grad_out.dtype)
    da = None
    if a is not None:
        da = (rows * grad_out.double()[:, None, :]).sum(-1).to(d_a_dtype or a.dtype)
    return dgo, da


def subkey_scores(query, keys, heads, mode="dot"):
    bf16 = query.dtype == torch.bfloat16
    s = po.subkey_scores(query.float().numpy(), keys.float().numpy(), heads, mode=mode, bf16=bf16)
    return torch.from_numpy(s).to(query.dtype)


def product_topk(scores, knn, want_psw=False, want_sub=False):
    bf16 = scores.dtype == torch.bfloat16
    r = po.product_topk(scores.float().numpy(), knn, bf16=bf16)
    idx = torch.from_numpy(r["indices"]).long()
    top = torch.from_numpy(r["scores"]).to(scores.dtype)
    psw = torch.from_numpy(po.softmax_rows(r["scores"], bf16=bf16)).to(scores.dtype) if want_psw else None
    s1 = torch.from_numpy(r["sub_indices1"]).long() if want_sub else None
    s2 = torch.from_numpy(r["sub_indices2"]).long() if want_sub else None
    return idx, top, psw, s1, s2


def score_grad_dense(indices, psw, dpsw, n_keys):
    d = dpsw.float()
    if psw is not None:
        p = psw.float()
        d = p * (d - (p * d).sum(-1, keepdim=True))
    d = d.to(dpsw.dtype).float()
    R = indices.shape[0]
    out = torch.zeros(R, 2, n_keys)
    out[:, 0].scatter_add_(1, indices // n_keys, d)
    out[:, 1].scatter_add_(1, indices % n_keys, d)
    return out.to(dpsw.dtype)


def fw_update(values, grad, indices, scale, lr, weight_decay, grad_clip, want_scaled=True):
    K = values.shape[0]
    counts = torch.bincount(indices.reshape(-1), minlength=K).to(torch.int32)
    c = counts.to(grad.dtype)
    c = torch.where(c == 0, torch.ones_like(c), c)
    scaled = grad * scale / c.unsqueeze(-1)
    u = torch.clamp(scaled, min=-1.0, max=1.0) if grad_clip else scaled
    new = values - lr * (u + weight_decay * values)
    return new, scaled, counts


def fw_update_bwd(d_new, d_scaled, scaled, counts, scale, lr, weight_decay, grad_clip, need_values=True,
                  need_grad=True):
    c = counts.to(d_new.dtype)
    f = (scale / torch.where(c == 0, torch.ones_like(c), c)).unsqueeze(-1)
    du = -lr * d_new
    if grad_clip:
        du = du * ((scaled >= -1) & (scaled <= 1)).to(d_new.dtype)
    dg = f * (du + (d_scaled if d_scaled is not None else 0))
    dv = d_new * (1 - lr * weight_decay)
    return (dv if need_values else None), (dg if need_grad else None)


def swiglu_fwd(a, h):
    return a * torch.nn.functional.silu(h)


def swiglu_bwd(dz, a, h, need_da=True, bias_dtype=None):
    s = torch.nn.functional.silu(h)
    sig = torch.sigmoid(h)
    da = dz * s if need_da else None
    dh = dz * a * sig * (1 + h * (1 - sig))
    db = dh.sum(0).to(bias_dtype) if bias_dtype is not None else None
    return da, dh, db


def colsum(x, out_dtype=None):
    return x.sum(0).to(out_dtype or x.dtype)


def segment_sum(rows, entry_row, entry_w, seg_offsets, out_dtype=None):
    n_segs = seg_offsets.numel() - 1
    seg = torch.repeat_interleave(torch.arange(n_segs), (seg_offsets[1:] - seg_offsets[:-1]).long())
    out = torch.zeros((n_segs, rows.shape[1]), dtype=torch.float32)
    out.index_add_(0, seg, rows[entry_row.long()].float() * entry_w.float()[:, None])
    return out.to(out_dtype or rows.dtype)


def bag_bwd_ragged(row_idx, src_of, psw, weight, grad_rows, need_dpsw=True):
    g = grad_rows.float()[src_of.long()]
    dW = torch.zeros(weight.shape, dtype=torch.float32)
    dW.index_add_(0, row_idx.long(), g * psw.float()[:, None])
    dpsw = (g * weight.float()[row_idx.long()]).sum(1).to(psw.dtype) if need_dpsw else None
    return dW.to(weight.dtype), dpsw


def route_pack(indices, psw, shard_rows, world):
    B, L = indices.shape
    flat = indices.reshape(-1)
    owner = torch.div(flat, shard_rows, rounding_mode="floor")
    ok = (flat >= 0) & (owner < world)
    key = torch.where(ok, owner, torch.full_like(owner, world))
    order = torch.argsort(key, stable=True)
    send = torch.bincount(key, minlength=world + 1)[:world]
    local_row = torch.where(ok[order], flat[order] - key[order] * shard_rows, torch.zeros_like(flat)).to(torch.int32)
    bag = torch.div(order, L, rounding_mode="floor").to(torch.int32)
    weight = psw.reshape(-1)[order].float() if psw is not None else torch.ones(flat.numel())
    return send, order.to(torch.int32), local_row, bag, weight


def route_segments(bag, group_counts, groups):
    n = bag.numel()
    grp = torch.repeat_interleave(torch.arange(groups), group_counts.long().cpu())
    grp = torch.cat([grp, torch.full((max(0, n - grp.numel()),), groups, dtype=grp.dtype)])[:n]
    start = torch.ones(n, dtype=torch.bool)
    if n > 1:
        start[1:] = (bag[1:] != bag[:-1]) | (grp[1:] != grp[:-1])
    seg_of = (torch.cumsum(start.to(torch.int32), 0) - 1).to(torch.int32)
    first = torch.nonzero(start).reshape(-1)
    n_seg = first.numel()
    seg_start = torch.zeros(n + 1, dtype=torch.int64)
    seg_start[:n_seg] = first
    seg_start[n_seg] = n
    seg_bag = torch.zeros(n, dtype=torch.int32)
    seg_bag[:n_seg] = bag[first].to(torch.int32)
    seg_counts = torch.bincount(grp[first], minlength=groups + 1)[:groups]
    return seg_of, seg_start, seg_bag, seg_counts


def route_combine(partial, seg_bag, seg_counts, groups, n_bags, out_dtype=None):
    out = torch.zeros((n_bags, partial.shape[1]), dtype=torch.float32)
    pos = 0
    for g in range(groups):  # group order: the summation order
        c = int(seg_counts[g])
        out.index_add_(0, seg_bag[pos:pos + c].long(), partial[pos:pos + c].float())
        pos += c
    return out.to(out_dtype or partial.dtype)


def score_transform_fwd(scores, temperature, mode="softmax"):
    x = scores / temperature
    if mode == "softmax":
        return torch.softmax(x, dim=-1).type_as(scores)
    return (torch.nn.functional.silu(x) if mode == "silu" else torch.relu(x)).type_as(scores)


def score_transform_bwd(scores, out, grad_out, temperature, mode="softmax"):
    g = grad_out.to(out.dtype if mode == "softmax" else scores.dtype)
    if mode == "softmax":
        d = out * (g - (g * out).sum(-1, keepdim=True))
    else:
        x = scores / temperature
        if mode == "silu":
            s = torch.sigmoid(x)
            d = g * s * (1 + x * (1 - s))
        else:
            d = g * (x > 0).to(g.dtype)
    return d / temperature


def read_device_errors(dev=None, reset=True):
    return 0


def check_device_errors(dev=None):
    return None


def _kernel(f):
    """A stand-in for a CUDA kernel: its outputs carry no autograd graph (a
    kernel's never do), even when it is called inside a backward that runs
    with ``create_graph``."""
    @functools.wraps(f)
    def run(*args, **kwargs):
        with torch.no_grad():
            return f(*args, **kwargs)
    return run


for _name in ("bag_fwd", "bag_bwd", "bag_bwd2", "subkey_scores", "product_topk", "score_grad_dense", "fw_update",
              "fw_update_bwd", "swiglu_fwd", "swiglu_bwd", "colsum", "segment_sum", "bag_bwd_ragged", "route_pack",
              "route_segments", "route_combine", "score_transform_fwd", "score_transform_bwd"):
    globals()[_name] = _kernel(globals()[_name])


def install(monkeypatch):
    """Route ``modelos_b200._native`` calls to this module for one test."""
    from modelos_b200 import _native
    for name in ("bag_fwd", "bag_bwd", "bag_bwd2", "subkey_scores", "product_topk", "score_grad_dense",
                 "fw_update", "fw_update_bwd", "swiglu_fwd", "swiglu_bwd", "colsum", "segment_sum",
                 "bag_bwd_ragged", "route_pack", "route_segments", "route_combine", "score_transform_fwd",
                 "score_transform_bwd", "read_device_errors",
                 "check_device_errors"):
        monkeypatch.setattr(_native, name, globals()[name])
    return np
