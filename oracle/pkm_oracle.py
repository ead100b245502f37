"""CPU oracle for the product-key-memory hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``modelos_b200`` imports this module;
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` use it, and only as the checker or
as the timed CPU baseline.  It is a numpy restatement of the reference
algorithm (APamplonat/Modelos, files cited per function) with every rounding
step written out, so that the CUDA kernels can be checked bit-for-bit where
the contract asks for it (top-k indices) and within a stated tolerance
elsewhere (fp32 1e-5 relative, bf16 2e-2).

Parity pin: ``tests/golden/*.npz`` hold outputs of the reference's own
PyTorch code (imported from the reference tree by
``tests/golden/make_golden.py``) on seeded inputs, and
``tests/test_oracle_golden.py`` checks this oracle against them.

Arithmetic definitions (these are the contract the kernels follow):

* Sub-key dot scores (``pkm/memory.py:267-268``, ``fwpkm/fwpkm.py:861``):
  ``acc = 0; for c in 0..half-1: acc = fl32(acc + fl32(q[c] * k[c]))``,
  i.e. a sequential fp32 sum with no fused multiply-add, then rounded to the
  score dtype (bf16 round-to-nearest-even when the query is bf16).
* idw scores (``fwpkm/fwpkm.py:862-866``, torch ``cdist`` with
  ``use_mm_for_euclid_dist``): ``r = fl32(fl32(qq - 2*qk) + kk)`` with the
  three sums sequential as above, ``r = max(r, 1e-30)``, ``d = sqrt(r)``,
  ``t = fl32(1e-3 + fl32(d*d))``, ``score = -fl32(log_f64(t))``.
* Top-k order everywhere: score descending, ties broken by the lowest index
  (sub-key index in stage 1, memory slot ``i1*n + i2`` in stage 2).  The
  reference's ``torch.topk`` leaves tie order implementation-defined; this
  rule is the build's definition and the golden comparisons are tie-aware.
* Cartesian sums (``pkm/memory.py:274-277``): ``fl32(s1 + s2)`` rounded to
  the score dtype.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "bf16_round",
    "subkey_scores",
    "topk_canonical",
    "product_topk",
    "softmax_rows",
    "pkm_get_indices",
    "bag_fwd",
    "bag_bwd",
    "bag_bwd2",
    "bincount",
    "fw_value_update",
    "marginal_entropy",
    "batchnorm_train",
    "batchnorm_bwd",
    "batchnorm_eval",
    "swiglu",
    "swiglu_bwd",
    "segment_sum",
    "bag_bwd_ragged",
    "addr_stats",
]


# --------------------------------------------------------------------------
# dtype helpers
# --------------------------------------------------------------------------
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even).

    Returns float32 values that are exactly representable in bf16, which is
    what torch's ``.to(torch.bfloat16)`` produces for finite inputs.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    bias = np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))
    r = ((u + bias) & np.uint64(0xFFFF0000)).astype(np.uint32)
    return r.view(np.float32)


def _round_to(x: np.ndarray, bf16: bool) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return bf16_round(x) if bf16 else x


# --------------------------------------------------------------------------
# K1: sub-key scores
# --------------------------------------------------------------------------
def _seq_dot(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Sequential fp32 dot products ``a[i] . b[j]`` for all i, j.

    a: [M, C] float32, b: [N, C] float32 -> [M, N] float32, summed in
    ascending c with every product and every partial sum rounded to fp32.
    """
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    acc = np.zeros((a.shape[0], b.shape[0]), dtype=np.float32)
    for c in range(a.shape[1]):
        acc += np.multiply.outer(a[:, c], b[:, c])  # fp32 product, fp32 add
    return acc


def _seq_sqnorm(a: np.ndarray) -> np.ndarray:
    a = np.asarray(a, dtype=np.float32)
    acc = np.zeros(a.shape[0], dtype=np.float32)
    for c in range(a.shape[1]):
        acc += a[:, c] * a[:, c]
    return acc


def subkey_scores(query: np.ndarray, keys: np.ndarray, heads: int, mode: str = "dot",
                  bf16: bool = False) -> np.ndarray:
    """All sub-key scores for both halves.

    Follows ``HashingMemory.get_indices`` (``pkm/memory.py:250-268``) and
    ``FastWeightProductKeyMemory.compute_qk_scores`` (``fwpkm/fwpkm.py:853-869``).

    query: [N*H, k_dim] (row = token*H + head); keys: [2*H*n, k_dim/2] viewed
    as (H, 2, n, half).  Returns scores [N*H, 2, n] float32 (bf16-rounded
    values when ``bf16``).
    """
    query = np.asarray(query, dtype=np.float32)
    keys = np.asarray(keys, dtype=np.float32)
    NH, kd = query.shape
    half = kd // 2
    n = keys.shape[0] // (2 * heads)
    assert keys.shape == (2 * heads * n, half)
    N = NH // heads
    q = query.reshape(N, heads, 2, half)
    kv = keys.reshape(heads, 2, n, half)
    out = np.empty((N, heads, 2, n), dtype=np.float32)
    for h in range(heads):
        for p in range(2):
            qa = q[:, h, p, :]
            kb = kv[h, p]
            if mode == "dot":
                s = _seq_dot(qa, kb)
            elif mode in ("idw", "dist"):
                qk = _seq_dot(qa, kb)
                qq = _seq_sqnorm(qa)
                kk = _seq_sqnorm(kb)
                r = (qq[:, None] - np.float32(2.0) * qk) + kk[None, :]
                r = np.maximum(r, np.float32(1e-30))
                d = np.sqrt(r)
                if mode == "dist":
                    s = d
                else:
                    t = np.float32(1e-3) + d * d
                    s = -(np.log(t.astype(np.float64)).astype(np.float32))
            else:
                raise ValueError(mode)
            out[:, h, p, :] = _round_to(s, bf16)
    return out.reshape(NH, 2, n)


# --------------------------------------------------------------------------
# K2: product top-k
# --------------------------------------------------------------------------
def topk_canonical(scores: np.ndarray, k: int, ids: np.ndarray | None = None):
    """Top-k along the last axis: score descending, then id ascending.

    ``ids`` defaults to the position along the axis.  Returns (values, ids).
    """
    scores = np.asarray(scores, dtype=np.float32)
    if ids is None:
        ids = np.broadcast_to(np.arange(scores.shape[-1], dtype=np.int64), scores.shape)
    flat_s = scores.reshape(-1, scores.shape[-1])
    flat_i = np.asarray(ids, dtype=np.int64).reshape(-1, scores.shape[-1])
    order = np.lexsort((flat_i, -flat_s.astype(np.float64)), axis=-1)[:, :k]
    vals = np.take_along_axis(flat_s, order, axis=-1)
    sel = np.take_along_axis(flat_i, order, axis=-1)
    shp = scores.shape[:-1] + (k,)
    return vals.reshape(shp), sel.reshape(shp)


def product_topk(scores: np.ndarray, knn: int, bf16: bool = False):
    """Dual top-k, cartesian product, second top-k.

    Follows ``pkm/memory.py:270-285`` and ``fwpkm/fwpkm.py:908-923``.
    scores: [R, 2, n].  Returns dict with ``scores`` [R, knn], ``indices``
    [R, knn] (slot = i1*n + i2), ``sub_indices1/2`` [R, knn] (stage-1 lists,
    sorted), ``sub_scores1/2``.
    """
    scores = np.asarray(scores, dtype=np.float32)
    R, two, n = scores.shape
    assert two == 2
    v1, i1 = topk_canonical(scores[:, 0, :], knn)
    v2, i2 = topk_canonical(scores[:, 1, :], knn)
    cand = _round_to(v1[:, :, None] + v2[:, None, :], bf16).reshape(R, knn * knn)
    slots = (i1[:, :, None] * n + i2[:, None, :]).reshape(R, knn * knn)
    best, best_slots = topk_canonical(cand, knn, ids=slots)
    return {
        "scores": best,
        "indices": best_slots,
        "sub_indices1": i1,
        "sub_indices2": i2,
        "sub_scores1": v1,
        "sub_scores2": v2,
    }


def softmax_rows(x: np.ndarray, bf16: bool = False) -> np.ndarray:
    """Softmax over the last axis in float64, returned as fp32 (bf16-rounded).

    Mirrors ``F.softmax(scores.float(), dim=-1).type_as(scores)``
    (``pkm/memory.py:218``, ``fwpkm/fwpkm.py:108``).
    """
    x = np.asarray(x, dtype=np.float64)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    p = (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
    return _round_to(p, bf16)


def pkm_get_indices(query, keys, heads, knn, mode="dot", bf16=False):
    """``HashingMemory.get_indices`` (``pkm/memory.py:250-289``)."""
    s = subkey_scores(query, keys, heads, mode=mode, bf16=bf16)
    res = product_topk(s, knn, bf16=bf16)
    res["all_scores"] = s
    return res


# --------------------------------------------------------------------------
# K3 / K4 / K5: embedding bag
# --------------------------------------------------------------------------
def bag_fwd(indices, psw, weight, chunk: int = 4096) -> np.ndarray:
    """``out[b] = sum_j psw[b,j] * W[idx[b,j]]`` in float64.

    Follows ``embedding_bag_k`` (``pkm/xformer_embeddingbag.py:97-113``) and
    the fwpkm gather (``fwpkm/xformer_embeddingbag_grad_wrapper.py:99-103``).
    """
    indices = np.asarray(indices, dtype=np.int64)
    psw = np.asarray(psw, dtype=np.float64)
    W = np.asarray(weight)
    B, L = indices.shape
    out = np.empty((B, W.shape[1]), dtype=np.float64)
    for s in range(0, B, chunk):
        e = min(B, s + chunk)
        rows = W[indices[s:e]].astype(np.float64)  # [b, L, D]
        out[s:e] = np.einsum("bl,bld->bd", psw[s:e], rows)
    return out


def bag_bwd(indices, psw, weight, grad_out, chunk: int = 4096):
    """First-order backward of the weighted embedding bag, float64.

    ``dW[k] = sum_{(b,j): idx=k} psw[b,j] * g[b]`` (dense, zero for untouched
    rows) and ``dPsw[b,j] = <W[idx[b,j]], g[b]>``.  Follows
    ``aggregate_gradient_for_embedding_k`` (``pkm/xformer_embeddingbag.py:291-328``)
    and ``_embedding_bag_bw_native`` (``fwpkm/xformer_embeddingbag_legacy.py:147-167``).
    """
    indices = np.asarray(indices, dtype=np.int64)
    psw = np.asarray(psw, dtype=np.float64)
    W = np.asarray(weight)
    g = np.asarray(grad_out, dtype=np.float64)
    B, L = indices.shape
    K, D = W.shape
    dW = np.zeros((K, D), dtype=np.float64)
    dpsw = np.empty((B, L), dtype=np.float64)
    for s in range(0, B, chunk):
        e = min(B, s + chunk)
        rows = W[indices[s:e]].astype(np.float64)
        dpsw[s:e] = np.einsum("bld,bd->bl", rows, g[s:e])
        flat = indices[s:e].reshape(-1)
        if flat.size == 0:
            continue
        order = np.argsort(flat, kind="stable")
        fs = flat[order]
        starts = np.flatnonzero(np.r_[True, fs[1:] != fs[:-1]])
        contrib = (psw[s:e, :, None] * g[s:e, None, :]).reshape(-1, D)[order]
        dW[fs[starts]] += np.add.reduceat(contrib, starts, axis=0)
    return dW, dpsw


def bag_bwd2(indices, a, gbar, g, chunk: int = 4096):
    """Double-backward VJP of the bag's weight gradient, float64.

    ``dG[b] = sum_j a[b,j] * gbar[idx[b,j]]`` and
    ``da[b,j] = <gbar[idx[b,j]], g[b]>``; follows ``EmbeddingBagBW.backward``
    (``fwpkm/xformer_embeddingbag_grad_wrapper.py:43-74``).
    """
    dG = bag_fwd(indices, a, gbar, chunk=chunk)
    indices = np.asarray(indices, dtype=np.int64)
    g = np.asarray(g, dtype=np.float64)
    gb = np.asarray(gbar)
    B, L = indices.shape
    da = np.empty((B, L), dtype=np.float64)
    for s in range(0, B, chunk):
        e = min(B, s + chunk)
        rows = gb[indices[s:e]].astype(np.float64)
        da[s:e] = np.einsum("bld,bd->bl", rows, g[s:e])
    return dG, da


def bincount(indices, K: int) -> np.ndarray:
    """Occurrences of each slot (``fwpkm/fwpkm.py:343``)."""
    return np.bincount(np.asarray(indices, dtype=np.int64).reshape(-1), minlength=K)


def fw_value_update(p, g, counts, scale, lr, wd, clip: bool = False):
    """Fast-weight value update of ``update_fw`` (``fwpkm/fwpkm.py:333-365``)
    and ``update_fw_param`` (``:266-272``).

    ``g' = g * scale / max(count, 1)``; ``u = clamp(g', -1, 1)`` when
    ``clip`` (``grad_clip``), else ``g'``; ``p' = p - lr * (u + wd * p)``,
    float64.  Returns (p', g').
    """
    p = np.asarray(p, dtype=np.float64)
    g = np.asarray(g, dtype=np.float64)
    c = np.maximum(np.asarray(counts, dtype=np.float64), 1.0)
    gs = g * scale / c[:, None]
    u = np.clip(gs, -1.0, 1.0) if clip else gs
    return p - lr * (u + wd * p), gs


# --------------------------------------------------------------------------
# query batch norm (pkm/memory.py:308-309: nn.BatchNorm1d(heads * k_dim,
# eps=1e-6, momentum=0.1) on the [n, c] query projection)
# --------------------------------------------------------------------------
def batchnorm_train(x, weight, bias, running_mean, running_var, momentum: float, eps: float):
    """Training forward in float64: batch mean and biased variance normalise,
    the running statistics move by ``momentum`` with the unbiased variance.
    Returns (out, mean, rstd, new_running_mean, new_running_var)."""
    x = np.asarray(x, dtype=np.float64)
    n = x.shape[0]
    mean = x.mean(axis=0)
    var = ((x - mean) ** 2).mean(axis=0)
    rstd = 1.0 / np.sqrt(var + eps)
    out = (x - mean) * rstd
    if weight is not None:
        out = out * np.asarray(weight, dtype=np.float64)
    if bias is not None:
        out = out + np.asarray(bias, dtype=np.float64)
    unbiased = var * n / max(n - 1, 1)
    rm = (1 - momentum) * np.asarray(running_mean, dtype=np.float64) + momentum * mean
    rv = (1 - momentum) * np.asarray(running_var, dtype=np.float64) + momentum * unbiased
    return out, mean, rstd, rm, rv


def batchnorm_bwd(dy, x, mean, rstd, weight):
    """Training backward in float64: (dx, dweight, dbias)."""
    dy = np.asarray(dy, dtype=np.float64)
    x = np.asarray(x, dtype=np.float64)
    n = x.shape[0]
    xhat = (x - mean) * rstd
    w = np.ones_like(mean) if weight is None else np.asarray(weight, dtype=np.float64)
    db = dy.sum(axis=0)
    dw = (dy * xhat).sum(axis=0)
    dx = w * rstd * (dy - db / n - xhat * dw / n)
    return dx, dw, db


def batchnorm_eval(x, weight, bias, running_mean, running_var, eps: float):
    """Evaluation forward in float64 with the running statistics."""
    x = np.asarray(x, dtype=np.float64)
    out = (x - running_mean) / np.sqrt(np.asarray(running_var, dtype=np.float64) + eps)
    if weight is not None:
        out = out * weight
    if bias is not None:
        out = out + bias
    return out


# --------------------------------------------------------------------------
# SwiGLU gate of the memory output (pkm/memory.py:226-229:
# value_proj(output * F.silu(swilu_projection(input))))
# --------------------------------------------------------------------------
def swiglu(a, h):
    """``a * silu(h)``, silu(h) = h / (1 + exp(-h)), float64."""
    a = np.asarray(a, dtype=np.float64)
    h = np.asarray(h, dtype=np.float64)
    return a * h / (1.0 + np.exp(-h))


def swiglu_bwd(dz, a, h):
    """(da, dh) of ``swiglu``: da = dz * silu(h), dh = dz * a * silu'(h),
    silu'(h) = sig * (1 + h * (1 - sig)), float64."""
    dz = np.asarray(dz, dtype=np.float64)
    a = np.asarray(a, dtype=np.float64)
    h = np.asarray(h, dtype=np.float64)
    sig = 1.0 / (1.0 + np.exp(-h))
    return dz * h * sig, dz * a * sig * (1.0 + h * (1.0 - sig))


# --------------------------------------------------------------------------
# ragged bags (one rank's shard of a row-sharded table)
# --------------------------------------------------------------------------
def segment_sum(rows, entry_row, entry_w, offsets):
    """``out[s] = sum_{e in [offsets[s], offsets[s+1])} w[e] * rows[row[e]]``:
    the bag forward (``pkm/xformer_embeddingbag.py:97-138``) over bags of
    different sizes, float64."""
    rows = np.asarray(rows, dtype=np.float64)
    offsets = np.asarray(offsets, dtype=np.int64)
    out = np.zeros((len(offsets) - 1, rows.shape[1]))
    for s in range(len(offsets) - 1):
        e0, e1 = offsets[s], offsets[s + 1]
        if e1 > e0:
            out[s] = (np.asarray(entry_w[e0:e1], dtype=np.float64)[:, None] * rows[entry_row[e0:e1]]).sum(0)
    return out


def bag_bwd_ragged(row_idx, src_of, psw, weight, grad_rows):
    """The bag backward (``pkm/xformer_embeddingbag.py:331-386``) where entry e
    reads upstream row ``src_of[e]``: (dW, dpsw), float64."""
    weight = np.asarray(weight, dtype=np.float64)
    g = np.asarray(grad_rows, dtype=np.float64)[np.asarray(src_of)]
    w = np.asarray(psw, dtype=np.float64)
    dW = np.zeros_like(weight)
    np.add.at(dW, np.asarray(row_idx), g * w[:, None])
    dpsw = (g * weight[np.asarray(row_idx)]).sum(1)
    return dW, dpsw


def marginal_entropy(M, topk: int, eps: float = 1e-8) -> float:
    """``compute_marginal_entropy`` (``fwpkm/fwpkm.py:117-147``), float64."""
    M = np.asarray(M, dtype=np.float64)
    thr = -np.sort(-M, axis=1)[:, topk - 1:topk]
    Mm = np.where(M >= thr, M, -np.inf)
    mx = Mm.max(axis=1, keepdims=True)
    e = np.exp(Mm - mx)
    P = e / e.sum(axis=1, keepdims=True)
    Pbar = P.mean(axis=0)
    return float(-(Pbar * np.log(Pbar + eps)).sum())


def addr_stats(indices, K: int) -> dict:
    """``compute_addr_stats`` (``modeling_qwen3pkm.py:454-463``), float64.

    The histogram's KL divergence from the uniform distribution follows
    torch.distributions' categorical KL: ``sum p*(log c(p) - log c(q))`` over
    the slots with ``p > 0``, ``c`` clamping to ``[eps, 1 - eps]`` with
    ``eps`` the fp32 machine epsilon (the probabilities are fp32 there).
    """
    idx = np.asarray(indices, dtype=np.int64).reshape(-1)
    c = np.bincount(idx, minlength=K).astype(np.int64)
    S = int(c.sum())
    eps = float(np.finfo(np.float32).eps)
    p = c / S
    lq = np.log(np.clip(1.0 / K, eps, 1 - eps))
    nz = c > 0
    kld = float((p[nz] * (np.log(np.clip(p[nz], eps, 1 - eps)) - lq)).sum())
    return {
        "collision_ratio": int(c[c > 1].sum()) / (idx.size + 1e-6),
        "coverage_ratio": int(nz.sum()) / K,
        "kld": kld,
    }
