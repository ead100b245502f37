"""numpy restatement of one ``HashingMemory`` training step (forward + backward).

TEST INFRASTRUCTURE / CPU REFERENCE TIMING ONLY: used by ``bench.py`` for the timed
CPU baseline (``cpu_baseline`` and ``--impl reference``), never by the
product package.  It follows ``HashingMemory.forward`` (``pkm/memory.py:190-248``)
and the autograd of each step, with BLAS matmuls for the dense parts and the
reference's default layer options (query bias, BatchNorm or RMSNorm, SwiLU
value projection, no gating, no dropout), computing in float32 (numpy has no
bf16).  Loss is ``sum(out**2)``.
"""
from __future__ import annotations

import numpy as np


def _topk_rows(s: np.ndarray, k: int):
    """Top-k per row (score desc, index asc), via argpartition + sort."""
    part = np.argpartition(-s, k - 1, axis=1)[:, :k]
    vals = np.take_along_axis(s, part, axis=1)
    order = np.lexsort((part, -vals), axis=1)
    return np.take_along_axis(vals, order, axis=1), np.take_along_axis(part, order, axis=1)


def layer_step(P: dict, x: np.ndarray, heads: int, knn: int, norm: str = "bn", eps: float = 1e-6,
               chunk: int = 1024):
    """One forward + backward.  P holds float32 parameters named as the
    module's state dict.  Returns (loss, grads dict)."""
    f32 = np.float32
    C = x.shape[-1]
    X = x.reshape(-1, C).astype(f32)
    N = X.shape[0]
    Wq, bq = P["query_proj.query_mlps.0.weight"], P["query_proj.query_mlps.0.bias"]
    keys = P["keys"]
    W = P["values.weight"]
    half = keys.shape[1]
    kd = 2 * half
    n = keys.shape[0] // (2 * heads)
    D = W.shape[1]
    # ---- forward ----
    Q = X @ Wq.T + bq
    gamma = P["query_proj.norm.weight"]
    if norm == "bn":
        mu = Q.mean(0)
        xc = Q - mu
        var = (xc * xc).mean(0)
        rstd = 1.0 / np.sqrt(var + eps)
        xh = xc * rstd
        Qn = xh * gamma + P["query_proj.norm.bias"]
    else:
        ms = (Q * Q).mean(1, keepdims=True)
        rstd = 1.0 / np.sqrt(ms + eps)
        xh = Q * rstd
        Qn = xh * gamma
    q = Qn.reshape(N, heads, 2, half)
    kv = keys.reshape(heads, 2, n, half)
    idx = np.empty((N, heads, knn), np.int64)
    sc = np.empty((N, heads, knn), f32)
    for h in range(heads):
        s1, i1 = _topk_rows(q[:, h, 0] @ kv[h, 0].T, knn)
        s2, i2 = _topk_rows(q[:, h, 1] @ kv[h, 1].T, knn)
        cs = (s1[:, :, None] + s2[:, None, :]).reshape(N, -1)
        cid = (i1[:, :, None] * n + i2[:, None, :]).reshape(N, -1)
        v, pos = _topk_rows(cs, knn)
        sc[:, h] = v
        idx[:, h] = np.take_along_axis(cid, pos, axis=1)
    e = np.exp(sc - sc.max(-1, keepdims=True))
    psw = (e / e.sum(-1, keepdims=True)).reshape(N, heads * knn).astype(f32)
    I = idx.reshape(N, heads * knn)
    bag = np.empty((N, D), f32)
    for s in range(0, N, chunk):
        bag[s:s + chunk] = np.einsum("bl,bld->bd", psw[s:s + chunk], W[I[s:s + chunk]])
    Ws, bs = P["swilu_projection.weight"], P["swilu_projection.bias"]
    Wv, bv = P["value_proj.weight"], P["value_proj.bias"]
    hs = X @ Ws.T + bs
    sig = 1.0 / (1.0 + np.exp(-hs))
    gate = hs * sig
    u = bag * gate
    out = u @ Wv.T + bv
    loss = float((out.astype(np.float64) ** 2).sum())
    # ---- backward ----
    G = {}
    dout = 2.0 * out
    G["value_proj.weight"] = dout.T @ u
    G["value_proj.bias"] = dout.sum(0)
    du = dout @ Wv
    dbag = du * gate
    dhs = du * bag * (sig * (1.0 + hs * (1.0 - sig)))
    G["swilu_projection.weight"] = dhs.T @ X
    G["swilu_projection.bias"] = dhs.sum(0)
    dX = dhs @ Ws
    # bag backward: dense dW, per-sample gradient
    dW = np.zeros_like(W)
    dpsw = np.empty_like(psw)
    for s in range(0, N, chunk):
        Ic = I[s:s + chunk]
        dpsw[s:s + chunk] = np.einsum("bld,bd->bl", W[Ic], dbag[s:s + chunk])
        flat = Ic.reshape(-1)
        order = np.argsort(flat, kind="stable")
        fs = flat[order]
        st = np.flatnonzero(np.r_[True, fs[1:] != fs[:-1]])
        contrib = (psw[s:s + chunk, :, None] * dbag[s:s + chunk, None, :]).reshape(-1, D)[order]
        dW[fs[st]] += np.add.reduceat(contrib, st, axis=0)
    G["values.weight"] = dW
    # softmax backward per head
    p3 = psw.reshape(N, heads, knn)
    g3 = dpsw.reshape(N, heads, knn)
    ds = p3 * (g3 - (p3 * g3).sum(-1, keepdims=True))
    # scores backward through the selected sub-keys
    dq = np.zeros((N, heads, 2, half), f32)
    dkeys = np.zeros_like(kv)
    for h in range(heads):
        a = idx[:, h] // n
        b = idx[:, h] % n
        dsh = ds[:, h]
        dq[:, h, 0] = np.einsum("bk,bkd->bd", dsh, kv[h, 0][a])
        dq[:, h, 1] = np.einsum("bk,bkd->bd", dsh, kv[h, 1][b])
        np.add.at(dkeys[h, 0], a.reshape(-1), (dsh[:, :, None] * q[:, h, 0][:, None, :]).reshape(-1, half))
        np.add.at(dkeys[h, 1], b.reshape(-1), (dsh[:, :, None] * q[:, h, 1][:, None, :]).reshape(-1, half))
    G["keys"] = dkeys.reshape(keys.shape)
    dQn = dq.reshape(N, heads * kd)
    G["query_proj.norm.weight"] = (dQn * xh).sum(0)
    dxh = dQn * gamma
    if norm == "bn":
        G["query_proj.norm.bias"] = dQn.sum(0)
        dQ = rstd * (dxh - dxh.mean(0) - xh * (dxh * xh).mean(0))
    else:
        dQ = rstd * (dxh - xh * (dxh * xh).mean(1, keepdims=True))
    G["query_proj.query_mlps.0.weight"] = dQ.T @ X
    G["query_proj.query_mlps.0.bias"] = dQ.sum(0)
    dX += dQ @ Wq
    G["x"] = dX.reshape(x.shape)
    return loss, G


def make_params(cfg: dict, seed: int = 0) -> dict:
    """float32 parameters for ``layer_step`` (same init as the tests' cases)."""
    rng = np.random.default_rng(seed)
    C, O, kd, H, n = cfg["input_dim"], cfg["output_dim"], cfg["mem_k_dim"], cfg["mem_heads"], cfg["mem_n_keys"]
    v = cfg.get("mem_v_dim", O)
    f = np.float32
    P = {
        "keys": rng.uniform(-1, 1, (2 * H * n, kd // 2)).astype(f) / np.sqrt(kd).astype(f),
        "values.weight": (rng.standard_normal((n * n, v), dtype=f) * f(v ** -0.5)),
        "value_proj.weight": rng.standard_normal((O, v), dtype=f) * f(O ** -0.5),
        "value_proj.bias": rng.uniform(-1, 1, O).astype(f) / f(np.sqrt(v)),
        "swilu_projection.weight": rng.standard_normal((v, C), dtype=f) * f(O ** -0.5),
        "swilu_projection.bias": rng.uniform(-1, 1, v).astype(f) / f(np.sqrt(C)),
        "query_proj.query_mlps.0.weight": rng.uniform(-1, 1, (H * kd, C)).astype(f) / f(np.sqrt(C)),
        "query_proj.query_mlps.0.bias": rng.uniform(-1, 1, H * kd).astype(f) / f(np.sqrt(C)),
        "query_proj.norm.weight": np.ones(H * kd, f),
        "query_proj.norm.bias": np.zeros(H * kd, f),
    }
    return P
