"""The oracle's restatements of the query batch norm, the SwiGLU gate, the
fast-weight value update and the ragged bag, pinned against the torch ops
the reference runs (nn.BatchNorm1d, F.silu, the update_fw sequence,
embedding-bag sums) on CPU."""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from oracle import pkm_oracle as po


def close(a, b, tol=1e-10):
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return np.abs(a - b).max() <= tol * max(np.abs(b).max(), 1e-30)


def test_batchnorm_train_eval_backward():
    g = torch.Generator().manual_seed(0)
    n, c = 300, 24
    x = (torch.randn(n, c, generator=g, dtype=torch.float64) * 2 + 1).requires_grad_()
    bn = torch.nn.BatchNorm1d(c, eps=1e-6, momentum=0.1).double()
    with torch.no_grad():
        bn.weight.copy_(torch.rand(c, generator=g, dtype=torch.float64) + 0.5)
        bn.bias.copy_(torch.randn(c, generator=g, dtype=torch.float64))
    rm0, rv0 = bn.running_mean.clone(), bn.running_var.clone()
    y = bn(x)
    dy = torch.randn(n, c, generator=g, dtype=torch.float64)
    y.backward(dy)
    out, mean, rstd, rm, rv = po.batchnorm_train(x.detach().numpy(), bn.weight.detach().numpy(),
                                                 bn.bias.detach().numpy(), rm0.numpy(), rv0.numpy(), 0.1, 1e-6)
    assert close(out, y.detach().numpy())
    assert close(rm, bn.running_mean.numpy()) and close(rv, bn.running_var.numpy())
    dx, dw, db = po.batchnorm_bwd(dy.numpy(), x.detach().numpy(), mean, rstd, bn.weight.detach().numpy())
    assert close(dx, x.grad.numpy(), 1e-9)
    assert close(dw, bn.weight.grad.numpy()) and close(db, bn.bias.grad.numpy())
    bn.eval()
    ye = bn(x.detach())
    assert close(po.batchnorm_eval(x.detach().numpy(), bn.weight.detach().numpy(), bn.bias.detach().numpy(),
                                   bn.running_mean.numpy(), bn.running_var.numpy(), 1e-6), ye.detach().numpy())


def test_swiglu_forward_backward():
    g = torch.Generator().manual_seed(1)
    a = torch.randn(50, 16, generator=g, dtype=torch.float64).requires_grad_()
    h = (torch.randn(50, 16, generator=g, dtype=torch.float64) * 3).requires_grad_()
    z = a * F.silu(h)
    dz = torch.randn(50, 16, generator=g, dtype=torch.float64)
    z.backward(dz)
    assert close(po.swiglu(a.detach().numpy(), h.detach().numpy()), z.detach().numpy())
    da, dh = po.swiglu_bwd(dz.numpy(), a.detach().numpy(), h.detach().numpy())
    assert close(da, a.grad.numpy()) and close(dh, h.grad.numpy())


def test_fw_value_update_with_clip():
    g = torch.Generator().manual_seed(2)
    K, D = 40, 8
    p = torch.randn(K, D, generator=g, dtype=torch.float64)
    grad = torch.randn(K, D, generator=g, dtype=torch.float64) * 1e-3
    idx = torch.randint(0, K // 2, (60,), generator=g)
    counts = torch.bincount(idx, minlength=K).to(torch.float64)
    c = torch.where(counts == 0, torch.ones_like(counts), counts)
    gs = grad * 1000 / c[:, None]
    ref = p - 0.1 * (torch.clamp(gs, -1, 1) + 0.01 * p)
    new, got_gs = po.fw_value_update(p.numpy(), grad.numpy(), counts.numpy(), 1000, 0.1, 0.01, clip=True)
    assert close(new, ref.numpy()) and close(got_gs, gs.numpy())


def test_ragged_bag_matches_dense_bag():
    g = torch.Generator().manual_seed(3)
    K, D = 30, 8
    W = torch.randn(K, D, generator=g, dtype=torch.float64)
    sizes = [3, 0, 5, 1]
    offsets = np.concatenate([[0], np.cumsum(sizes)])
    rows = torch.randint(0, K, (int(offsets[-1]),), generator=g)
    w = torch.rand(int(offsets[-1]), generator=g, dtype=torch.float64)
    out = po.segment_sum(W.numpy(), rows.numpy(), w.numpy(), offsets)
    for s in range(len(sizes)):
        e0, e1 = offsets[s], offsets[s + 1]
        ref = (W[rows[e0:e1]] * w[e0:e1, None]).sum(0)
        assert close(out[s], ref.numpy())
    # backward: entries of segment s read upstream row s
    src = np.repeat(np.arange(len(sizes)), sizes)
    gr = torch.randn(len(sizes), D, generator=g, dtype=torch.float64)
    dW, dpsw = po.bag_bwd_ragged(rows.numpy(), src, w.numpy(), W.numpy(), gr.numpy())
    Wt = W.clone().requires_grad_()
    wt = w.clone().requires_grad_()
    o = torch.zeros(len(sizes), D, dtype=torch.float64).index_add(0, torch.from_numpy(src),
                                                                 Wt[rows] * wt[:, None])
    o.backward(gr)
    assert close(dW, Wt.grad.numpy()) and close(dpsw, wt.grad.numpy())
