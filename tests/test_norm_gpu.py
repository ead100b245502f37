"""Query batch normalisation kernels against torch's nn.BatchNorm1d (the
reference's query norm, pkm/memory.py:308-309): outputs, running statistics
and gradients, training and evaluation, in fp32 (1e-5) and bf16 (2e-2)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def pair(c, momentum=0.1, dtype=torch.float32, seed=0):
    from modelos_b200.pkm.memory import QueryBatchNorm
    g = torch.Generator().manual_seed(seed)
    ref = torch.nn.BatchNorm1d(c, eps=1e-6, momentum=momentum)
    with torch.no_grad():
        ref.weight.copy_(torch.randn(c, generator=g) * 0.5 + 1.0)
        ref.bias.copy_(torch.randn(c, generator=g) * 0.1)
        ref.running_mean.copy_(torch.randn(c, generator=g))
        ref.running_var.copy_(torch.rand(c, generator=g) + 0.5)
    ours = QueryBatchNorm(c, eps=1e-6, momentum=momentum)
    ours.load_state_dict(ref.state_dict())
    return ref.to(DEV), ours.to(DEV, dtype)


@pytest.mark.parametrize("n,c,momentum", [(4096, 2048, 0.1), (3, 8, 0.1), (1000, 264, None)])
def test_train_fp32(n, c, momentum):
    ref, ours = pair(c, momentum)
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(n, c, generator=g) * 2 + 3).to(DEV)
    dy = torch.randn(n, c, generator=g).to(DEV)
    for _ in range(2):  # two steps: running statistics and the counter
        xr = x.clone().requires_grad_()
        xo = x.clone().requires_grad_()
        yr = ref(xr)
        yo = ours(xo)
        yr.backward(dy)
        yo.backward(dy)
    assert rel(yo, yr) < 1e-5
    assert rel(xo.grad, xr.grad) < 1e-5
    assert rel(ours.weight.grad, ref.weight.grad) < 1e-5
    assert rel(ours.bias.grad, ref.bias.grad) < 1e-5
    assert rel(ours.running_mean, ref.running_mean) < 1e-5
    assert rel(ours.running_var, ref.running_var) < 1e-5
    assert int(ours.num_batches_tracked) == int(ref.num_batches_tracked) == 2


def test_eval_fp32():
    ref, ours = pair(520)
    ref.eval()
    ours.eval()
    g = torch.Generator().manual_seed(2)
    x = torch.randn(777, 520, generator=g).to(DEV)
    dy = torch.randn(777, 520, generator=g).to(DEV)
    xr = x.clone().requires_grad_()
    xo = x.clone().requires_grad_()
    yr, yo = ref(xr), ours(xo)
    yr.backward(dy)
    yo.backward(dy)
    assert rel(yo, yr) < 1e-5
    assert rel(xo.grad, xr.grad) < 1e-5
    assert rel(ours.weight.grad, ref.weight.grad) < 1e-5
    assert rel(ours.bias.grad, ref.bias.grad) < 1e-5


def test_train_bf16_config2_shape():
    ref, ours = pair(2048, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(16384, 2048, generator=g) * 0.7 + 0.2).bfloat16().to(DEV)
    dy = torch.randn(16384, 2048, generator=g).bfloat16().to(DEV)
    xr = x.float().requires_grad_()
    xo = x.clone().requires_grad_()
    yr = ref(xr)
    yo = ours(xo)
    yr.backward(dy.float())
    yo.backward(dy)
    assert yo.dtype == torch.bfloat16 and xo.grad.dtype == torch.bfloat16
    assert rel(yo, yr) < 2e-2
    assert rel(xo.grad, xr.grad) < 2e-2
    assert rel(ours.weight.grad, ref.weight.grad) < 2e-2
    assert rel(ours.bias.grad, ref.bias.grad) < 2e-2
    assert rel(ours.running_mean, ref.running_mean) < 2e-2
    assert rel(ours.running_var, ref.running_var) < 2e-2


def test_deterministic():
    _, ours = pair(2048, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(8192, 2048, generator=g).bfloat16().to(DEV)
    dy = torch.randn(8192, 2048, generator=g).bfloat16().to(DEV)
    outs = []
    for _ in range(2):
        xo = x.clone().requires_grad_()
        y = ours(xo)
        y.backward(dy)
        outs.append((y, xo.grad, ours.weight.grad.clone()))
        ours.weight.grad = None
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_against_oracle():
    """fp32 kernels against the oracle's float64 restatement."""
    import numpy as np

    from modelos_b200 import _native
    from oracle import pkm_oracle as po
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2000, 64, generator=g) * 3 + 2
    w = torch.rand(64, generator=g) + 0.5
    b = torch.randn(64, generator=g)
    rm, rv = torch.zeros(64), torch.ones(64)
    dy = torch.randn(2000, 64, generator=g)
    xd, wd, bd, rmd, rvd = (t.to(DEV) for t in (x, w, b, rm, rv))
    out, mean, rstd = _native.batchnorm_fwd(xd, wd, bd, rmd, rvd, True, 0.1, 1e-6)
    ro, rmean, rrstd, rrm, rrv = po.batchnorm_train(x.numpy(), w.numpy(), b.numpy(), rm.numpy(), rv.numpy(), 0.1,
                                                    1e-6)
    assert rel(out.cpu(), torch.from_numpy(ro)) < 1e-5
    assert rel(rmd.cpu(), torch.from_numpy(rrm)) < 1e-5 and rel(rvd.cpu(), torch.from_numpy(rrv)) < 1e-5
    dx, dw, db = _native.batchnorm_bwd(dy.to(DEV), xd, mean, rstd, wd)
    rdx, rdw, rdb = po.batchnorm_bwd(dy.numpy(), x.numpy(), rmean, rrstd, w.numpy())
    for a, r in ((dx, rdx), (dw, rdw), (db, rdb)):
        assert rel(a.cpu(), torch.from_numpy(np.asarray(r))) < 1e-5
