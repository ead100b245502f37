"""SwiGLU output projection of HashingMemory (pkm/memory.py:226-229) on the
library's gate and column-sum kernels against torch's eager ops: outputs and
all gradients, fp32 (1e-5) and bf16 (2e-2)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
@pytest.mark.parametrize("n", [4096, 37])
def test_swiglu_projection(dtype, tol, n):
    from modelos_b200.pkm.memory import SwiGLUProjection
    g = torch.Generator(device=DEV).manual_seed(0)
    C, V, O = 256, 512, 256
    a0 = torch.randn(n, V, generator=g, device=DEV).to(dtype)
    x0 = torch.randn(n, C, generator=g, device=DEV).to(dtype)
    ws0 = (torch.randn(V, C, generator=g, device=DEV) * C ** -0.5).to(dtype)
    bs0 = (torch.randn(V, generator=g, device=DEV) * 0.1).to(dtype)
    wv0 = (torch.randn(O, V, generator=g, device=DEV) * V ** -0.5).to(dtype)
    bv0 = (torch.randn(O, generator=g, device=DEV) * 0.1).to(dtype)
    dy = torch.randn(n, O, generator=g, device=DEV).to(dtype)
    ours = [t.clone().requires_grad_() for t in (a0, x0, ws0, bs0, wv0, bv0)]
    ref = [t.clone().requires_grad_() for t in (a0, x0, ws0, bs0, wv0, bv0)]
    y = SwiGLUProjection.apply(*ours)
    a, x, ws, bs, wv, bv = ref
    yr = F.linear(a * F.silu(F.linear(x, ws, bs)), wv, bv)
    y.backward(dy)
    yr.backward(dy)
    assert rel(y, yr) < tol
    for o, r in zip(ours, ref):
        assert o.grad.dtype == dtype
        assert rel(o.grad, r.grad) < tol


def test_colsum_deterministic_and_exact_order_free():
    from modelos_b200 import _native
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(16384, 1024, generator=g, device=DEV).bfloat16()
    s1 = _native.colsum(x)
    s2 = _native.colsum(x)
    assert torch.equal(s1, s2)
    assert rel(s1, x.float().sum(0)) < 2e-2
    f = torch.randn(1000, 64, generator=g, device=DEV)
    assert rel(_native.colsum(f), f.double().sum(0)) < 1e-6


def test_gate_against_oracle():
    from modelos_b200 import _native
    from oracle import pkm_oracle as po
    g = torch.Generator().manual_seed(2)
    a = torch.randn(333, 64, generator=g)
    h = torch.randn(333, 64, generator=g) * 3
    dz = torch.randn(333, 64, generator=g)
    z = _native.swiglu_fwd(a.to(DEV), h.to(DEV))
    assert rel(z.cpu(), torch.from_numpy(po.swiglu(a.numpy(), h.numpy()))) < 1e-5
    da, dh, db = _native.swiglu_bwd(dz.to(DEV), a.to(DEV), h.to(DEV), bias_dtype=torch.float32)
    rda, rdh = po.swiglu_bwd(dz.numpy(), a.numpy(), h.numpy())
    assert rel(da.cpu(), torch.from_numpy(rda)) < 1e-5
    assert rel(dh.cpu(), torch.from_numpy(rdh)) < 1e-5
    assert rel(db.cpu(), torch.from_numpy(rdh.sum(0))) < 1e-5
