"""Fused FwPKM value update (update_fw's value branch, fwpkm/fwpkm.py:274-367)
against the reference's torch sequence: bit-exact forward in fp32 and bf16,
backward against torch autograd."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def reference(values, grad, indices, scale, lr, wd, clip):
    counts = torch.bincount(indices.reshape(-1), minlength=values.shape[0]).to(grad.dtype)
    counts = torch.where(counts == 0, torch.ones_like(counts), counts)
    g = grad * scale
    scaled = g / counts.unsqueeze(-1)
    u = torch.clamp(scaled, min=-1.0, max=1.0) if clip else scaled
    return values - lr * (u + wd * values), scaled


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("clip,wd", [(True, 0.0), (False, 0.01), (True, 0.1)])
def test_forward_bit_exact(dtype, clip, wd):
    from modelos_b200 import _native
    g = torch.Generator(device=DEV).manual_seed(0)
    K, D = 4096, 256
    values = torch.randn(K, D, generator=g, device=DEV).to(dtype)
    grad = (torch.randn(K, D, generator=g, device=DEV) * 1e-7).to(dtype)
    indices = torch.randint(0, K // 2, (512, 4, 32), generator=g, device=DEV)  # half the rows unread
    scale = 512 * 1024 * 32 * 4
    new, scaled, counts = _native.fw_update(values, grad, indices, scale, 0.1, wd, clip)
    ref_new, ref_scaled = reference(values, grad, indices, scale, 0.1, wd, clip)
    assert torch.equal(counts.long(), torch.bincount(indices.reshape(-1), minlength=K))
    assert torch.equal(scaled, ref_scaled)
    assert torch.equal(new, ref_new)


@pytest.mark.parametrize("clip", [True, False])
def test_backward_matches_autograd(clip):
    from modelos_b200.fwpkm.fwpkm import FusedValueUpdate
    g = torch.Generator(device=DEV).manual_seed(1)
    K, D = 2048, 128
    v0 = torch.randn(K, D, generator=g, device=DEV)
    g0 = torch.randn(K, D, generator=g, device=DEV) * 2e-7
    indices = torch.randint(0, K, (256, 4, 16), generator=g, device=DEV)
    scale, lr, wd = 256 * 128 * 16 * 4, 0.1, 0.05
    w1 = torch.randn(K, D, generator=g, device=DEV)
    w2 = torch.randn(K, D, generator=g, device=DEV)
    v, gr = v0.clone().requires_grad_(), g0.clone().requires_grad_()
    new, scaled = FusedValueUpdate.apply(v, gr, indices, scale, lr, wd, clip)
    ((new * w1).sum() + (scaled * w2).sum()).backward()
    vr, grr = v0.clone().requires_grad_(), g0.clone().requires_grad_()
    rn, rs = reference(vr, grr, indices, scale, lr, wd, clip)
    ((rn * w1).sum() + (rs * w2).sum()).backward()
    for a, b in ((v.grad, vr.grad), (gr.grad, grr.grad)):
        assert ((a - b).abs().max() / b.abs().max()).item() < 1e-6


def test_against_oracle():
    from modelos_b200 import _native
    from oracle import pkm_oracle as po
    g = torch.Generator().manual_seed(3)
    K, D = 1000, 64
    values = torch.randn(K, D, generator=g)
    grad = torch.randn(K, D, generator=g) * 1e-6
    indices = torch.randint(0, K, (64, 4, 8), generator=g)
    new, scaled, counts = _native.fw_update(values.to(DEV), grad.to(DEV), indices.to(DEV), 65536, 0.1, 0.02, True)
    rnew, rs = po.fw_value_update(values.numpy(), grad.numpy(), counts.cpu().numpy(), 65536, 0.1, 0.02, clip=True)
    assert ((new.cpu().double() - torch.from_numpy(rnew)).abs().max() / torch.from_numpy(rnew).abs().max()) < 1e-6
    assert ((scaled.cpu().double() - torch.from_numpy(rs)).abs().max() / torch.from_numpy(rs).abs().max()) < 1e-6
