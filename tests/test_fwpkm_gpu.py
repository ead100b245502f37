"""Module-level parity of ``FastWeightProductKeyMemory`` (chunked inner-loop
updates with double-backward) against the reference's outputs, losses, final
fast weights and outer gradients (fp32, tolerance 1e-5 normwise)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"
FW_KW = cases.FW_KW


def rel_err(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("score_type,fname", [("dot_product", "fwpkm_dot.npz"), ("idw", "fwpkm_idw.npz")])
def test_forward_wo_past_matches_reference(score_type, fname):
    torch.backends.cuda.matmul.allow_tf32 = False
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    d = np.load(os.path.join(GOLD, fname))
    m = FastWeightProductKeyMemory(qk_score_type=score_type, **FW_KW).to(DEV).train()
    keys, values, q, ref_v = cases.fwpkm_case(0)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    q = q.to(DEV).requires_grad_(True)
    ref_v = ref_v.to(DEV).requires_grad_(True)
    res = m(q, ref_v, None, 8)
    loss = (res["output"] ** 2).sum() + res["addr_loss"]
    loss.backward()
    np.testing.assert_array_equal(res["indices"].cpu().numpy(), d["indices"])
    tol = 1e-5
    assert rel_err(res["output"].detach().cpu().numpy(), d["output"]) < tol
    assert rel_err(res["scores"].detach().cpu().numpy(), d["scores"]) < tol
    assert rel_err(res["losses"].cpu().numpy(), d["losses"]) < tol
    assert abs(res["addr_loss"].item() - float(d["addr_loss"])) <= tol * abs(float(d["addr_loss"])) + 1e-7
    gn = np.array([g.item() for g in res["grad_norms"]])
    assert rel_err(gn, d["grad_norms"]) < tol
    assert rel_err(m.keys.detach().cpu().numpy(), d["final_keys"]) < tol
    assert rel_err(m.values.detach().cpu().numpy(), d["final_values"]) < tol
    assert rel_err(q.grad.cpu().numpy(), d["q_grad"]) < tol
    assert rel_err(ref_v.grad.cpu().numpy(), d["ref_v_grad"]) < tol
    assert rel_err(m.keys.grad.cpu().numpy(), d["keys_grad"]) < tol
    assert rel_err(m.values.grad.cpu().numpy(), d["values_grad"]) < tol


@pytest.mark.parametrize("fname", sorted(cases.FW_VARIANTS))
def test_variant_matches_reference(fname):
    """Non-default options (silu / relu transforms, temperature, keys trained
    by the memorisation loss, clipping, weight decay, no look-ahead, no
    addressing loss, gates, loss mask, a bf16 module) through the kernels
    against the reference's run, to 1e-5 of each tensor's largest magnitude
    (1e-2 for the bf16 module's bf16 results)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    cases.run_fw_variant(FastWeightProductKeyMemory, FW_KW, fname, np.load(os.path.join(GOLD, fname)), rel_err,
                         tol=cases.FW_VARIANT_TOL[cases.FW_VARIANTS[fname][3]], device=DEV)


def test_double_backward_wrapper_gradgradcheck():
    """EmbeddingBagBW (K5) against autograd's numerical second derivatives of
    the bag in float64-accumulated fp32 (small shapes)."""
    from modelos_b200.fwpkm.xformer_embeddingbag_grad_wrapper import xformers_embedding_bag
    g = torch.Generator().manual_seed(0)
    B, L, K, D = 6, 5, 11, 8
    idx = torch.randint(0, K, (B, L), generator=g).to(DEV)
    W = torch.randn(K, D, generator=g).to(DEV).requires_grad_(True)
    a = torch.rand(B, L, generator=g).to(DEV).requires_grad_(True)
    go = torch.randn(B, D, generator=g).to(DEV).requires_grad_(True)
    gbar = torch.randn(K, D, generator=g).to(DEV)
    y = xformers_embedding_bag(idx, W, a)
    (dW,) = torch.autograd.grad(y, W, grad_outputs=go, create_graph=True)
    d_go, d_a = torch.autograd.grad((dW * gbar).sum(), (go, a))
    # closed form: dW = sum_j a_bj go_b at idx; d/dgo <dW, gbar> = sum_j a_bj gbar[idx]
    ref_go = (a.detach()[..., None] * gbar[idx]).sum(1)
    ref_a = (gbar[idx] * go.detach()[:, None, :]).sum(-1)
    assert rel_err(d_go.cpu().numpy(), ref_go.cpu().numpy()) < 1e-6
    assert rel_err(d_a.cpu().numpy(), ref_a.cpu().numpy()) < 1e-6


@pytest.mark.parametrize("fname", sorted(cases.STREAM_FIXTURES))
def test_forward_w_past_matches_reference(fname):
    """``forward_w_past`` (``fwpkm/fwpkm.py:560-820``) over three calls that
    carry the signal queue (queue only; update then queue; update; the
    variant queues gates and a loss mask too): outputs, indices, losses,
    queues and fast weights after every call."""
    torch.backends.cuda.matmul.allow_tf32 = False
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    d = np.load(os.path.join(GOLD, fname))
    m = FastWeightProductKeyMemory(**dict(FW_KW, **cases.STREAM_FIXTURES[fname][0])).to(DEV).train()
    keys, values, _, _ = cases.fwpkm_case(1)
    q, ref_v, gates, mask = cases.stream_inputs(fname, device=DEV)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    cases.run_stream(m, q, ref_v, d, rel_err, gates=gates, mask=mask)


def test_forward_w_past_streaming_runs_and_updates():
    """Streaming path (``fwpkm/fwpkm.py:560-820``): output of the first call
    equals the no-past read of the same weights; the queue carries lookahead."""
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    m = FastWeightProductKeyMemory(**FW_KW).to(DEV)
    keys, values, q, ref_v = cases.fwpkm_case(1)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    q, ref_v = q.to(DEV), ref_v.to(DEV)
    empty = (None,) * 6
    res = m(q[:, :4], ref_v[:, :4], None, 8, past_key_values=empty)
    assert res["output"].shape == (2, 4, 32)
    assert res["past_key_values"][0].shape[1] == 4  # not enough signal yet: all queued
    res2 = m(q[:, 4:16], ref_v[:, 4:16], None, 8, past_key_values=res["past_key_values"])
    assert res2["losses"] is not None
    assert res2["past_key_values"][0].shape[1] == 1  # lookahead tail
    assert not torch.equal(m.values.detach().cpu(), values)


def test_config4_full_size_properties():
    """Benchmark config 4 at full size: k_dim 512, v_dim 1024, 4 heads x
    top-32 over 512^2 fp32 fast-weight slots (idw scores, joint softmax,
    addressing loss "me"), bf16 inputs [8, 4096] in chunks of 512 positions
    (eight inner updates of 4096 tokens, create_graph), then the outer
    backward.  Size-independent checks: indices in range, each token's
    scores sum to 1, everything finite; and on 256 sampled tokens of the
    first chunk, the selection equals the oracle's and the output equals the
    oracle's bag of the initial fast weights."""
    from modelos_b200 import _native
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    torch.manual_seed(0)
    B, T, CH, H, KNN, N_SUB = 8, 4096, 512, 4, 32, 512
    m = FastWeightProductKeyMemory(mem_k_dim=512, mem_v_dim=1024, mem_heads=H, mem_topk=KNN, mem_n_subkeys=N_SUB,
                                   learning_rate=0.1).to(DEV).train()
    m.reset_parameters()
    values0 = m.values.detach().clone()
    keys0 = m.keys.detach().clone()
    g = torch.Generator(device=DEV).manual_seed(4)
    q = torch.randn(B, T, H * 512, generator=g, device=DEV).bfloat16().requires_grad_()
    ref_v = torch.randn(B, T, 1024, generator=g, device=DEV).bfloat16().requires_grad_()
    res = m(q, ref_v, None, CH)
    out = res["output"]
    loss = (out.float() ** 2).sum() + res["addr_loss"]
    loss.backward()
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert out.shape == (B, T, 1024) and out.dtype == torch.bfloat16
    idx = res["indices"]
    assert idx.shape == (B, T, H, KNN)
    assert int(idx.min()) >= 0 and int(idx.max()) < N_SUB * N_SUB
    ssum = res["scores"].float().reshape(B, T, -1).sum(-1)
    assert (ssum - 1).abs().max().item() < 1e-5
    for name, t in (("output", out), ("losses", res["losses"]), ("q.grad", q.grad), ("ref_v.grad", ref_v.grad),
                    ("keys.grad", m.keys.grad), ("values.grad", m.values.grad), ("keys", m.keys),
                    ("values", m.values)):
        assert torch.isfinite(t.float()).all(), name
    assert m.values.grad.abs().max().item() > 0 and q.grad.abs().max().item() > 0
    # the first chunk reads the initial fast weights: on 256 sampled tokens,
    # its selection equals the oracle's on the same fp32 query and keys
    # (bit-exact scores and indices), and its output equals the oracle's
    # float64 bag of the initial values with those indices and the joint
    # softmax of those scores, within one bf16 rounding of the output
    import numpy as np

    from oracle import pkm_oracle as po
    rows = np.sort(np.random.default_rng(0).choice(B * CH, size=256, replace=False))
    q0 = q.detach()[:, :CH].reshape(B * CH, H, 512)[torch.from_numpy(rows).to(DEV)].float()
    sel = po.pkm_get_indices(q0.reshape(-1, 512).cpu().numpy(), keys0.cpu().numpy(), H, KNN, mode="idw")
    c0_idx = idx[:, :CH].reshape(B * CH, H * KNN)[torch.from_numpy(rows).to(DEV)].cpu().numpy()
    np.testing.assert_array_equal(c0_idx, sel["indices"].reshape(256, H * KNN))
    w = po.softmax_rows(sel["scores"].reshape(256, H * KNN))
    ref0 = po.bag_fwd(c0_idx, w, values0.cpu().numpy())
    got0 = out.detach()[:, :CH].reshape(B * CH, -1)[torch.from_numpy(rows).to(DEV)].float().cpu().numpy()
    assert rel_err(got0, ref0) < 2 ** -8


@pytest.mark.parametrize("mode", ["softmax", "silu", "relu"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("width,temp", [(128, 1.0), (37, 0.7), (512, 2.5)])
def test_score_transform_matches_torch(mode, dtype, width, temp):
    """``score_transform`` (``fwpkm/fwpkm.py:105-115``) on the kernel vs the
    reference's torch ops (fp32), forward and backward."""
    import torch.nn.functional as F

    from modelos_b200.fwpkm.fwpkm import ScoreTransform
    g = torch.Generator().manual_seed(width)
    s = (torch.randn(300, width, generator=g) * 3).to(dtype)
    dy = torch.randn(300, width, generator=g).to(dtype)
    x = s.to(DEV).requires_grad_(True)
    y = ScoreTransform.apply(x, temp, mode)
    (dx,) = torch.autograd.grad(y, x, dy.to(DEV))
    r = s.float().requires_grad_(True)
    z = r / temp
    yr = {"softmax": lambda: F.softmax(z, dim=-1), "silu": lambda: F.silu(z), "relu": lambda: F.relu(z)}[mode]()
    (dr,) = torch.autograd.grad(yr, r, dy.float())
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert y.dtype == dtype
    assert rel_err(y.detach().float().cpu().numpy(), yr.detach().numpy()) < tol
    assert rel_err(dx.float().cpu().numpy(), dr.numpy()) < tol
