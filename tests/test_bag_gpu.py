"""Parity of the embedding-bag kernels (K3 forward, K4 backward, K5
double-backward) with the CPU oracle and with the reference's own outputs.

Tolerance: normwise relative error max|a-b|/max|b| below 1e-5 for fp32 and
2e-2 for bf16 (the contract's fp32 / bf16 bounds).
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import cases
from oracle import pkm_oracle as po

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


def rel_err(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if b.size == 0:
        return 0.0
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def tol(dtype):
    return 2e-2 if dtype == torch.bfloat16 else 1e-5


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from modelos_b200 import _native
    _native.lib()
    torch.cuda.init()
    yield
    _native.check_device_errors()


def run_all(idx, psw, W, g, gbar):
    from modelos_b200 import _native
    idx_d, psw_d, W_d, g_d, gb_d = (t.to(DEV) for t in (idx, psw, W, g, gbar))
    out = _native.bag_fwd(idx_d, W_d, psw_d)
    dW, dpsw, counts = _native.bag_bwd(idx_d, W_d, psw_d, g_d, want_counts=True)
    dG, da = _native.bag_bwd2(idx_d, psw_d, gb_d, g_d)
    torch.cuda.synchronize()
    return [t.float().cpu().numpy() for t in (out, dW, dpsw, dG, da)] + [counts.cpu().numpy()]


NAMES = ["f32_small", "f32_ragged", "f32_hot", "f32_L1", "bf16_c1like"]


@pytest.mark.parametrize("name", NAMES)
def test_golden_cases(name):
    d = np.load(os.path.join(GOLD, "embbag.npz"))
    p = lambda k: d[f"{name}__{k}"]  # noqa: E731
    dt = torch.bfloat16 if bool(p("bf16")) else torch.float32
    idx = torch.from_numpy(p("idx"))
    psw = torch.from_numpy(p("psw")).to(dt)
    W = torch.from_numpy(p("W")).to(dt)
    g = torch.from_numpy(p("g")).to(dt)
    gbar = torch.from_numpy(p("gbar")).to(dt)
    out, dW, dpsw, dG, da, counts = run_all(idx, psw, W, g, gbar)
    t = tol(dt)
    # against the reference's own outputs
    assert rel_err(out, p("out")) < t
    assert rel_err(dW, p("dW")) < t
    assert rel_err(dpsw, p("dpsw")) < t
    assert rel_err(dG, p("bw2_dg")) < t
    assert rel_err(da, p("bw2_da")) < t
    # against the float64 oracle
    o_out = po.bag_fwd(p("idx"), p("psw"), p("W"))
    o_dW, o_dpsw = po.bag_bwd(p("idx"), p("psw"), p("W"), p("g"))
    assert rel_err(out, o_out) < t
    assert rel_err(dW, o_dW) < t
    assert rel_err(dpsw, o_dpsw) < t
    np.testing.assert_array_equal(counts, po.bincount(p("idx"), W.shape[0]))
    # untouched rows are exactly zero
    assert (dW[counts == 0] == 0).all()


def test_backward_is_deterministic():
    from modelos_b200 import _native
    idx, psw, W, g = cases.embbag_case(512, 128, 2048, 256, seed=7, heads=4)
    idx[:, :40] = 3  # a hot row whose segment spans several chunks
    idx_d, psw_d, W_d, g_d = (t.to(DEV) for t in (idx, psw, W, g))
    a = _native.bag_bwd(idx_d, W_d, psw_d, g_d)
    b = _native.bag_bwd(idx_d, W_d, psw_d, g_d)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    o_dW, o_dpsw = po.bag_bwd(idx.numpy(), psw.numpy(), W.numpy(), g.numpy())
    assert rel_err(a[0].cpu().numpy(), o_dW) < 1e-5
    assert rel_err(a[1].cpu().numpy(), o_dpsw) < 1e-5


@pytest.mark.parametrize("D,dt", [(16, torch.float32), (48, torch.float32), (1024, torch.float32),
                                  (8, torch.bfloat16), (1024, torch.bfloat16), (2048, torch.bfloat16)])
def test_row_sizes(D, dt):
    from modelos_b200 import _native
    idx, psw, W, g = cases.embbag_case(300, 9, 777, D, seed=D)
    gbar = torch.randn(W.shape)
    out, dW, dpsw, dG, da, counts = run_all(idx, psw.to(dt), W.to(dt), g.to(dt), gbar.to(dt))
    f = lambda x: x.to(dt).float().numpy()  # noqa: E731
    t = tol(dt)
    assert rel_err(out, po.bag_fwd(idx.numpy(), f(psw), f(W))) < t
    o_dW, o_dpsw = po.bag_bwd(idx.numpy(), f(psw), f(W), f(g))
    assert rel_err(dW, o_dW) < t and rel_err(dpsw, o_dpsw) < t
    o_dG, o_da = po.bag_bwd2(idx.numpy(), f(psw), f(gbar), f(g))
    assert rel_err(dG, o_dG) < t and rel_err(da, o_da) < t


def test_no_weights_and_empty_inputs():
    from modelos_b200 import _native
    idx, psw, W, g = cases.embbag_case(20, 5, 50, 32, seed=3)
    out = _native.bag_fwd(idx.to(DEV), W.to(DEV), None).cpu().numpy()
    assert rel_err(out, po.bag_fwd(idx.numpy(), np.ones((20, 5)), W.numpy())) < 1e-5
    # zero bags
    e = torch.empty((0, 5), dtype=torch.long, device=DEV)
    assert _native.bag_fwd(e, W.to(DEV), None).shape == (0, 32)
    dW, _, _ = _native.bag_bwd(e, W.to(DEV), None, torch.empty((0, 32), device=DEV), need_dpsw=False)
    assert dW.abs().sum().item() == 0
    # zero-length bags
    e2 = torch.empty((4, 0), dtype=torch.long, device=DEV)
    assert _native.bag_fwd(e2, W.to(DEV), torch.empty((4, 0), device=DEV)).abs().sum().item() == 0


def test_out_of_range_indices_are_skipped_and_flagged():
    from modelos_b200 import _native
    idx, psw, W, g = cases.embbag_case(16, 8, 64, 32, seed=5)
    bad = idx.clone()
    bad[0, 0] = -1
    bad[3, 7] = 64
    _native.read_device_errors()
    out = _native.bag_fwd(bad.to(DEV), W.to(DEV), psw.to(DEV)).cpu().numpy()
    assert _native.read_device_errors() & _native.DEVERR_INDEX
    valid_psw = psw.clone()
    valid_psw[0, 0] = 0
    valid_psw[3, 7] = 0
    ref = po.bag_fwd(idx.numpy(), valid_psw.numpy(), W.numpy())
    assert rel_err(out, ref) < 1e-5
    dW, dpsw, _ = _native.bag_bwd(bad.to(DEV), W.to(DEV), psw.to(DEV), g.to(DEV))
    assert _native.read_device_errors() & _native.DEVERR_INDEX
    o_dW, o_dpsw = po.bag_bwd(idx.numpy(), valid_psw.numpy(), W.numpy(), g.numpy())
    dp = dpsw.cpu().numpy()
    assert dp[0, 0] == 0 and dp[3, 7] == 0
    assert rel_err(dW.cpu().numpy(), o_dW) < 1e-5


def test_config1_full_size_properties():
    """Benchmark config 1 at full size (16384 bags x 128, 262144 x 1024 bf16):
    sampled bags and rows against the oracle plus checksum identities."""
    from modelos_b200 import _native
    B, L, K, D = 16384, 128, 262144, 1024
    g = torch.Generator().manual_seed(1)
    idx = torch.randint(0, K, (B, L), generator=g)
    psw = torch.softmax(torch.randn(B, 4, L // 4, generator=g), -1).reshape(B, L).bfloat16()
    W = (torch.randn(K, D, generator=g) * 0.03).bfloat16()
    go = torch.randn(B, D, generator=g).bfloat16()
    idx_d, psw_d, W_d, g_d = (t.to(DEV) for t in (idx, psw, W, go))
    out = _native.bag_fwd(idx_d, W_d, psw_d)
    dW, dpsw, counts = _native.bag_bwd(idx_d, W_d, psw_d, g_d, want_counts=True)
    torch.cuda.synchronize()
    sb = torch.randint(0, B, (64,), generator=g)
    o = po.bag_fwd(idx[sb].numpy(), psw[sb].float().numpy(), W.float().numpy())
    assert rel_err(out[sb.to(DEV)].float().cpu().numpy(), o) < 2e-2
    # sampled dW rows: oracle on the occurrences of those rows
    rows = torch.randint(0, K, (32,), generator=g)
    flat = idx.reshape(-1)
    for r in rows.tolist():
        occ = (flat == r).nonzero().reshape(-1)
        ref = (psw.reshape(-1)[occ].double()[:, None] * go[occ // L].double()).sum(0).numpy()
        got = dW[r].double().cpu().numpy()
        assert np.abs(got - ref).max() <= 2e-2 * max(np.abs(ref).max(), 1e-3)
    # sampled per-sample gradients
    ob = torch.randint(0, B, (16,), generator=g)
    ref = (W[idx[ob]].double() * go[ob].double()[:, None, :]).sum(-1).numpy()
    assert rel_err(dpsw[ob.to(DEV)].float().cpu().numpy(), ref) < 2e-2
    # counts are the bincount; column sums of dW equal sum_b (sum_j psw) g_b
    assert torch.equal(counts.cpu().long(), torch.bincount(flat, minlength=K).int().long())
    lhs = dW.double().sum(0)
    rhs = (psw_d.double().sum(1)[:, None] * g_d.double()).sum(0)
    assert (lhs - rhs).abs().max().item() <= 2e-2 * rhs.abs().max().item() + 1e-2


def test_phased_backward_equals_one_call():
    """pkm_bag_bwd_sort + pkm_bag_bwd_rows over row ranges == pkm_bag_bwd, bit for bit."""
    from modelos_b200 import _native
    g = torch.Generator(device=DEV).manual_seed(9)
    B, L, K, D = 700, 64, 3000, 256
    idx = torch.randint(0, K, (B, L), generator=g, device=DEV)
    idx[:40, :] = 17  # a hot row split over several chunks
    psw = torch.rand(B, L, generator=g, device=DEV).bfloat16()
    W = torch.randn(K, D, generator=g, device=DEV).bfloat16()
    go = torch.randn(B, D, generator=g, device=DEV).bfloat16()
    dW, dpsw, _ = _native.bag_bwd(idx, W, psw, go)
    ph = _native.BagBwdPhases(idx, W, psw, go)
    ph.sort()
    out = torch.full_like(W, float("nan"))
    for r0, r1 in ((0, 17), (17, 18), (18, 1500), (1500, K)):
        ph.rows(r0, r1, out)
    torch.cuda.synchronize()
    assert torch.equal(out, dW)
    assert torch.equal(ph.dpsw, dpsw)
    _native.check_device_errors()


def test_ragged_kernels_against_oracle():
    """pkm_segment_sum and pkm_bag_bwd_ragged (the shard-local kernels of the
    row-sharded table) against the oracle; empty segments included."""
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(12)
    K, D = 500, 128
    sizes = torch.randint(0, 40, (300,), generator=g)
    sizes[5] = 0
    offsets = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(sizes, 0)])
    E = int(offsets[-1])
    rows = torch.randint(0, K, (E,), generator=g)
    w = torch.rand(E, generator=g)
    W = torch.randn(K, D, generator=g)
    out = _native.segment_sum(W.to(DEV), rows.to(DEV), w.to(DEV), offsets.to(DEV))
    ref = po.segment_sum(W.numpy(), rows.numpy(), w.numpy(), offsets.numpy())
    assert rel_err(out.cpu().numpy(), ref) < 1e-5
    src = torch.repeat_interleave(torch.arange(len(sizes)), sizes)
    gr = torch.randn(len(sizes), D, generator=g)
    dW, dpsw = _native.bag_bwd_ragged(rows.to(DEV), src.to(DEV), w.to(DEV), W.to(DEV), gr.to(DEV))
    rdW, rdpsw = po.bag_bwd_ragged(rows.numpy(), src.numpy(), w.numpy(), W.numpy(), gr.numpy())
    assert rel_err(dW.cpu().numpy(), rdW) < 1e-5
    assert rel_err(dpsw.cpu().numpy(), rdpsw) < 1e-5
    _native.check_device_errors()
