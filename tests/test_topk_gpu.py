"""Parity of the sub-key scores (K1) and the product top-k (K2): fp32 scores
and indices bit-exact with the oracle's definition, bf16 top-k bit-exact for
identical input scores, and the reference's indices matched tie-aware."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import cases
from oracle import pkm_oracle as po
from tiecmp import compare_topk

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


def rel_err(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("mode", ["dot", "idw"])
def test_scores_fp32_bit_exact(mode):
    from modelos_b200 import _native
    c0 = np.load(os.path.join(GOLD, "c0_pkm.npz"))
    q = c0["query"]
    keys = cases.pkm_state(cases.CONFIG0, 0)["keys"].numpy()
    got = _native.subkey_scores(torch.from_numpy(q).to(DEV), torch.from_numpy(keys).to(DEV), 4, mode)
    ref = po.subkey_scores(q, keys, 4, mode=mode)
    g = got.cpu().numpy()
    if mode == "dot":
        np.testing.assert_array_equal(g, ref)
    else:
        # the only non-IEEE-exact step is log(): fp64 log rounded to fp32 on
        # both sides, so mismatches would be isolated 1-ulp cases
        mism = (g != ref).sum()
        assert mism <= 2, mism
        assert rel_err(g, ref) < 1e-6


def test_scores_bf16_against_oracle():
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(3)
    q = torch.randn(512 * 4, 512, generator=g).bfloat16()
    keys = (torch.rand(2 * 4 * 512, 256, generator=g) * 2 - 1).div(512 ** 0.5).bfloat16()
    got = _native.subkey_scores(q.to(DEV), keys.to(DEV), 4, "dot_seq").float().cpu().numpy()
    ref = po.subkey_scores(q.float().numpy(), keys.float().numpy(), 4, bf16=True)
    # same products, same fp32 summation order, same bf16 rounding
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("N,H,kd,n", [(2048, 4, 512, 512), (300, 4, 512, 512), (1000, 2, 128, 200),
                                      (16384, 4, 512, 512)])
def test_scores_bf16_tensor_cores(N, H, kd, n):
    """tcgen05 path: fp32 accumulation in the tensor core's order, rounded to
    bf16 -- equal to the sequential oracle up to one bf16 ulp, and within
    fp32-accumulation error of an fp64 evaluation."""
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(N + n)
    q = torch.randn(N * H, kd, generator=g).bfloat16()
    keys = (torch.rand(2 * H * n, kd // 2, generator=g) * 2 - 1).div(kd ** 0.5).bfloat16()
    got = _native.subkey_scores(q.to(DEV), keys.to(DEV), H, "dot").float().cpu()
    q64 = q.double().view(N, H, 2, kd // 2)
    k64 = keys.double().view(H, 2, n, kd // 2)
    exact = torch.einsum("thpd,hpnd->thpn", q64, k64).reshape(N * H, 2, n)
    ref = exact.float().bfloat16().double()
    ulp = torch.clamp(exact.abs(), min=1e-3) * 2.0 ** -7
    assert ((got.double() - exact).abs() <= ulp).all()
    assert (got.double() == ref).float().mean().item() > 0.99


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,knn", [(128, 32), (512, 32), (512, 7), (256, 32), (256, 8), (100, 7), (16, 4),
                                   (1024, 32), (33, 1)])
def test_product_topk_bit_exact(dtype, n, knn):
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(n * 100 + knn)
    s = torch.randn(700, 2, n, generator=g)
    if dtype == torch.bfloat16:
        s = s.bfloat16()
    else:
        s = (s * 64).round() / 64  # coarse values: many exact ties in both stages
    idx, top, psw, s1, s2 = _native.product_topk(s.to(DEV).contiguous(), knn, want_psw=True, want_sub=True)
    ref = po.product_topk(s.float().numpy(), knn, bf16=dtype == torch.bfloat16)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref["indices"])
    np.testing.assert_array_equal(top.float().cpu().numpy(), ref["scores"])
    np.testing.assert_array_equal(s1.cpu().numpy(), ref["sub_indices1"])
    np.testing.assert_array_equal(s2.cpu().numpy(), ref["sub_indices2"])
    p_ref = po.softmax_rows(ref["scores"], bf16=dtype == torch.bfloat16)
    assert rel_err(psw.float().cpu().numpy(), p_ref) < (2e-2 if dtype == torch.bfloat16 else 1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("kind", ["integers", "zeros", "two_levels", "unaligned"])
def test_product_topk_heavy_ties(dtype, kind):
    """Rows whose knn-th pair sum is shared by pairs outside the pruned
    candidate set (the exact-merge path), all-equal rows, and a score
    tensor that does not start on a 16-byte boundary (scalar loads)."""
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(5)
    n, knn = 512, 32
    if kind == "integers":
        s = torch.randint(-3, 4, (300, 2, n), generator=g).float()
    elif kind == "zeros":
        s = torch.zeros(40, 2, n)
    elif kind == "two_levels":
        s = (torch.rand(300, 2, n, generator=g) < 0.1).float()
    else:
        s = torch.randn(300, 2, n, generator=g)
    s = s.to(dtype)
    if kind == "unaligned":
        buf = torch.empty(s.numel() + 1, dtype=dtype, device=DEV)
        dev = buf[1:].view(s.shape)
        dev.copy_(s.to(DEV))
    else:
        dev = s.to(DEV).contiguous()
    idx, top, psw, s1, s2 = _native.product_topk(dev, knn, want_psw=True, want_sub=True)
    ref = po.product_topk(s.float().numpy(), knn, bf16=dtype == torch.bfloat16)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref["indices"])
    np.testing.assert_array_equal(top.float().cpu().numpy(), ref["scores"])
    np.testing.assert_array_equal(s1.cpu().numpy(), ref["sub_indices1"])
    np.testing.assert_array_equal(s2.cpu().numpy(), ref["sub_indices2"])


def test_config0_indices_bit_exact_and_match_reference():
    from modelos_b200 import _native
    c0 = np.load(os.path.join(GOLD, "c0_pkm.npz"))
    keys = cases.pkm_state(cases.CONFIG0, 0)["keys"]
    sc = _native.subkey_scores(torch.from_numpy(c0["query"]).to(DEV), keys.to(DEV), 4)
    idx, top, _, _, _ = _native.product_topk(sc, 32)
    ref = po.pkm_get_indices(c0["query"], keys.numpy(), 4, 32)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref["indices"])
    np.testing.assert_array_equal(top.cpu().numpy(), ref["scores"])
    # the reference's own indices at seed 0 of config 0: identical
    np.testing.assert_array_equal(idx.cpu().numpy(), c0["gi_indices"])


def test_exact_ties_case():
    from modelos_b200 import _native
    d = np.load(os.path.join(GOLD, "ties.npz"))
    heads, knn = int(d["heads"]), int(d["knn"])
    sc = _native.subkey_scores(torch.from_numpy(d["q"]).to(DEV), torch.from_numpy(d["keys"]).to(DEV), heads)
    idx, top, _, _, _ = _native.product_topk(sc, knn)
    ref = po.pkm_get_indices(d["q"], d["keys"], heads, knn)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref["indices"])
    compare_topk(top.cpu().numpy(), idx.cpu().numpy(), d["scores"], d["indices"], ref["all_scores"], 0.0)


def test_score_bwd_prep_matches_softmax_backward():
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(11)
    R, knn, heads, n = 64, 32, 4, 128
    logits = torch.randn(R, knn, generator=g)
    psw = torch.softmax(logits, -1)
    dpsw = torch.randn(R, knn, generator=g)
    idx = torch.randint(0, n * n, (R, knn), generator=g)
    sub_idx, sub_w = _native.score_bwd_prep(idx.to(DEV), psw.to(DEV), dpsw.to(DEV), heads, n)
    ref_ds = psw * (dpsw - (psw * dpsw).sum(-1, keepdim=True))
    sw = sub_w.cpu()
    assert rel_err(sw[0::2].numpy(), ref_ds.numpy()) < 1e-6
    assert torch.equal(sw[0::2], sw[1::2])
    h = torch.arange(R)[:, None] % heads
    assert torch.equal(sub_idx.cpu()[0::2], (h * 2) * n + idx // n)
    assert torch.equal(sub_idx.cpu()[1::2], (h * 2 + 1) * n + idx % n)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_score_grad_dense_matches_scatter_of_softmax_backward(dtype):
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(12)
    R, knn, n = 96, 32, 64
    # distinct slots per row, many sharing a sub-key
    idx = torch.stack([torch.randperm(n * n, generator=g)[:knn] for _ in range(R)])
    idx[:, 1] = (idx[:, 0] // n) * n + (idx[:, 1] % n)  # force a shared half-0 sub-key
    psw = torch.softmax(torch.randn(R, knn, generator=g), -1).to(dtype)
    dpsw = torch.randn(R, knn, generator=g).to(dtype)
    dS = _native.score_grad_dense(idx.to(DEV), psw.to(DEV), dpsw.to(DEV), n).float().cpu()
    p, d = psw.float(), dpsw.float()
    ds = (p * (d - (p * d).sum(-1, keepdim=True))).to(dtype).float()
    ref = torch.zeros(R, 2, n)
    ref[:, 0].scatter_add_(1, idx // n, ds)
    ref[:, 1].scatter_add_(1, idx % n, ds)
    ref = ref.to(dtype).float()
    tolr = 1e-6 if dtype == torch.float32 else 2e-2
    assert rel_err(dS.numpy(), ref.numpy()) < tolr
    assert (dS[ref == 0] == 0).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_product_topk_nonfinite_scores(dtype):
    """Scores with NaN and +-inf (what a diverged model produces): every
    index stays a distinct valid slot built from the stage-1 lists, NaN
    ranks above everything (torch.topk's order), and finite rows are
    unaffected."""
    from modelos_b200 import _native
    n, knn = 512, 32
    g = torch.Generator().manual_seed(11)
    s = torch.randn(64, 2, n, generator=g)
    nan, inf = float("nan"), float("inf")
    s[0] = nan                      # all NaN
    s[1, 0, 7] = nan                # one NaN in half 0
    s[2, 1, :300] = nan             # most of half 1 NaN
    s[3, 0, 5] = inf
    s[3, 1, 9] = -inf               # inf + (-inf) pairs
    s[4, 0] = inf
    s[4, 1] = -inf                  # every pair inf - inf
    s[5, 0, 3] = -inf
    s[5, 1, 4] = inf
    s[6] = -inf
    s[7, 0, ::2] = nan
    s[7, 1, 1::3] = inf
    s = s.to(dtype)
    idx, top, psw, s1, s2 = _native.product_topk(s.to(DEV).contiguous(), knn, want_psw=True, want_sub=True)
    idx, s1, s2 = idx.cpu(), s1.cpu(), s2.cpu()
    assert ((idx >= 0) & (idx < n * n)).all()
    assert ((s1 >= 0) & (s1 < n)).all() and ((s2 >= 0) & (s2 < n)).all()
    for r in range(s.shape[0]):
        assert idx[r].unique().numel() == knn, r
        assert set((idx[r] // n).tolist()) <= set(s1[r].tolist()), r
        assert set((idx[r] % n).tolist()) <= set(s2[r].tolist()), r
    # a NaN sub-key is the best of its half, and every chosen slot uses it
    assert s1[1, 0].item() == 7 and ((idx[1] // n) == 7).all()
    # half 1 of row 2: the 32 lowest-index NaNs, in index order
    assert s2[2].tolist() == list(range(knn))
    ref = po.product_topk(s[8:].float().numpy(), knn, bf16=dtype == torch.bfloat16)
    np.testing.assert_array_equal(idx[8:].numpy(), ref["indices"])
    # rows with NaN but no -inf follow torch.topk's order (NaN above every
    # number, +inf next), ties to the lowest index: both stages exactly
    bf16 = dtype == torch.bfloat16
    sf = s.float().numpy()
    for r in (1, 2, 7):
        lists = [_nan_first_topk(sf[r, p], np.arange(n), knn) for p in (0, 1)]
        assert s1[r].tolist() == lists[0].tolist() and s2[r].tolist() == lists[1].tolist(), r
        i1, i2 = np.meshgrid(lists[0], lists[1], indexing="ij")
        sums = (sf[r, 0][i1] + sf[r, 1][i2]).astype(np.float32).reshape(-1)
        if bf16:
            sums = po.bf16_round(sums)
        want = _nan_first_topk(sums, (i1 * n + i2).reshape(-1), knn)
        assert idx[r].tolist() == want.tolist(), r
    # every pair inf - inf (row 4): the reference's sums are NaN; here the
    # pairs are summed as FLT_MAX - FLT_MAX = 0, so all tie and the lowest
    # slots win (a documented departure in scores and order)
    assert idx[4].tolist() == list(range(knn))
    assert (top[4].float().cpu() == 0).all()


def _nan_first_topk(vals: np.ndarray, ids: np.ndarray, k: int) -> np.ndarray:
    """Ids of the k best values: NaN first, then descending, ties by lowest id."""
    nan = np.isnan(vals)
    v = np.where(nan, 0.0, vals.astype(np.float64))
    order = np.lexsort((ids, -v, -nan.astype(np.int64)))
    return ids[order[:k]]


def test_score_grad_dense_ignores_out_of_range_slots():
    """A slot outside [0, n^2) credits no sub-key; the rest of the row is the
    same as without it."""
    from modelos_b200 import _native
    g = torch.Generator().manual_seed(2)
    R, knn, n = 64, 32, 128
    idx = torch.stack([torch.randperm(n * n, generator=g)[:knn] for _ in range(R)])
    dpsw = torch.randn(R, knn, generator=g)
    full = _native.score_grad_dense(idx.to(DEV), None, dpsw.to(DEV), n).cpu()
    bad = idx.clone()
    bad[:, 3] = -1
    bad[:, 7] = n * n + 5
    d2 = dpsw.clone()
    d2[:, 3] = 0
    d2[:, 7] = 0
    got = _native.score_grad_dense(bad.to(DEV), None, dpsw.to(DEV), n).cpu()
    ref = _native.score_grad_dense(idx.to(DEV), None, d2.to(DEV), n).cpu()
    assert torch.equal(got, ref)
    assert not torch.equal(got, full)
