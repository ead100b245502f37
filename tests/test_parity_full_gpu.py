"""Parity at the benchmarked geometries, against the reference's own outputs.

* Config 2 (``HashingMemory`` in bf16, n_keys 512 -> 262144 slots of 1024,
  k_dim 512, 4 heads x top-32, query BatchNorm) on one 2048-token sequence:
  fixture ``c2_full_bf16.npz``, the reference's layer forward + backward on
  CPU (``pkm/memory.py:190-289``).
* Config 4 geometry (``FastWeightProductKeyMemory``, fp32 fast weights over
  the same 262144 x 1024 table, idw and dot scores) on a 512-position
  sequence in two chunks: fixtures ``fwpkm_c4_{dot,idw}.npz``, the
  reference's ``forward_wo_past`` and the outer backward through the double
  backward (``fwpkm/fwpkm.py:395-558``).

The selection is checked on one query (bit-exact against the oracle on this
library's own scores, tie-aware against the reference) and then pinned to
the reference's for the value and gradient comparison (``tests/pinned.py``
explains why).  Tolerances: normwise 2e-2 in bf16, 1e-5 in fp32.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import cases
from oracle import pkm_oracle as po
from pinned import check_summary, pin_fwpkm_selection, pin_pkm_selection, rel_err
from tiecmp import compare_topk

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"
BF16_TOL = 2e-2
FP32_TOL = 1e-5


@pytest.fixture(scope="module")
def c2():
    from modelos_b200.pkm.memory import HashingMemory
    d = np.load(os.path.join(GOLD, "c2_full_bf16.npz"))
    st = cases.pkm_state(cases.CONFIG2, 0)
    sums = np.stack([cases.checksum(st[k]) for k in sorted(st)])
    np.testing.assert_allclose(sums, d["param_checksums"], rtol=1e-12)  # same seeded draws
    m = HashingMemory(**cases.CONFIG2)
    m.load_state_dict(st)
    del st
    return d, m


def _c2_model(c2):
    d, m0 = c2
    from modelos_b200.pkm.memory import HashingMemory
    m = HashingMemory(**cases.CONFIG2)
    m.load_state_dict(m0.state_dict())
    return d, m.to(DEV, torch.bfloat16).train()


def test_config2_full_geometry_selection(c2):
    """K1 + K2 on the reference's own bf16 query (512 tokens x 4 heads):
    K1 within one bf16 ulp of the oracle's sequential sum, K2 bit-exact with
    the oracle's top-k of the same scores, and the selection tie-aware equal
    to the reference's ``get_indices``."""
    from modelos_b200 import _native
    d, m = _c2_model(c2)
    q = cases.from_bf16_bits(d["gi_query"]).to(DEV)
    keys = m.keys.detach()
    s_all = _native.subkey_scores(q, keys, 4)
    s_np = s_all.float().cpu().numpy()
    ref_s = po.subkey_scores(q.float().cpu().numpy(), keys.float().cpu().numpy(), 4, bf16=True)
    # the tensor cores sum in another order than the sequential fp32 sum: the
    # fp32 results differ by a few ulps of the partial sums, so after rounding
    # a score differs by at most one bf16 ulp of itself, or (near zero, where
    # the sum cancels) by a few fp32 ulps of the row's scale
    ulp = np.spacing(np.abs(ref_s).astype(np.float32)) * 2.0 ** 16
    scale = np.abs(ref_s).max(axis=-1, keepdims=True) * 2.0 ** -20
    err = np.abs(s_np - ref_s)
    assert (err <= ulp + scale).all(), float((err / (ulp + scale)).max())
    idx, top, _, _, _ = _native.product_topk(s_all, 32)
    o = po.product_topk(s_np, 32, bf16=True)
    np.testing.assert_array_equal(idx.cpu().numpy(), o["indices"])
    np.testing.assert_array_equal(top.float().cpu().numpy(), o["scores"])
    # the module's get_indices equals that, and agrees with the reference up to near-ties
    s, i = m.get_indices(q, 32)
    np.testing.assert_array_equal(i.cpu().numpy(), idx.cpu().numpy())
    full = po.pkm_get_indices(q.float().cpu().numpy(), keys.float().cpu().numpy(), 4, 32, bf16=True)
    bound = 4 * 2.0 ** -8 * np.maximum(np.abs(d["gi_scores"]).max(axis=1), 1e-3)
    exact, ties, _ = compare_topk(full["scores"], full["indices"], d["gi_scores"], d["gi_indices"].astype(np.int64),
                                  full["all_scores"], bound=bound, bf16=True)
    assert exact + ties == d["gi_indices"].shape[0]


def test_config2_full_geometry_layer_matches_reference(c2, monkeypatch):
    """The whole layer forward + backward at config-2 geometry with the
    reference's selection: loss, output and every gradient (query projection
    and batch norm, keys, value table, SwiLU and value projections) within
    2e-2 of the reference's."""
    from modelos_b200 import _native
    d, m = _c2_model(c2)
    x = cases.pkm_input((1, 2048, 1024), 0)
    np.testing.assert_allclose(cases.checksum(x.bfloat16()), d["x_checksum"], rtol=1e-12)
    x = x.to(DEV, torch.bfloat16).requires_grad_(True)
    ref_idx = torch.from_numpy(d["indices"].astype(np.int64)).view(-1, 32)
    calls = pin_pkm_selection(monkeypatch, _native, ref_idx)
    y, idx = m(x)
    loss = (y.float() ** 2).sum()
    loss.backward()
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert len(calls) == 1
    np.testing.assert_array_equal(idx.view(d["indices"].shape).cpu().numpy(), d["indices"])
    assert abs(loss.item() - float(d["loss"])) <= BF16_TOL * abs(float(d["loss"]))
    check_summary(y.view(2048, -1).float(), d, "out", BF16_TOL)
    check_summary(x.grad.view(2048, -1).float(), d, "x_grad", BF16_TOL)
    kg = cases.from_bf16_bits(d["keys_grad"]).float().numpy()
    assert rel_err(m.keys.grad.float().cpu().numpy(), kg) < BF16_TOL
    check_summary(m.values.weight.grad.float(), d, "values_grad", BF16_TOL)
    qp = m.query_proj
    check_summary(qp.query_mlps[0].weight.grad.float(), d, "wq_grad", BF16_TOL)
    # batch norm removes the column mean, so the projection's bias gradient
    # is zero up to rounding on both sides; bound it by the scale of a column
    # sum of the normalised query's gradient (the norm's bias gradient)
    bq = qp.query_mlps[0].bias.grad.float().cpu().numpy()
    assert np.abs(bq - d["bq_grad"]).max() <= BF16_TOL * np.abs(d["bn_b_grad"]).max()
    for got, key in ((qp.norm.weight.grad, "bn_w_grad"),
                     (qp.norm.bias.grad, "bn_b_grad"), (qp.norm.running_mean, "bn_running_mean"),
                     (qp.norm.running_var, "bn_running_var"), (m.value_proj.bias.grad, "bv_grad"),
                     (m.swilu_projection.bias.grad, "bs_grad")):
        assert rel_err(got.float().cpu().numpy(), d[key]) < BF16_TOL, key
    check_summary(m.value_proj.weight.grad.float(), d, "wv_grad", BF16_TOL)
    check_summary(m.swilu_projection.weight.grad.float(), d, "ws_grad", BF16_TOL)


FW_CASES = [("dot_product", "fwpkm_c4_dot.npz"), ("idw", "fwpkm_c4_idw.npz")]


def _fw_model(score_type):
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    m = FastWeightProductKeyMemory(qk_score_type=score_type, **cases.FW_C4).to(DEV).train()
    keys, values, q, ref_v = cases.fwpkm_c4_case(0)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    return m, keys, values, q, ref_v


@pytest.mark.parametrize("score_type,fname", FW_CASES)
def test_config4_geometry_selection(score_type, fname):
    """First chunk, initial fast weights: the module's selection equals the
    oracle's bit for bit (fp32 scores are bit-exact by definition) and agrees
    with the reference's up to near-ties."""
    d = np.load(os.path.join(GOLD, fname))
    m, keys, values, q, ref_v = _fw_model(score_type)
    H, kd, knn = 4, 512, 32
    q0 = q[0, :cases.FW_C4_CHUNK].reshape(-1, H, kd)
    with torch.no_grad():
        s, i, _, _, _, _ = m.get_indices(q0.to(DEV), m.keys.float())
    mode = "dot" if score_type == "dot_product" else "idw"
    full = po.pkm_get_indices(q0.reshape(-1, kd).numpy(), keys.numpy(), H, knn, mode=mode)
    np.testing.assert_array_equal(i.reshape(-1, knn).cpu().numpy(), full["indices"])
    assert rel_err(s.reshape(-1, knn).cpu().numpy(), full["scores"]) == 0.0
    bound = 8 * np.spacing(np.abs(d["gi0_scores"]).max(axis=1).astype(np.float32)).astype(np.float64)
    exact, ties, _ = compare_topk(full["scores"], full["indices"], d["gi0_scores"],
                                  d["gi0_indices"].astype(np.int64), full["all_scores"], bound=bound)
    assert exact + ties == d["gi0_indices"].shape[0]


@pytest.mark.parametrize("score_type,fname", FW_CASES)
def test_config4_geometry_matches_reference(score_type, fname, monkeypatch):
    """``forward_wo_past`` over two chunks at config-4 geometry with the
    reference's selection, then the outer backward: output, scores, losses,
    grad norms, final fast weights and every outer gradient within 1e-5."""
    from modelos_b200 import _native
    d = np.load(os.path.join(GOLD, fname))
    m, keys, values, q, ref_v = _fw_model(score_type)
    np.testing.assert_allclose(cases.checksum(values), d["values_checksum"], rtol=1e-12)
    calls = pin_fwpkm_selection(monkeypatch, _native, torch.from_numpy(d["indices"].astype(np.int64)),
                                cases.FW_C4_CHUNK)
    T = q.shape[1]
    q = q.to(DEV).requires_grad_(True)
    ref_v = ref_v.to(DEV).requires_grad_(True)
    res = m(q, ref_v, None, cases.FW_C4_CHUNK)
    loss = (res["output"] ** 2).sum() + res["addr_loss"]
    loss.backward()
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert calls[0] == T // cases.FW_C4_CHUNK
    tol = FP32_TOL
    assert rel_err(res["output"].detach().cpu().numpy(), d["output"]) < tol
    assert rel_err(res["scores"].detach().cpu().numpy(), d["scores"]) < tol
    assert rel_err(res["losses"].cpu().numpy(), d["losses"]) < tol
    assert abs(res["addr_loss"].item() - float(d["addr_loss"])) <= tol * abs(float(d["addr_loss"]))
    # the inner gradients' norms: against their float64 values on the
    # reference's side (its own fp32 CPU reduction is 0.2 % low at this size)
    assert rel_err(np.array([g.item() for g in res["grad_norms"]]), d["grad_norms_f64"]) < tol
    assert abs(loss.item() - float(d["loss"])) <= tol * abs(float(d["loss"]))
    check_summary(m.keys.detach(), d, "final_keys", tol)
    check_summary(m.values.detach() - values.to(DEV), d, "values_delta", tol)
    check_summary(q.grad.view(T, -1), d, "q_grad", tol)
    check_summary(ref_v.grad.view(T, -1), d, "ref_v_grad", tol)
    check_summary(m.keys.grad, d, "keys_grad", tol)
    check_summary(m.values.grad, d, "values_grad", tol)
