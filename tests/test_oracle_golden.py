"""Pin the CPU oracle against fixtures produced by the reference itself.

These run without a GPU and without the reference tree: the fixtures under
``tests/golden`` were written by ``tests/golden/make_golden.py``.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import cases
from oracle import pkm_oracle as po
from tiecmp import compare_topk

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def rel_err(a, b):
    """Normwise relative error max|a-b| / max|b| (the tolerance definition used
    throughout the tests: fp32 1e-5, bf16 2e-2)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = max(np.abs(b).max(), 1e-30) if b.size else 1.0
    return float(np.abs(a - b).max() / den) if b.size else 0.0


@pytest.fixture(scope="module")
def c0():
    return np.load(os.path.join(GOLD, "c0_pkm.npz"))


def test_case_generator_is_stable(c0):
    st = cases.pkm_state(cases.CONFIG0, 0)
    got = np.stack([cases.checksum(st[k]) for k in sorted(st)])
    np.testing.assert_allclose(got, c0["param_checksums"], rtol=1e-12, atol=1e-9)
    x = cases.pkm_input((2, 128, 512), 0)
    np.testing.assert_allclose(cases.checksum(x), c0["x_checksum"], rtol=1e-12, atol=1e-9)


def test_c0_get_indices_matches_reference(c0):
    st = cases.pkm_state(cases.CONFIG0, 0)
    q = c0["query"]
    res = po.pkm_get_indices(q, st["keys"].numpy(), heads=4, knn=32)
    n_exact, n_tie, worst = compare_topk(res["scores"], res["indices"], c0["gi_scores"],
                                         c0["gi_indices"], res["all_scores"], bound=1e-5)
    # seed 0 of config 0: the reference and the oracle agree on every row
    assert n_tie == 0, (n_exact, n_tie, worst)
    np.testing.assert_array_equal(res["indices"], c0["gi_indices"])


def test_indices_other_seeds_tie_aware():
    d = np.load(os.path.join(GOLD, "c0_indices_seeds.npz"))
    total_tie = 0
    for sd in (1, 2):
        st = cases.pkm_state(cases.CONFIG0, sd)
        g = torch.Generator().manual_seed(40_000 + sd)
        q = torch.randn((256 * 4, 256), generator=g)
        np.testing.assert_allclose(cases.checksum(q), d[f"s{sd}_q_checksum"], rtol=1e-12)
        res = po.pkm_get_indices(q.numpy(), st["keys"].numpy(), heads=4, knn=32)
        n_exact, n_tie, worst = compare_topk(res["scores"], res["indices"], d[f"s{sd}_scores"],
                                             d[f"s{sd}_indices"], res["all_scores"], bound=1e-5)
        total_tie += n_tie
        assert n_exact + n_tie == 1024
    # near-tie reorderings between MKL's blocked sums and the sequential sum
    # are rare (about 1 in 1024 rows at seed 1)
    assert total_tie <= 8


def test_exact_ties_follow_lowest_index_rule():
    d = np.load(os.path.join(GOLD, "ties.npz"))
    heads, knn = int(d["heads"]), int(d["knn"])
    res = po.pkm_get_indices(d["q"], d["keys"], heads=heads, knn=knn)
    # quantised inputs: every score is exact, so the score lists agree exactly
    np.testing.assert_array_equal(res["scores"], d["scores"])
    n_exact, n_tie, worst = compare_topk(res["scores"], res["indices"], d["scores"], d["indices"],
                                         res["all_scores"], bound=0.0)
    assert worst == 0.0
    # the oracle's own order is canonical: score desc, slot asc
    s, i = res["scores"], res["indices"]
    same = s[:, 1:] == s[:, :-1]
    assert (s[:, 1:] <= s[:, :-1]).all()
    assert (i[:, 1:][same] > i[:, :-1][same]).all()


def test_softmax_and_bag_forward_reproduce_layer_output(c0):
    """Oracle bag on the reference's indices, then the (float64) SwiLU/value
    projection of ``pkm/memory.py:228-229``, equals the reference output."""
    st = {k: v.double().numpy() for k, v in cases.pkm_state(cases.CONFIG0, 0).items()}
    x = cases.pkm_input((2, 128, 512), 0).double().numpy().reshape(-1, 512)
    scores = c0["gi_scores"].reshape(256, 4, 32)
    psw = po.softmax_rows(scores).reshape(256, 128)
    idx = c0["gi_indices"].reshape(256, 128)
    bag = po.bag_fwd(idx, psw, st["values.weight"])
    h = x @ st["swilu_projection.weight"].T + st["swilu_projection.bias"]
    out = (bag * (h / (1 + np.exp(-h)))) @ st["value_proj.weight"].T + st["value_proj.bias"]
    assert rel_err(out.reshape(2, 128, 512), c0["out"]) < 1e-5
    np.testing.assert_array_equal(idx.reshape(2, 128, 128), c0["indices"])


EMB_NAMES = ["f32_small", "f32_ragged", "f32_hot", "f32_L1", "bf16_c1like"]


@pytest.mark.parametrize("name", EMB_NAMES)
def test_embbag_oracle_matches_reference(name):
    d = np.load(os.path.join(GOLD, "embbag.npz"))
    p = lambda k: d[f"{name}__{k}"]  # noqa: E731
    bf16 = bool(p("bf16"))
    tol = 2e-2 if bf16 else 1e-5
    idx, psw, W, g, gbar = p("idx"), p("psw"), p("W"), p("g"), p("gbar")
    out = po.bag_fwd(idx, psw, W)
    assert rel_err(out, p("out")) < tol
    assert rel_err(out, p("out_fw")) < tol
    dW, dpsw = po.bag_bwd(idx, psw, W, g)
    assert rel_err(dW, p("dW")) < tol
    assert rel_err(dpsw, p("dpsw")) < tol
    assert rel_err(dW, p("dW_native")) < tol
    assert rel_err(dpsw, p("dpsw_native")) < tol
    dG, da = po.bag_bwd2(idx, psw, gbar, g)
    assert rel_err(dG, p("bw2_dg")) < tol
    assert rel_err(da, p("bw2_da")) < tol
    # untouched rows of the dense weight gradient are exactly zero
    touched = np.zeros(W.shape[0], bool)
    touched[idx.reshape(-1)] = True
    assert (p("dW")[~touched] == 0).all() and (dW[~touched] == 0).all()


@pytest.mark.parametrize("kind", ["dot", "idw"])
def test_fwpkm_first_chunk_output(kind):
    """First chunk of ``forward_wo_past`` reads the initial fast weights:
    oracle scores (joint softmax over heads*topk, ``fwpkm/fwpkm.py:179``) and
    bag reproduce the reference output for those tokens."""
    d = np.load(os.path.join(GOLD, f"fwpkm_{'dot' if kind == 'dot' else 'idw'}.npz"))
    keys, values, q, ref_v = cases.fwpkm_case(0)
    B, T, H, kd, topk = 2, 16, 2, 16, 4
    qc = q[:, :8].reshape(-1, kd).numpy()
    res = po.pkm_get_indices(qc, keys.numpy(), heads=H, knn=topk, mode=kind)
    idx = res["indices"].reshape(B * 8, H * topk)
    ref_idx = d["indices"][:, :8].reshape(B * 8, H * topk)
    np.testing.assert_array_equal(idx, ref_idx)
    psw = po.softmax_rows(res["scores"].reshape(B * 8, H * topk))
    out = po.bag_fwd(idx, psw, values.numpy())
    assert rel_err(out, d["output"][:, :8].reshape(B * 8, -1)) < 1e-5
    assert rel_err(psw, d["scores"][:, :8].reshape(B * 8, -1)) < 1e-5


def test_c2_small_bf16_indices_tie_aware():
    d = np.load(os.path.join(GOLD, "c2_small_bf16.npz"))
    cfg = dict(cases.CONFIG2)
    cfg.update(mem_n_keys=64)
    st = cases.pkm_state(cfg, 0)
    keys = po.bf16_round(st["keys"].numpy())
    q = d["query"]  # bf16 values stored as fp32
    res = po.pkm_get_indices(q, keys, heads=4, knn=32, bf16=True)
    bound = 4 * 2.0 ** -8 * np.maximum(np.abs(d["gi_scores"]).max(axis=1), 1e-3)
    n_exact, n_tie, worst = compare_topk(res["scores"], res["indices"], d["gi_scores"],
                                         d["gi_indices"], res["all_scores"], bound=bound, bf16=True)
    assert n_exact + n_tie == q.shape[0]


def test_bincount_and_fw_update_math():
    rng = np.random.default_rng(0)
    idx = rng.integers(0, 10, size=(6, 4))
    c = po.bincount(idx, 12)
    assert c.sum() == 24 and c[10:].sum() == 0
    p = rng.standard_normal((12, 3))
    g = rng.standard_normal((12, 3))
    p2, gs = po.fw_value_update(p, g, c, scale=5.0, lr=0.1, wd=0.01)
    np.testing.assert_allclose(gs, g * 5.0 / np.maximum(c, 1)[:, None])
    np.testing.assert_allclose(p2, p - 0.1 * (gs + 0.01 * p))


def test_bf16_round_matches_torch():
    x = torch.randn(10000) * 3
    np.testing.assert_array_equal(po.bf16_round(x.numpy()), x.bfloat16().float().numpy())


def test_numpy_layer_port_matches_reference_step(c0):
    """The CPU port timed as the baseline computes the reference's step."""
    from oracle.pkm_layer import layer_step
    st = {k: v.numpy() for k, v in cases.pkm_state(cases.CONFIG0, 0).items()}
    x = cases.pkm_input((2, 128, 512), 0).numpy()
    loss, G = layer_step(st, x, heads=4, knn=32, norm="rms")
    assert abs(loss - float(c0["loss"])) <= 1e-4 * abs(float(c0["loss"]))
    assert rel_err(G["x"], c0["x_grad"]) < 1e-4
    assert rel_err(G["keys"], c0["keys_grad"]) < 1e-4
    assert rel_err(np.linalg.norm(G["values.weight"], axis=1), c0["values_grad_rownorm"]) < 1e-4
    assert rel_err(G["query_proj.query_mlps.0.bias"], c0["bq_grad"]) < 1e-4


@pytest.mark.parametrize("name", cases.ADDR_CASES)
def test_addr_stats_oracle_matches_reference(name):
    """``compute_addr_stats`` of the reference's decoder layer: the two ratios
    are integer counts over the same denominators (equal exactly); the KL is
    fp32 in the reference and fp64 here."""
    d = np.load(os.path.join(GOLD, "addr_stats.npz"))
    idx, K, _ = cases.addr_case(name)
    np.testing.assert_allclose(cases.checksum(idx), d[name + "_idx_checksum"], rtol=1e-12, atol=1e-9)
    st = po.addr_stats(idx.numpy(), K)
    ref = d[name + "_stats"]
    assert st["collision_ratio"] == ref[0]
    assert st["coverage_ratio"] == ref[1]
    assert abs(st["kld"] - ref[2]) <= 1e-5 * max(1.0, abs(ref[2]))


def test_c2_full_geometry_selection_tie_aware():
    """Config-2 geometry (262144 slots, bf16) on the reference's own query:
    the oracle's selection agrees with the reference's ``get_indices`` up to
    near-ties (bf16 score lists tie at the top-k boundary)."""
    d = np.load(os.path.join(GOLD, "c2_full_bf16.npz"))
    g = torch.Generator().manual_seed(0)
    cfg = cases.CONFIG2
    H, n, kd = cfg["mem_heads"], cfg["mem_n_keys"], cfg["mem_k_dim"]
    # the keys are the first draw of ``cases.pkm_state`` (no need to draw the table)
    keys = cases._u(g, (2 * H * n, kd // 2), 1 / np.sqrt(kd)).bfloat16().float().numpy()
    q = cases.from_bf16_bits(d["gi_query"]).float().numpy()
    res = po.pkm_get_indices(q, keys, H, 32, bf16=True)
    bound = 4 * 2.0 ** -8 * np.maximum(np.abs(d["gi_scores"]).max(axis=1), 1e-3)
    n_exact, n_tie, _ = compare_topk(res["scores"], res["indices"], d["gi_scores"],
                                     d["gi_indices"].astype(np.int64), res["all_scores"], bound=bound, bf16=True)
    # exact bf16 ties inside the lists are ordered differently on the two
    # sides (lowest index first here), so rows pass through the near-tie rule
    assert n_exact + n_tie == q.shape[0]


@pytest.mark.parametrize("mode,fname", [("dot", "fwpkm_c4_dot.npz"), ("idw", "fwpkm_c4_idw.npz")])
def test_c4_geometry_first_chunk_selection_tie_aware(mode, fname):
    """Config-4 geometry, first chunk on the initial keys: the oracle's fp32
    selection agrees with the reference's up to near-ties (the idw scores of
    512 sub-keys pack into exact fp32 ties, ordered by torch's partial sort
    on the reference's side and by the lowest index here)."""
    d = np.load(os.path.join(GOLD, fname))
    keys, values, q, ref_v = cases.fwpkm_c4_case(0)
    np.testing.assert_allclose(cases.checksum(keys), d["keys_checksum"], rtol=1e-12)
    H, kd, knn = 4, 512, 32
    q0 = q[0, :cases.FW_C4_CHUNK].reshape(-1, kd).numpy()
    res = po.pkm_get_indices(q0, keys.numpy(), H, knn, mode=mode)
    bound = 8 * np.spacing(np.abs(d["gi0_scores"]).max(axis=1).astype(np.float32)).astype(np.float64)
    n_exact, n_tie, _ = compare_topk(res["scores"], res["indices"], d["gi0_scores"],
                                     d["gi0_indices"].astype(np.int64), res["all_scores"], bound=bound)
    assert n_exact + n_tie == q0.shape[0] and n_exact > 0


def test_torch_restatement_equals_reference_at_config2_geometry():
    """``oracle/ref_torch.py`` (the timed reference arm of ``bench.py``) runs
    the reference's CPU operators in the reference's order: at config-2
    geometry its indices, loss, output and key gradient equal the
    reference's bit for bit, and the value-table gradient's fingerprint to
    the fixture's float32 storage."""
    from oracle import ref_torch as rt
    d = np.load(os.path.join(GOLD, "c2_full_bf16.npz"))
    P = rt.params_from_state(cases.pkm_state(cases.CONFIG2, 0), torch.bfloat16)
    x = cases.pkm_input((1, 2048, 1024), 0).bfloat16()
    out, slots, loss = rt.layer_step(P, x, 4, 32, 512, "bn")
    np.testing.assert_array_equal(slots.numpy(), d["indices"])
    assert loss.item() == float(d["loss"])
    s = cases.summarize(out.view(2048, -1).float(), rows_idx=d["out_rows_idx"])
    for part in ("rownorm", "proj", "rows"):
        np.testing.assert_array_equal(s[part], d["out_" + part])
    np.testing.assert_array_equal(cases.bf16_bits(P["keys"].grad), d["keys_grad"])
    s = cases.summarize(P["values"].grad.float(), rows_idx=d["values_grad_rows_idx"])
    np.testing.assert_array_equal(s["rows"], d["values_grad_rows"])
    assert rel_err(s["rownorm"], d["values_grad_rownorm"]) < 1e-7
    np.testing.assert_array_equal(P["bq"].grad.float().numpy(), d["bq_grad"])


def test_torch_restatement_of_the_fast_weight_layer_equals_reference():
    """``oracle/ref_torch.fw_forward`` (the config-4 reference arm of
    ``bench.py``) runs the fast-weight memory's CPU operators in the
    reference's order: at config-4 geometry (idw) its indices, output, loss
    and outer gradients equal the reference's bit for bit."""
    from oracle import ref_torch as rt
    d = np.load(os.path.join(GOLD, "fwpkm_c4_idw.npz"))
    keys, values, q, ref_v = cases.fwpkm_c4_case(0)
    P = {"keys": keys.clone().requires_grad_(True), "values": values.clone().requires_grad_(True)}
    q.requires_grad_(True)
    ref_v.requires_grad_(True)
    out, idx, addr = rt.fw_forward(P, q, ref_v, cases.FW_C4, cases.FW_C4_CHUNK, "idw")
    loss = (out ** 2).sum() + addr
    loss.backward()
    np.testing.assert_array_equal(idx.numpy().reshape(d["indices"].shape), d["indices"])
    np.testing.assert_array_equal(out.detach().numpy(), d["output"])
    assert loss.item() == float(d["loss"])
    for t, key in ((q.grad.view(q.shape[1], -1), "q_grad"), (P["values"].grad, "values_grad"),
                   (P["keys"].grad, "keys_grad")):
        s = cases.summarize(t, rows_idx=d[key + "_rows_idx"])
        np.testing.assert_array_equal(s["rows"], d[key + "_rows"])
