"""Module-level parity: ``modelos_b200.pkm.memory.HashingMemory`` on the GPU
against the reference's outputs and gradients (fixtures from the reference
run on CPU with the same seeded state)."""
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


def build(cfg, seed, dtype):
    from modelos_b200.pkm.memory import HashingMemory
    m = HashingMemory(**cfg)
    m.load_state_dict(cases.pkm_state(cfg, seed))
    return m.to(DEV, dtype).train()


def test_config0_forward_backward_matches_reference():
    torch.backends.cuda.matmul.allow_tf32 = False
    c0 = np.load(os.path.join(GOLD, "c0_pkm.npz"))
    m = build(cases.CONFIG0, 0, torch.float32)
    x = cases.pkm_input((2, 128, 512), 0).to(DEV).requires_grad_(True)
    y, idx = m(x)
    loss = (y.float() ** 2).sum()
    loss.backward()
    np.testing.assert_array_equal(idx.cpu().numpy(), c0["indices"])
    assert rel_err(y.detach().cpu().numpy(), c0["out"]) < 1e-5
    assert abs(loss.item() - float(c0["loss"])) <= 1e-5 * abs(float(c0["loss"]))
    assert rel_err(x.grad.cpu().numpy(), c0["x_grad"]) < 1e-5
    assert rel_err(m.keys.grad.cpu().numpy(), c0["keys_grad"]) < 1e-5
    vg = m.values.weight.grad.double().cpu()
    assert rel_err(vg.norm(dim=1).numpy(), c0["values_grad_rownorm"]) < 1e-5
    assert rel_err(vg[torch.from_numpy(c0["values_grad_rows_idx"])].numpy(), c0["values_grad_rows"]) < 1e-5
    wg = m.query_proj.query_mlps[0].weight.grad.double().cpu()
    assert rel_err(wg.norm(dim=1).numpy(), c0["wq_grad_rownorm"]) < 1e-5
    assert rel_err(wg[torch.from_numpy(c0["wq_grad_rows_idx"])].numpy(), c0["wq_grad_rows"]) < 1e-5
    assert rel_err(m.query_proj.query_mlps[0].bias.grad.cpu().numpy(), c0["bq_grad"]) < 1e-5


def test_config0_get_indices_matches_reference():
    c0 = np.load(os.path.join(GOLD, "c0_pkm.npz"))
    m = build(cases.CONFIG0, 0, torch.float32)
    q = torch.from_numpy(c0["query"]).to(DEV)
    s, i = m.get_indices(q, 32)
    np.testing.assert_array_equal(i.cpu().numpy(), c0["gi_indices"])
    assert rel_err(s.detach().cpu().numpy(), c0["gi_scores"]) < 1e-5


def test_get_indices_gradient_matches_autograd_of_dense_formula():
    """d(scores)/d(query, keys) through the sub-key bags equals autograd of
    the reference's dense einsum formulation (``pkm/memory.py:267-285``)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    cfg = dict(cases.CONFIG0)
    m = build(cfg, 1, torch.float32)
    g = torch.Generator().manual_seed(5)
    q = torch.randn(64 * 4, 256, generator=g).to(DEV).requires_grad_(True)
    s, i = m.get_indices(q, 32)
    w = torch.randn(s.shape, generator=g).to(DEV)
    dq, dk = torch.autograd.grad((s * w).sum(), (q, m.keys))
    # dense reference formula evaluated at the same indices
    q2 = q.detach().clone().requires_grad_(True)
    k2 = m.keys.detach().clone().requires_grad_(True)
    kv = k2.view(4, 2, 128, 128)
    qv = q2.view(64, 4, 256)
    s1 = torch.einsum("blh,lkh->blk", qv[:, :, :128], kv[:, 0])
    s2 = torch.einsum("blh,lkh->blk", qv[:, :, 128:], kv[:, 1])
    iv = i.view(64, 4, 32)
    sel = s1.gather(2, iv // 128) + s2.gather(2, iv % 128)
    dq2, dk2 = torch.autograd.grad((sel.view(-1, 32) * w).sum(), (q2, k2))
    assert rel_err(dq.cpu().numpy(), dq2.cpu().numpy()) < 1e-5
    assert rel_err(dk.cpu().numpy(), dk2.cpu().numpy()) < 1e-5


def _dense_fp32_layer(m, x, idx):
    """fp32 torch evaluation of the layer (``pkm/memory.py:190-248``) with the
    top-k selection fixed to ``idx`` [N, H*knn]: scores by dense einsum and
    gather, per-head softmax, bag by gather, SwiLU/value projection."""
    H, kd, knn = m.heads, m.k_dim, m.knn
    n = int(round(m.size ** 0.5))
    N = x.shape[0] * x.shape[1]
    xf = x.reshape(N, -1)
    q = m.query_proj(xf).view(N, H, kd)
    kv = m.keys.view(H, 2, n, kd // 2)
    s1 = torch.einsum("bhd,hkd->bhk", q[:, :, : kd // 2], kv[:, 0])
    s2 = torch.einsum("bhd,hkd->bhk", q[:, :, kd // 2:], kv[:, 1])
    iv = idx.view(N, H, knn)
    sel = s1.gather(2, iv // n) + s2.gather(2, iv % n)
    psw = torch.softmax(sel, -1).view(N, H * knn)
    bag = (psw[..., None] * m.values.weight[idx.view(N, -1)]).sum(1)
    out = m.value_proj(bag * torch.nn.functional.silu(m.swilu_projection(xf)))
    return out.view(x.shape[0], x.shape[1], -1)


def test_config2_geometry_bf16_matches_reference():
    """Config-2 layer (bf16, query BatchNorm) with a 64x64 table, 64 tokens.

    In bf16 most scores tie at the top-k boundary, so the reference's own
    selection among exact ties (torch.topk order, unspecified) decides a few
    slots; the selection is therefore checked tie-aware against the reference,
    bit-exact against the oracle, and the layer's values and gradients against
    an fp32 torch evaluation that uses the same selection."""
    torch.backends.cuda.matmul.allow_tf32 = False
    d = np.load(os.path.join(GOLD, "c2_small_bf16.npz"))
    cfg = dict(cases.CONFIG2)
    cfg.update(mem_n_keys=64)
    m = build(cfg, 0, torch.bfloat16)
    x = cases.pkm_input((2, 32, 1024), 0).to(DEV, torch.bfloat16).requires_grad_(True)
    with torch.no_grad():
        q = m.query_proj(x.view(-1, 1024))
    # the bf16 query (cuBLAS here, CPU in the fixture) agrees within bf16 tolerance
    assert rel_err(q.float().cpu().numpy(), d["query"]) < 2e-2
    # selection on the fixture's query: bit-exact vs oracle, tie-aware vs reference
    keys_b = po.bf16_round(cases.pkm_state(cfg, 0)["keys"].numpy())
    res = po.pkm_get_indices(d["query"], keys_b, 4, 32, bf16=True)
    s, i = m.get_indices(torch.from_numpy(d["query"]).to(DEV, torch.bfloat16), 32)
    # tensor-core sums may round a bf16 score one ulp apart from the oracle's
    # sequential sum; the selection must agree up to such near-ties
    ulp = 2 * 2.0 ** -8 * np.maximum(np.abs(res["scores"]).max(axis=1), 1e-3)
    compare_topk(res["scores"], res["indices"], s.detach().float().cpu().numpy(), i.cpu().numpy(),
                 res["all_scores"], bound=ulp, bf16=True)
    bound = 4 * 2.0 ** -8 * np.maximum(np.abs(d["gi_scores"]).max(axis=1), 1e-3)
    compare_topk(res["scores"], res["indices"], d["gi_scores"], d["gi_indices"], res["all_scores"],
                 bound=bound, bf16=True)
    # the bf16 layer vs an fp32 evaluation with the same selection
    m.train()
    y, idx = m(x)
    (y.float() ** 2).sum().backward()
    m32 = build(cfg, 0, torch.float32)
    m32.load_state_dict({k: v.float() for k, v in m.state_dict().items()})
    m32.query_proj.norm.load_state_dict(build(cfg, 0, torch.float32).query_proj.norm.state_dict())
    x32 = x.detach().float().requires_grad_(True)
    y32 = _dense_fp32_layer(m32, x32, idx.view(64, -1))
    (y32 ** 2).sum().backward()
    assert rel_err(y.detach().float().cpu().numpy(), y32.detach().cpu().numpy()) < 2e-2
    assert rel_err(x.grad.float().cpu().numpy(), x32.grad.cpu().numpy()) < 2e-2
    assert rel_err(m.keys.grad.float().cpu().numpy(), m32.keys.grad.cpu().numpy()) < 2e-2
    assert rel_err(m.values.weight.grad.float().cpu().numpy(), m32.values.weight.grad.cpu().numpy()) < 2e-2
    wq, wq32 = m.query_proj.query_mlps[0].weight.grad, m32.query_proj.query_mlps[0].weight.grad
    assert rel_err(wq.float().cpu().numpy(), wq32.cpu().numpy()) < 2e-2
    # and the values against the reference output where its selection agrees
    same = (idx.view(64, -1).cpu().numpy() == d["indices"].reshape(64, -1)).all(axis=1)
    if same.any():
        yo = y.detach().float().cpu().numpy().reshape(64, -1)[same]
        assert rel_err(yo, d["out"].reshape(64, -1)[same]) < 2e-2


@pytest.mark.parametrize("fname", sorted(cases.PKM_VARIANTS))
def test_variant_matches_reference(fname):
    """Options beyond the benchmark configs (gate, no query bias, no query
    norm, value projection without SwiLU, no projection, three heads, eval
    mode's ``last_indices`` / ``last_scores``) in fp32 through the kernels
    against the reference's run: indices exactly, outputs and every gradient
    to 1e-5 of each tensor's largest magnitude."""
    torch.backends.cuda.matmul.allow_tf32 = False
    from modelos_b200.pkm.memory import HashingMemory
    kw, _ = cases.PKM_VARIANTS[fname]
    m = HashingMemory(**dict(cases.PKM_VARIANT_BASE, **kw))
    res = cases.run_pkm_variant(m, fname, device=DEV)
    cases.check_pkm_variant(res, np.load(os.path.join(GOLD, fname)), rel_err)


def test_eval_mode_usage_statistics():
    m = build(cases.CONFIG0, 0, torch.float32).eval()
    x = cases.pkm_input((1, 8, 512), 0).to(DEV)
    with torch.no_grad():
        y, idx = m(x)
    li = m.last_indices
    assert li.device.type == "cpu" and li.shape == (8, 4, 32)
    assert torch.equal(li.reshape(8, -1), idx.view(8, -1).cpu())
    assert m.last_scores.dtype == torch.float32


def test_fused_gate_path_equals_default_layer_step():
    """``SwiGLUProjection.FUSE_GATE`` (the gate in the GEMM epilogues) gives
    the same bits as the default (GEMM, then the gate kernel) through a whole
    bf16 layer step: output and every parameter and input gradient (the gate
    projection's bias gradient within a bf16 rounding).  4096
    tokens and 256-wide projections keep every unfused GEMM from splitting K
    (the same summation order)."""
    from modelos_b200.pkm import memory
    cfg = dict(cases.CONFIG2)
    cfg.update(input_dim=256, output_dim=256, mem_v_dim=256, mem_n_keys=64)
    runs = []
    try:
        for fuse in (False, True):
            memory.SwiGLUProjection.FUSE_GATE = fuse
            m = build(cfg, 0, torch.bfloat16)
            x = cases.pkm_input((2, 2048, 256), 0).to(DEV, torch.bfloat16).requires_grad_(True)
            out, _ = m(x)
            (out.float() ** 2).sum().backward()
            got = {"out": out.detach(), "x": x.grad}
            got.update({n: p.grad for n, p in m.named_parameters()})
            runs.append(got)
    finally:
        memory.SwiGLUProjection.FUSE_GATE = False
    torch.cuda.synchronize()
    for name, a in runs[0].items():
        b = runs[1][name]
        if name == "swilu_projection.bias":
            # a column sum of the same dh by another kernel (another order)
            assert rel_err(a.float().cpu().numpy(), b.float().cpu().numpy()) < 2.0 ** -8, name
        else:
            assert torch.equal(a, b), name
