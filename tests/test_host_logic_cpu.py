"""Host-side module logic on CPU, with the kernels replaced by the CPU
stand-in of ``tests/fake_native.py``: autograd wiring of the lookup, the
FwPKM chunk loop, inner updates and double-backward, checked against the
reference's golden outputs.  No GPU and no reference tree needed."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import cases
import fake_native

GOLD = os.path.join(os.path.dirname(__file__), "golden")
FW_KW = cases.FW_KW


def rel_err(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture
def cpu_kernels(monkeypatch):
    fake_native.install(monkeypatch)
    from modelos_b200.pkm import colwise_embedding_bag, xformer_embeddingbag

    def bag(indices, weight, per_sample_weights, mode="sum", bw_algo="reverse_indices"):
        return xformer_embeddingbag.xFormersEmbeddingBag.apply(indices, weight, per_sample_weights, bw_algo)

    monkeypatch.setattr(xformer_embeddingbag, "xformers_embedding_bag", bag)
    monkeypatch.setattr(colwise_embedding_bag, "xformers_embedding_bag", bag)


@pytest.mark.parametrize("score_type,fname", [("dot_product", "fwpkm_dot.npz"), ("idw", "fwpkm_idw.npz")])
def test_fwpkm_chunk_loop_matches_reference(cpu_kernels, score_type, fname):
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    d = np.load(os.path.join(GOLD, fname))
    m = FastWeightProductKeyMemory(qk_score_type=score_type, **FW_KW).train()
    keys, values, q, ref_v = cases.fwpkm_case(0)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    q.requires_grad_(True)
    ref_v.requires_grad_(True)
    res = m(q, ref_v, None, 8)
    ((res["output"] ** 2).sum() + res["addr_loss"]).backward()
    np.testing.assert_array_equal(res["indices"].numpy(), d["indices"])
    for got, key in ((res["output"], "output"), (m.keys, "final_keys"), (m.values, "final_values"),
                     (q.grad, "q_grad"), (ref_v.grad, "ref_v_grad"), (m.keys.grad, "keys_grad"),
                     (m.values.grad, "values_grad"), (res["losses"], "losses")):
        assert rel_err(got.detach().numpy(), d[key]) < 1e-5, key


@pytest.mark.parametrize("fname", sorted(cases.STREAM_FIXTURES))
def test_fwpkm_streaming_matches_reference(cpu_kernels, fname):
    """``forward_w_past`` over three calls carrying the signal queue (gates
    and a loss mask queued too in the variant): outputs, losses, queues and
    fast weights after every call equal the reference's."""
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    d = np.load(os.path.join(GOLD, fname))
    m = FastWeightProductKeyMemory(**dict(FW_KW, **cases.STREAM_FIXTURES[fname][0])).train()
    keys, values, _, _ = cases.fwpkm_case(1)
    q, ref_v, gates, mask = cases.stream_inputs(fname)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    cases.run_stream(m, q, ref_v, d, rel_err, gates=gates, mask=mask)


@pytest.mark.parametrize("fname", sorted(cases.FW_VARIANTS))
def test_fwpkm_variant_matches_reference(cpu_kernels, fname):
    """Non-default options (silu / relu transforms, temperature, keys trained
    by the memorisation loss, clipping, weight decay, no look-ahead, no
    addressing loss, gates, loss mask, a bf16 module) against the
    reference's run."""
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    cases.run_fw_variant(FastWeightProductKeyMemory, FW_KW, fname, np.load(os.path.join(GOLD, fname)), rel_err,
                         tol=cases.FW_VARIANT_TOL[cases.FW_VARIANTS[fname][3]])


def test_fwpkm_without_addressing_loss_keeps_keys(cpu_kernels):
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    m = FastWeightProductKeyMemory(addr_loss=None, **FW_KW).train()
    keys, values, q, ref_v = cases.fwpkm_case(0)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    res = m(q, ref_v, None, 8)
    assert res["addr_loss"] is None
    assert torch.equal(m.keys.detach(), keys)
    assert not torch.equal(m.values.detach(), values)


@pytest.mark.parametrize("fname", sorted(cases.PKM_VARIANTS))
def test_hashing_memory_variant_matches_reference(cpu_kernels, fname):
    """``HashingMemory`` options beyond the benchmark configs (gate, no query
    bias, no query norm, value projection without SwiLU, no projection,
    three heads, eval mode) against the reference's run."""
    from modelos_b200.pkm.memory import HashingMemory
    kw, _ = cases.PKM_VARIANTS[fname]
    m = HashingMemory(**dict(cases.PKM_VARIANT_BASE, **kw))
    cases.check_pkm_variant(cases.run_pkm_variant(m, fname), np.load(os.path.join(GOLD, fname)), rel_err)


def test_hashing_memory_config0_matches_reference(cpu_kernels):
    from modelos_b200.pkm.memory import HashingMemory
    c0 = np.load(os.path.join(GOLD, "c0_pkm.npz"))
    m = HashingMemory(**cases.CONFIG0)
    m.load_state_dict(cases.pkm_state(cases.CONFIG0, 0))
    x = cases.pkm_input((2, 128, 512), 0).requires_grad_(True)
    y, idx = m(x)
    (y ** 2).sum().backward()
    np.testing.assert_array_equal(idx.numpy(), c0["indices"])
    assert rel_err(y.detach().numpy(), c0["out"]) < 1e-5
    assert rel_err(x.grad.numpy(), c0["x_grad"]) < 1e-5
    assert rel_err(m.keys.grad.numpy(), c0["keys_grad"]) < 1e-5
    assert rel_err(m.values.weight.grad.norm(dim=1).numpy(), c0["values_grad_rownorm"]) < 1e-5


def test_product_path_refuses_cpu_tensors():
    from modelos_b200.pkm.xformer_embeddingbag import xformers_embedding_bag
    with pytest.raises(RuntimeError, match="CUDA"):
        xformers_embedding_bag(torch.zeros(2, 3, dtype=torch.long), torch.zeros(4, 16), torch.ones(2, 3))


# ---------------------------------------------------------------------------
# benchmarked geometries with the selection pinned to the reference's
# (``tests/pinned.py``); the kernels are the CPU stand-ins
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("score_type,fname", [("dot_product", "fwpkm_c4_dot.npz"), ("idw", "fwpkm_c4_idw.npz")])
def test_fwpkm_config4_geometry_pinned_matches_reference(cpu_kernels, monkeypatch, score_type, fname):
    from pinned import check_summary, pin_fwpkm_selection

    from modelos_b200 import _native
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    d = np.load(os.path.join(GOLD, fname))
    calls = pin_fwpkm_selection(monkeypatch, _native, torch.from_numpy(d["indices"].astype(np.int64)),
                                cases.FW_C4_CHUNK)
    m = FastWeightProductKeyMemory(qk_score_type=score_type, **cases.FW_C4).train()
    keys, values, q, ref_v = cases.fwpkm_c4_case(0)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    q.requires_grad_(True)
    ref_v.requires_grad_(True)
    res = m(q, ref_v, None, cases.FW_C4_CHUNK)
    ((res["output"] ** 2).sum() + res["addr_loss"]).backward()
    assert calls[0] == 2
    T = q.shape[1]
    assert rel_err(res["output"].detach().numpy(), d["output"]) < 1e-5
    assert rel_err(res["losses"].numpy(), d["losses"]) < 1e-5
    for t, key in ((m.keys.detach(), "final_keys"), (m.values.detach() - values, "values_delta"),
                   (q.grad.view(T, -1), "q_grad"), (ref_v.grad.view(T, -1), "ref_v_grad"),
                   (m.keys.grad, "keys_grad"), (m.values.grad, "values_grad")):
        check_summary(t, d, key, 1e-5)


def test_hashing_memory_config2_geometry_pinned_matches_reference(cpu_kernels, monkeypatch):
    """The bf16 layer at config-2 geometry on one 2048-token sequence (the
    query batch norm is torch's on CPU here; on the GPU it is the library's)."""
    import torch.nn.functional as F
    from pinned import check_summary, pin_pkm_selection

    from modelos_b200 import _native
    from modelos_b200.pkm import memory as mem
    d = np.load(os.path.join(GOLD, "c2_full_bf16.npz"))

    def torch_bn(self, x):
        return F.batch_norm(x, self.running_mean, self.running_var, self.weight, self.bias, True, self.momentum,
                            self.eps)

    monkeypatch.setattr(mem.QueryBatchNorm, "forward", torch_bn)
    pin_pkm_selection(monkeypatch, _native, torch.from_numpy(d["indices"].astype(np.int64)).view(-1, 32))
    m = mem.HashingMemory(**cases.CONFIG2)
    m.load_state_dict(cases.pkm_state(cases.CONFIG2, 0))
    m = m.bfloat16().train()
    x = cases.pkm_input((1, 2048, 1024), 0).bfloat16().requires_grad_(True)
    y, _ = m(x)
    loss = (y.float() ** 2).sum()
    loss.backward()
    assert abs(loss.item() - float(d["loss"])) <= 2e-2 * abs(float(d["loss"]))
    check_summary(y.view(2048, -1).float(), d, "out", 2e-2)
    check_summary(x.grad.view(2048, -1).float(), d, "x_grad", 2e-2)
    check_summary(m.values.weight.grad.float(), d, "values_grad", 2e-2)
    check_summary(m.query_proj.query_mlps[0].weight.grad.float(), d, "wq_grad", 2e-2)
    kg = cases.from_bf16_bits(d["keys_grad"]).float().numpy()
    assert rel_err(m.keys.grad.float().numpy(), kg) < 2e-2
