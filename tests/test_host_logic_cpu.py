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
FW_KW = dict(mem_k_dim=16, mem_v_dim=32, mem_heads=2, mem_topk=4, mem_n_subkeys=16, lookahead=1,
             learning_rate=0.1)


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


@pytest.mark.parametrize("score_type,fname", [("dot_product", "fwpkm_stream_dot.npz"),
                                              ("idw", "fwpkm_stream_idw.npz")])
def test_fwpkm_streaming_matches_reference(cpu_kernels, score_type, fname):
    """``forward_w_past`` over three calls carrying the signal queue: outputs,
    losses, queues and fast weights after every call equal the reference's."""
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    d = np.load(os.path.join(GOLD, fname))
    m = FastWeightProductKeyMemory(qk_score_type=score_type, **FW_KW).train()
    keys, values, q, ref_v = cases.fwpkm_case(1)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    cases.run_stream(m, q, ref_v, d, rel_err)


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
