"""The config-3 model assembly (``modelos_b200.qwen3pkm``: transformers'
Qwen3 blocks with this package's ``HashingMemory`` in the PKM layers' feed-
forward slot) computes the same network as the reference's
``modeling_qwen3pkm.py`` (``:302-333, 699-707``).

The reference model runs on CPU over its own ``pkm`` package; the assembly
runs on CPU with the kernels replaced by the CPU stand-ins of
``tests/fake_native.py``.  Both load the same weights (the reference's state
dict through ``reference_state_dict_names``) and must give the same logits,
loss and gradients (fp32, 1e-5 normwise).  Skipped without the reference tree.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import fake_native
import refmodel

pytestmark = pytest.mark.skipif(not refmodel.available(), reason="reference tree not present")

TINY_MODEL = dict(vocab_size=96, hidden_size=64, intermediate_size=128, num_hidden_layers=3, num_attention_heads=2,
                  num_key_value_heads=1, head_dim=32, max_position_embeddings=128, rms_norm_eps=1e-6,
                  rope_theta=1_000_000.0, tie_word_embeddings=False)
TINY_PKM = dict(pkm_layers=[1], pkm_k_dim=32, pkm_v_dim=48, pkm_heads=2, pkm_topk=4, pkm_n_subkeys=8,
                pkm_query_rmsnorm=True)


def rel_err(a, b):
    a = a.detach().double().numpy()
    b = b.detach().double().numpy()
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("rmsnorm", [True, False])
def test_assembly_matches_reference_model(monkeypatch, rmsnorm):
    from modelos_b200 import qwen3pkm
    from modelos_b200.pkm import colwise_embedding_bag, xformer_embeddingbag
    fake_native.install(monkeypatch)

    def bag(indices, weight, per_sample_weights, mode="sum", bw_algo="reverse_indices"):
        return xformer_embeddingbag.xFormersEmbeddingBag.apply(indices, weight, per_sample_weights, bw_algo)

    monkeypatch.setattr(xformer_embeddingbag, "xformers_embedding_bag", bag)
    monkeypatch.setattr(colwise_embedding_bag, "xformers_embedding_bag", bag)
    ref_mod = refmodel.load("refmodel_refpkg", ours=False)
    pkm_kw = dict(TINY_PKM, pkm_query_rmsnorm=rmsnorm)
    cfg = ref_mod.Qwen3PKMConfig(**TINY_MODEL, **pkm_kw)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    ref = ref_mod.Qwen3PKMForCausalLM(cfg).float().train()
    ours = qwen3pkm.build_qwen3_pkm(TINY_MODEL, pkm_kw, attn_implementation="eager", dtype=torch.float32,
                                    device="cpu").train()
    sd = {qwen3pkm.reference_state_dict_names(k): v for k, v in ref.state_dict().items()}
    ours.load_state_dict(sd, strict=True)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, TINY_MODEL["vocab_size"], (2, 24), generator=g)
    out_r = ref(input_ids=ids, labels=ids, use_cache=False)
    out_o = ours(input_ids=ids, labels=ids, use_cache=False)
    assert rel_err(out_o.logits, out_r.logits) < 1e-5
    assert abs(out_o.loss.item() - out_r.loss.item()) <= 1e-5 * abs(out_r.loss.item())
    out_r.loss.backward()
    out_o.loss.backward()
    named_o = dict(ours.named_parameters())
    for name, p in ref.named_parameters():
        if p.grad is None:
            continue
        q = named_o[qwen3pkm.reference_state_dict_names(name)]
        assert rel_err(q.grad, p.grad) < 1e-5, name
    # the memory layer's indices equal the reference layer's
    pkm_r = ref.model.layers[1].pkm
    assert isinstance(ours.model.layers[1].mlp, qwen3pkm.PKMFeedForward)
    assert ours.model.layers[1].mlp.last_pkm_indices.shape == (2, 24, pkm_kw["pkm_heads"] * pkm_kw["pkm_topk"])
    assert pkm_r is not None
