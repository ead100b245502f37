"""The reference's Qwen3-PKM model file runs its constructors on this package.

``modeling_qwen3pkm.py`` imports ``HashingMemory`` (``:22``),
``FastWeightProductKeyMemory`` and ``l2norm`` (``:23``) and ``FastWeightMLP``
(``:24``) from its sibling ``pkm`` / ``fwpkm`` packages, builds them from its
config (``:319-390``) and re-initialises them through ``reset_parameters``
from ``_init_weights`` (``:733-737``).  These tests import that file twice
from the reference tree, once over the reference's own packages and once
with this package's ``pkm`` / ``fwpkm`` standing in for them, build the same
small model from the same seed, and require identical state dicts: same
keys, shapes, dtypes and values.  The forward needs a GPU and the reference
tree together, so it is not run here.

Without the reference tree (``tests/refmodel.py`` finds it) the tests skip.
"""
from __future__ import annotations

import pytest
import torch

import refmodel

pytestmark = pytest.mark.skipif(not refmodel.available(), reason="reference tree not present")


def _tiny_config(cfg_cls, **over):
    kw = dict(vocab_size=96, hidden_size=64, intermediate_size=128, num_hidden_layers=3,
              num_attention_heads=2, num_key_value_heads=1, head_dim=32, max_position_embeddings=128,
              pkm_layers=[1], pkm_k_dim=32, pkm_v_dim=48, pkm_heads=2, pkm_topk=4, pkm_n_subkeys=8,
              fwpkm_layers=[0, 2], fwpkm_k_dim=16, fwpkm_v_dim=32, fwpkm_heads=2, fwpkm_topk=4,
              fwpkm_n_subkeys=8)
    kw.update(over)
    return cfg_cls(**kw)


@pytest.fixture(scope="module")
def models():
    return refmodel.load("refmodel_refpkg", ours=False), refmodel.load("refmodel_b200pkg", ours=True)


@pytest.mark.parametrize("over", [
    {},
    {"pkm_query_rmsnorm": False},
    {"fwpkm_qk_score_type": "dot_product", "fwpkm_out_fuse_gate": False},
], ids=["defaults", "no_rmsnorm", "dot_product"])
def test_model_builds_identically(models, over):
    ref_mod, our_mod = models
    built = []
    for mod in (ref_mod, our_mod):
        cfg = _tiny_config(mod.Qwen3PKMConfig, **over)
        torch.manual_seed(0)
        built.append(mod.Qwen3PKMForCausalLM(cfg))
    ref, ours = built
    import modelos_b200.fwpkm.fwpkm as fw
    import modelos_b200.pkm.memory as mem
    assert isinstance(ours.model.layers[1].pkm, mem.HashingMemory)
    assert isinstance(ours.model.layers[0].fwpkm, fw.FastWeightProductKeyMemory)
    sd_ref, sd_ours = ref.state_dict(), ours.state_dict()
    assert list(sd_ref) == list(sd_ours)
    for k in sd_ref:
        a, b = sd_ref[k], sd_ours[k]
        assert a.shape == b.shape and a.dtype == b.dtype, k
        assert torch.equal(a, b), k
    # and the state dict loads strictly in both directions
    ours.load_state_dict(sd_ref, strict=True)
    ref.load_state_dict(sd_ours, strict=True)


def test_mlp_variant_raises(models):
    _, our_mod = models
    cfg = _tiny_config(our_mod.Qwen3PKMConfig, fwpkm_variant="mlp", fwpkm_heads=1)
    with pytest.raises(NotImplementedError):
        our_mod.Qwen3PKMForCausalLM(cfg)
