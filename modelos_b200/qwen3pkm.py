"""Qwen3 with product-key memory layers (the consumer of the PKM path).

The reference's ``modeling_qwen3pkm.py`` builds a Qwen3 decoder whose layers
listed in ``config.pkm_layers`` replace the feed-forward block with a
``HashingMemory`` read (``modeling_qwen3pkm.py:318-333``): after the
post-attention RMSNorm the layer computes ``pkm(hidden)[0]`` instead of
``mlp(hidden)`` and adds it to the residual (``:699-707``).  Its memory is
built as ``HashingMemory(hidden, hidden, mem_k_dim=pkm_k_dim,
mem_v_dim=pkm_v_dim, mem_heads=pkm_heads, mem_knn=pkm_topk,
mem_n_keys=pkm_n_subkeys, mem_share_values=False,
mem_query_rmsnorm=pkm_query_rmsnorm)`` and re-initialised with
``reset_parameters`` (``:733-737``).

This module assembles the same network from transformers' own Qwen3 blocks
(``Qwen3ForCausalLM``) with this package's ``HashingMemory`` in those
positions, so the benchmark machine (which has transformers but not the
reference tree) can run the model: a training step, a prefill and a decode
loop.  ``reference_state_dict_names`` maps parameter names between this
assembly and the reference model (``layers.i.pkm.*`` there,
``layers.i.mlp.pkm.*`` here), which is how the CPU test checks the two give
the same logits from the same weights.
"""
from __future__ import annotations

from typing import Iterable, Optional

import torch
from torch import nn

from .pkm.memory import HashingMemory

# Benchmark config 3: a Qwen3-0.6B-shaped decoder with PKM layers of the
# config-2 geometry at layers 6, 12 and 18.
CONFIG3 = dict(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
               num_attention_heads=16, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6,
               rope_theta=1_000_000.0, max_position_embeddings=40960, tie_word_embeddings=True)
PKM3 = dict(pkm_layers=(6, 12, 18), pkm_k_dim=512, pkm_v_dim=1024, pkm_heads=4, pkm_topk=32, pkm_n_subkeys=512,
            pkm_query_rmsnorm=True)


class PKMFeedForward(nn.Module):
    """The feed-forward slot of a PKM layer: ``HashingMemory(hidden)[0]``; the
    memory's indices of the last call stay in ``last_pkm_indices``."""

    def __init__(self, hidden: int, pkm_k_dim: int, pkm_v_dim: int, pkm_heads: int, pkm_topk: int,
                 pkm_n_subkeys: int, pkm_query_rmsnorm: bool):
        super().__init__()
        self.pkm = HashingMemory(input_dim=hidden, output_dim=hidden, mem_k_dim=pkm_k_dim, mem_v_dim=pkm_v_dim,
                                 mem_heads=pkm_heads, mem_knn=pkm_topk, mem_n_keys=pkm_n_subkeys,
                                 mem_share_values=False, mem_query_rmsnorm=pkm_query_rmsnorm)
        self.last_pkm_indices = None

    def forward(self, x):
        out, idx = self.pkm(x)
        self.last_pkm_indices = idx
        return out


def build_qwen3_pkm(model_kw: Optional[dict] = None, pkm_kw: Optional[dict] = None,
                    attn_implementation: str = "sdpa", dtype=torch.bfloat16, device=None, seed: int = 0):
    """A ``Qwen3ForCausalLM`` (random init) whose ``pkm_layers`` carry a
    ``PKMFeedForward`` in place of the MLP, re-initialised like the
    reference (``reset_parameters`` of every memory)."""
    from transformers import Qwen3Config, Qwen3ForCausalLM

    mk = dict(CONFIG3)
    mk.update(model_kw or {})
    pk = dict(PKM3)
    pk.update(pkm_kw or {})
    layers: Iterable[int] = pk.pop("pkm_layers")
    cfg = Qwen3Config(**mk)
    cfg._attn_implementation = attn_implementation
    torch.manual_seed(seed)
    model = Qwen3ForCausalLM(cfg)
    for i in layers:
        ff = PKMFeedForward(mk["hidden_size"], **pk)
        ff.pkm.reset_parameters()
        model.model.layers[i].mlp = ff
    return model.to(device=device, dtype=dtype)


def reference_state_dict_names(name: str) -> str:
    """This assembly's parameter name for a name of the reference model
    (``model.layers.i.pkm.*`` -> ``model.layers.i.mlp.pkm.*``)."""
    parts = name.split(".")
    if len(parts) > 3 and parts[0] == "model" and parts[1] == "layers" and parts[3] == "pkm":
        return ".".join(parts[:3] + ["mlp"] + parts[3:])
    return name
