"""The config-3 model assembly (``modelos_b200.qwen3pkm``) on the GPU kernels.

* A tiny model in fp32: logits, loss and gradients on the GPU equal the same
  model on CPU with the kernels replaced by the CPU stand-ins (which
  ``tests/test_qwen3pkm_cpu.py`` ties to the reference's model file).
* A training step, a prefill and a few cached decode steps of a bf16 model
  with the config-2 memory geometry run, stay finite and reach the memory's
  parameters.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import fake_native

pytestmark = pytest.mark.gpu
DEV = "cuda"
TINY_MODEL = dict(vocab_size=96, hidden_size=64, intermediate_size=128, num_hidden_layers=3, num_attention_heads=2,
                  num_key_value_heads=1, head_dim=32, max_position_embeddings=128, tie_word_embeddings=False)
TINY_PKM = dict(pkm_layers=[1], pkm_k_dim=32, pkm_v_dim=48, pkm_heads=2, pkm_topk=4, pkm_n_subkeys=8)


def rel_err(a, b):
    a = a.detach().double().cpu().numpy()
    b = b.detach().double().cpu().numpy()
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def test_assembly_on_gpu_equals_cpu_stand_ins(monkeypatch):
    torch.backends.cuda.matmul.allow_tf32 = False
    from modelos_b200 import qwen3pkm
    gpu = qwen3pkm.build_qwen3_pkm(TINY_MODEL, TINY_PKM, attn_implementation="eager", dtype=torch.float32,
                                   device=DEV).train()
    ids = torch.randint(0, 96, (2, 24), generator=torch.Generator().manual_seed(1))
    out_g = gpu(input_ids=ids.to(DEV), labels=ids.to(DEV), use_cache=False)
    out_g.loss.backward()
    torch.cuda.synchronize()
    # the same weights on CPU with the stand-in kernels
    from modelos_b200.pkm import colwise_embedding_bag, xformer_embeddingbag
    fake_native.install(monkeypatch)

    def bag(indices, weight, per_sample_weights, mode="sum", bw_algo="reverse_indices"):
        return xformer_embeddingbag.xFormersEmbeddingBag.apply(indices, weight, per_sample_weights, bw_algo)

    monkeypatch.setattr(xformer_embeddingbag, "xformers_embedding_bag", bag)
    monkeypatch.setattr(colwise_embedding_bag, "xformers_embedding_bag", bag)
    cpu = qwen3pkm.build_qwen3_pkm(TINY_MODEL, TINY_PKM, attn_implementation="eager", dtype=torch.float32,
                                   device="cpu").train()
    cpu.load_state_dict({k: v.cpu() for k, v in gpu.state_dict().items()}, strict=True)
    out_c = cpu(input_ids=ids, labels=ids, use_cache=False)
    out_c.loss.backward()
    assert rel_err(out_g.logits, out_c.logits) < 1e-5
    assert abs(out_g.loss.item() - out_c.loss.item()) <= 1e-5 * abs(out_c.loss.item())
    gp = dict(gpu.named_parameters())
    for name, p in cpu.named_parameters():
        assert rel_err(gp[name].grad, p.grad) < 1e-5, name


def test_config3_memory_geometry_trains_prefills_and_decodes():
    """Two decoder layers of the config-3 width with a config-2-geometry memory
    in bf16: a training step reaches the memory's parameters, and a prefill
    plus 8 cached decode steps give the same next tokens as recomputing the
    whole prefix."""
    from modelos_b200 import _native, qwen3pkm
    model = qwen3pkm.build_qwen3_pkm(dict(num_hidden_layers=2, vocab_size=4096), dict(pkm_layers=[1]),
                                     device=DEV, dtype=torch.bfloat16).train()
    g = torch.Generator(device=DEV).manual_seed(0)
    ids = torch.randint(0, 4096, (2, 256), generator=g, device=DEV)
    out = model(input_ids=ids, labels=ids, use_cache=False)
    out.loss.backward()
    torch.cuda.synchronize()
    _native.check_device_errors()
    pkm = model.model.layers[1].mlp.pkm
    assert torch.isfinite(out.loss) and pkm.values.weight.grad.abs().max() > 0 and pkm.keys.grad.abs().max() > 0
    model.eval()
    with torch.no_grad():
        pre = model(input_ids=ids, use_cache=True)
        cache, nxt = pre.past_key_values, pre.logits[:, -1].argmax(-1, keepdim=True)
        seq = torch.cat([ids, nxt], 1)
        for _ in range(8):
            o = model(input_ids=nxt, past_key_values=cache, use_cache=True)
            cache, nxt = o.past_key_values, o.logits[:, -1].argmax(-1, keepdim=True)
            seq = torch.cat([seq, nxt], 1)
        full = model(input_ids=seq[:, :-1], use_cache=False).logits
    assert torch.isfinite(full.float()).all()
    # cached and recomputed last-position logits agree within bf16 rounding
    assert rel_err(o.logits[:, -1].float(), full[:, -1].float()) < 5e-2
