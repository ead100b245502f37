"""Generate the golden fixtures in this folder from the reference itself.

Run in a container that has the reference tree (read-only) at
``$MODELOS_REF`` (default: a ``reference`` folder beside this repository)::

    python tests/golden/make_golden.py

The reference's ``pkm/`` and ``fwpkm/`` packages are imported in place
through a synthetic namespace package (no file is written into the reference
tree) and run on CPU, which is their stock path: ``F.embedding_bag`` for the
PKM bag (``pkm/xformer_embeddingbag.py:436-437``) and the torch gather plus
``_embedding_bag_bw_native`` for FwPKM
(``fwpkm/xformer_embeddingbag_legacy.py:177-178``).  Inputs come from
``tests/cases.py`` so the GPU tests can regenerate them without the reference.
"""
from __future__ import annotations

import importlib
import os
import sys
import types

sys.dont_write_bytecode = True
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import numpy as np  # noqa: E402
import torch  # noqa: E402

import cases  # noqa: E402

REF = os.environ.get("MODELOS_REF",
                     os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))), "reference"))


def _import_ref():
    pkg = types.ModuleType("refmodelos")
    pkg.__path__ = [REF]
    sys.modules["refmodelos"] = pkg
    mem = importlib.import_module("refmodelos.pkm.memory")
    xeb = importlib.import_module("refmodelos.pkm.xformer_embeddingbag")
    fw = importlib.import_module("refmodelos.fwpkm.fwpkm")
    gw = importlib.import_module("refmodelos.fwpkm.xformer_embeddingbag_grad_wrapper")
    leg = importlib.import_module("refmodelos.fwpkm.xformer_embeddingbag_legacy")
    return mem, xeb, fw, gw, leg


def _np(t):
    t = t.detach()
    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.cpu().numpy()


def _rows_summary(prefix, t, out, nsample=64, seed=0):
    """Row norms of a big gradient plus a few full rows, to keep fixtures small."""
    t = t.detach().double()
    out[prefix + "_rownorm"] = t.norm(dim=1).numpy()
    g = np.random.default_rng(seed)
    rows = np.sort(g.choice(t.shape[0], size=min(nsample, t.shape[0]), replace=False))
    out[prefix + "_rows_idx"] = rows
    out[prefix + "_rows"] = t[torch.from_numpy(rows)].numpy()


def gen_pkm(mem, cfg, name, batch_shape, dtype, seed=0):
    torch.manual_seed(0)
    m = mem.HashingMemory(**cfg)
    st = cases.pkm_state(cfg, seed)
    m.load_state_dict(st)
    m = m.to(dtype).train()
    x = cases.pkm_input(batch_shape, seed).to(dtype).requires_grad_(True)
    out = {}
    out["param_checksums"] = np.stack([cases.checksum(st[k]) for k in sorted(st)])
    out["x_checksum"] = cases.checksum(x)
    # query and get_indices on their own (no grad)
    with torch.no_grad():
        q = m.query_proj(x.view(-1, cfg["input_dim"]))
        s, i = m.get_indices(q, cfg["mem_knn"])
    out["query"] = _np(q)
    out["gi_scores"] = _np(s)
    out["gi_indices"] = i.numpy()
    y, idx = m(x)
    loss = (y.float() ** 2).sum()
    loss.backward()
    out["out"] = _np(y)
    out["indices"] = idx.numpy()
    out["loss"] = np.array(loss.item())
    out["x_grad"] = _np(x.grad)
    out["keys_grad"] = _np(m.keys.grad)
    _rows_summary("values_grad", m.values.weight.grad.float(), out)
    _rows_summary("wq_grad", m.query_proj.query_mlps[0].weight.grad.float(), out)
    out["bq_grad"] = _np(m.query_proj.query_mlps[0].bias.grad)
    out["value_proj_w_grad_norm"] = np.array(m.value_proj.weight.grad.float().norm().item())
    np.savez_compressed(os.path.join(HERE, name), **out)
    print("wrote", name)


def gen_pkm_variant(mem, name):
    kw, _ = cases.PKM_VARIANTS[name]
    torch.manual_seed(0)
    m = mem.HashingMemory(**dict(cases.PKM_VARIANT_BASE, **kw))
    res = cases.run_pkm_variant(m, name)
    np.savez_compressed(os.path.join(HERE, name),
                        **{k: (v.numpy() if v.dtype == torch.long else _np(v)) for k, v in res.items()})
    print("wrote", name)


def gen_indices_seeds(mem, name, seeds=(1, 2)):
    cfg = cases.CONFIG0
    out = {}
    for sd in seeds:
        torch.manual_seed(0)
        m = mem.HashingMemory(**cfg)
        m.load_state_dict(cases.pkm_state(cfg, sd))
        g = torch.Generator().manual_seed(40_000 + sd)
        q = torch.randn((256 * cfg["mem_heads"], cfg["mem_k_dim"]), generator=g)
        with torch.no_grad():
            s, i = m.get_indices(q, cfg["mem_knn"])
        out[f"s{sd}_q_checksum"] = cases.checksum(q)
        out[f"s{sd}_scores"] = _np(s)
        out[f"s{sd}_indices"] = i.numpy()
    np.savez_compressed(os.path.join(HERE, name), **out)
    print("wrote", name)


def gen_ties(mem, name):
    """Quantised queries/keys so that many scores tie exactly."""
    cfg = dict(cases.CONFIG0)
    cfg.update(mem_n_keys=32, mem_knn=8, mem_k_dim=16)
    torch.manual_seed(0)
    m = mem.HashingMemory(**cfg)
    g = torch.Generator().manual_seed(50_000)
    keys = torch.randint(-1, 2, m.keys.shape, generator=g).float() * 0.25
    q = torch.randint(-1, 2, (64 * cfg["mem_heads"], cfg["mem_k_dim"]), generator=g).float() * 0.5
    with torch.no_grad():
        m.keys.copy_(keys)
        s, i = m.get_indices(q, cfg["mem_knn"])
    np.savez_compressed(os.path.join(HERE, name), keys=keys.numpy(), q=q.numpy(),
                        scores=_np(s), indices=i.numpy(), n_keys=32, knn=8, heads=cfg["mem_heads"])
    print("wrote", name)


EMB_CASES = {
    # name: (B, L, K, D, dtype, heads, seed, hot)
    "f32_small": (64, 16, 512, 64, torch.float32, 1, 1, False),
    "f32_ragged": (37, 7, 100, 48, torch.float32, 1, 2, False),
    "f32_hot": (50, 20, 64, 32, torch.float32, 1, 3, True),
    "f32_L1": (5, 1, 8, 16, torch.float32, 1, 4, False),
    "bf16_c1like": (96, 128, 4096, 128, torch.bfloat16, 4, 5, False),
}


def gen_embbag(xeb, gw, leg, name):
    out = {}
    for cname, (B, L, K, D, dt, heads, sd, hot) in EMB_CASES.items():
        idx, psw, W, gout = cases.embbag_case(B, L, K, D, seed=sd, heads=heads)
        if hot:  # few distinct rows, long segments
            idx = idx % 5
        W = W.to(dt)
        psw = psw.to(dt)
        gout = gout.to(dt)
        # PKM module path: xformers_embedding_bag -> F.embedding_bag on CPU
        Wp = W.clone().requires_grad_(True)
        pp = psw.clone().requires_grad_(True)
        y = xeb.xformers_embedding_bag(idx, Wp, pp, mode="sum")
        y.backward(gout)
        # FwPKM first-order kernel (CPU path) and the double-backward wrapper
        dW_n, dp_n = leg.embedding_bag_bw_rev_indices(idx, W, psw, gout)
        g2 = torch.Generator().manual_seed(60_000 + sd)
        gbar = torch.randn((K, D), generator=g2).to(dt)
        Wf = W.clone().requires_grad_(True)
        pf = psw.clone().requires_grad_(True)
        go = gout.clone().requires_grad_(True)
        yf = gw.xformers_embedding_bag(idx, Wf, pf)
        (dWf,) = torch.autograd.grad(yf, Wf, grad_outputs=go, create_graph=True)
        dgo, dpf = torch.autograd.grad((dWf * gbar).sum(), (go, pf))
        pre = f"{cname}__"
        out[pre + "idx"] = idx.numpy()
        out[pre + "psw"] = _np(psw)
        out[pre + "W"] = _np(W)
        out[pre + "g"] = _np(gout)
        out[pre + "gbar"] = _np(gbar)
        out[pre + "bf16"] = np.array(dt == torch.bfloat16)
        out[pre + "out"] = _np(y)
        out[pre + "dW"] = _np(Wp.grad)
        out[pre + "dpsw"] = _np(pp.grad)
        out[pre + "dW_native"] = _np(dW_n)
        out[pre + "dpsw_native"] = _np(dp_n)
        out[pre + "out_fw"] = _np(yf)
        out[pre + "bw2_dg"] = _np(dgo)
        out[pre + "bw2_da"] = _np(dpf)
    np.savez_compressed(os.path.join(HERE, name), **out)
    print("wrote", name)


FW_KW = cases.FW_KW


def gen_fwpkm(fw, name, score_type, seed=0):
    torch.manual_seed(0)
    m = fw.FastWeightProductKeyMemory(qk_score_type=score_type, **FW_KW).train()
    keys, values, q, ref_v = cases.fwpkm_case(seed)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    q = q.clone().requires_grad_(True)
    ref_v = ref_v.clone().requires_grad_(True)
    res = m(q, ref_v, None, 8)
    loss = (res["output"] ** 2).sum() + res["addr_loss"]
    loss.backward()
    out = {
        "output": _np(res["output"]),
        "indices": res["indices"].numpy(),
        "scores": _np(res["scores"]),
        "losses": _np(res["losses"]),
        "addr_loss": np.array(res["addr_loss"].item()),
        "grad_norms": np.array([g.item() for g in res["grad_norms"]]),
        "final_keys": _np(m.keys),
        "final_values": _np(m.values),
        "q_grad": _np(q.grad),
        "ref_v_grad": _np(ref_v.grad),
        "keys_grad": _np(m.keys.grad),
        "values_grad": _np(m.values.grad),
        "loss": np.array(loss.item()),
    }
    np.savez_compressed(os.path.join(HERE, name), **out)
    print("wrote", name)


def gen_fwpkm_variant(fw, gw, name):
    """The reference's first-order bag backward (``bw_kernel`` of
    ``fwpkm/xformer_embeddingbag_grad_wrapper.py:131``) is a Triton kernel on
    CUDA (``fwpkm/xformer_embeddingbag_legacy.py:177-220``): its score-weight
    gradient carries no autograd graph.  Its CPU stand-in
    (``_embedding_bag_bw_native``, ``:147-167``) computes that gradient in
    torch ops, which under a ``create_graph`` backward do build a graph, so
    with ``mem_grad_to_values_only=False`` a CPU run gains second-order terms
    the CUDA path does not have.  These fixtures run the stand-in under
    ``no_grad`` to follow the CUDA path, as that function's own docstring
    says it runs."""
    kw, with_gates, with_mask, dt = cases.FW_VARIANTS[name]
    orig_bw = gw.embedding_bag_bw_rev_indices
    gw.embedding_bag_bw_rev_indices = torch.no_grad()(orig_bw)
    try:
        _gen_fwpkm_variant(fw, name, kw, with_gates, with_mask, torch.bfloat16 if dt == "bf16" else torch.float32)
    finally:
        gw.embedding_bag_bw_rev_indices = orig_bw


def _gen_fwpkm_variant(fw, name, kw, with_gates, with_mask, dt):
    torch.manual_seed(0)
    m = fw.FastWeightProductKeyMemory(**dict(FW_KW, **kw)).to(dt).train()
    keys, values, q, ref_v = (t.to(dt) for t in cases.fwpkm_case(2))
    gates, mask = (None if t is None else t.to(dt)
                   for t in cases.fw_variant_inputs(q.shape[0], q.shape[1], with_gates, with_mask))
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    q = q.clone().requires_grad_(True)
    ref_v = ref_v.clone().requires_grad_(True)
    res = m(q, ref_v, gates, 8, loss_mask=mask)
    loss = (res["output"] ** 2).sum()
    if res["addr_loss"] is not None:
        loss = loss + res["addr_loss"]
    loss.backward()
    out = {
        "output": _np(res["output"]),
        "indices": res["indices"].numpy(),
        "losses": _np(res["losses"]),
        "final_keys": _np(m.keys),
        "final_values": _np(m.values),
        "q_grad": _np(q.grad),
        "ref_v_grad": _np(ref_v.grad),
        "values_grad": _np(m.values.grad),
    }
    if m.keys.grad is not None:
        out["keys_grad"] = _np(m.keys.grad)
    if res["addr_loss"] is not None:
        out["addr_loss"] = np.array(res["addr_loss"].item())
    np.savez_compressed(os.path.join(HERE, name), **out)
    print("wrote", name)


def gen_fwpkm_stream(fw, name, seed=1):
    """``forward_w_past`` (``fwpkm/fwpkm.py:560-820``) over three successive
    calls that carry the signal queue: the first only queues, the second
    updates once and queues the rest, the third updates again.  Run under
    ``no_grad`` as in generation, with token ids (the reference's queue pop
    indexes them when ``lookahead > 0``), and with the gates and loss mask
    the fixture's entry in ``cases.STREAM_FIXTURES`` asks for."""
    kw, _, _ = cases.STREAM_FIXTURES[name]
    torch.manual_seed(0)
    m = fw.FastWeightProductKeyMemory(**dict(FW_KW, **kw)).train()
    keys, values, _, _ = cases.fwpkm_case(seed)
    q, ref_v, gates, mask = cases.stream_inputs(name, seed)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    out = {}
    for c, res, past in cases.stream_calls(m, q, ref_v, gates, mask):
        out[f"c{c}_output"] = _np(res["output"])
        out[f"c{c}_indices"] = res["indices"].numpy()
        out[f"c{c}_scores"] = _np(res["scores"])
        out[f"c{c}_updated"] = np.array(res["losses"] is not None)
        if res["losses"] is not None:
            out[f"c{c}_losses"] = _np(res["losses"])
            out[f"c{c}_addr_loss"] = np.array(res["addr_loss"].item())
        for k, t in zip(("q", "hyp", "ref", "gates", "mask"), past[:5]):
            if t is not None:
                out[f"c{c}_past_{k}"] = _np(t)
        out[f"c{c}_past_ids"] = past[5].numpy()
        # copies: the module updates its parameters in place
        out[f"c{c}_keys"] = _np(m.keys).copy()
        out[f"c{c}_values"] = _np(m.values).copy()
    np.savez_compressed(os.path.join(HERE, name), **out)
    print("wrote", name)


def _put_summary(out, prefix, t, nonzero_rows=False, f32=False):
    s = cases.summarize(t, nonzero_rows=nonzero_rows)
    for k, v in s.items():
        if f32 and k in ("rownorm", "proj"):
            v = v.astype(np.float32)
        out[f"{prefix}_{k}"] = v


C2_FULL_TOKENS = 2048   # one 2048-position sequence of the config-2 batch
C2_FULL_GI_TOKENS = 512  # tokens whose query is stored for the selection check


def gen_c2_full(mem, name, seed=0):
    """Config 2 at full table geometry (n_keys 512 -> 262144 slots of 1024
    bf16, k_dim 512, 4 heads x top-32, query BatchNorm) on one 2048-token
    sequence: the reference's bf16 layer forward + backward on CPU
    (``pkm/memory.py:190-248``, bag through ``F.embedding_bag``).

    Stored: the reference's indices (the selection the checker pins), loss,
    fingerprints (``cases.summarize``) of the output and of every gradient,
    and, for the first 512 tokens, the reference's bf16 query with its
    ``get_indices`` scores and indices (the selection check on one query)."""
    cfg = cases.CONFIG2
    torch.manual_seed(0)
    m = mem.HashingMemory(**cfg)
    st = cases.pkm_state(cfg, seed)
    m.load_state_dict(st)
    m = m.to(torch.bfloat16).train()
    x = cases.pkm_input((1, C2_FULL_TOKENS, cfg["input_dim"]), seed).to(torch.bfloat16).requires_grad_(True)
    out = {"param_checksums": np.stack([cases.checksum(st[k]) for k in sorted(st)]),
           "x_checksum": cases.checksum(x)}
    with torch.no_grad():
        q = m.query_proj(x.view(-1, cfg["input_dim"])[:C2_FULL_GI_TOKENS])
        s, i = m.get_indices(q, cfg["mem_knn"])
    m.query_proj.norm.reset_running_stats()  # the slice above updated them
    out["gi_query"] = cases.bf16_bits(q)
    out["gi_scores"] = _np(s)
    out["gi_indices"] = i.numpy().astype(np.int32)
    y, idx = m(x)
    loss = (y.float() ** 2).sum()
    loss.backward()
    out["indices"] = idx.numpy().astype(np.int32)
    out["loss"] = np.array(loss.item())
    _put_summary(out, "out", y.view(C2_FULL_TOKENS, -1).float())
    _put_summary(out, "x_grad", x.grad.view(C2_FULL_TOKENS, -1).float())
    out["keys_grad"] = cases.bf16_bits(m.keys.grad)
    _put_summary(out, "values_grad", m.values.weight.grad.float(), nonzero_rows=True, f32=True)
    _put_summary(out, "wq_grad", m.query_proj.query_mlps[0].weight.grad.float())
    out["bq_grad"] = _np(m.query_proj.query_mlps[0].bias.grad)
    out["bn_w_grad"] = _np(m.query_proj.norm.weight.grad)
    out["bn_b_grad"] = _np(m.query_proj.norm.bias.grad)
    out["bn_running_mean"] = _np(m.query_proj.norm.running_mean)
    out["bn_running_var"] = _np(m.query_proj.norm.running_var)
    _put_summary(out, "wv_grad", m.value_proj.weight.grad.float())
    out["bv_grad"] = _np(m.value_proj.bias.grad)
    _put_summary(out, "ws_grad", m.swilu_projection.weight.grad.float())
    out["bs_grad"] = _np(m.swilu_projection.bias.grad)
    np.savez_compressed(os.path.join(HERE, name), **out)
    print("wrote", name)


def gen_fwpkm_c4(fw, name, score_type, seed=0):
    """``forward_wo_past`` (``fwpkm/fwpkm.py:395-558``) at config-4 geometry
    (``cases.FW_C4``: 262144 slots of 1024 fp32 values) on a 512-position
    sequence in two chunks of 256, then the outer backward of
    ``sum(out^2) + addr_loss`` through the double backward.  Stored: indices,
    scores, per-token losses, the addressing loss, grad norms, the output,
    and fingerprints of the final fast weights (the values as their change)
    and of every outer gradient."""
    torch.manual_seed(0)
    m = fw.FastWeightProductKeyMemory(qk_score_type=score_type, **cases.FW_C4).train()
    keys, values, q, ref_v = cases.fwpkm_c4_case(seed)
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
        # the first chunk's selection on the initial keys (raw scores)
        H, kd = cases.FW_C4["mem_heads"], cases.FW_C4["mem_k_dim"]
        q0 = q[0, :cases.FW_C4_CHUNK].reshape(-1, H, kd)
        s0, i0, _, _, _, _ = m.get_indices(q0, m.keys.float())
    q = q.clone().requires_grad_(True)
    ref_v = ref_v.clone().requires_grad_(True)
    # the inner gradients' norms in float64 as well: torch's fp32 norm on CPU
    # (what the reference's ``grad_norms`` holds) is 0.2 % low on these
    # 268M-element gradients, while a device reduction in fp32 is not
    norms64 = []
    update_fw = m.update_fw

    def recording_update_fw(*a, **kw):
        new, grads = update_fw(*a, **kw)
        norms64.append([torch.linalg.vector_norm(g.detach(), dtype=torch.float64).item() for g in grads])
        return new, grads

    m.update_fw = recording_update_fw
    res = m(q, ref_v, None, cases.FW_C4_CHUNK)
    loss = (res["output"] ** 2).sum() + res["addr_loss"]
    loss.backward()
    T = q.shape[1]
    out = {
        "keys_checksum": cases.checksum(keys), "values_checksum": cases.checksum(values),
        "q_checksum": cases.checksum(q), "ref_v_checksum": cases.checksum(ref_v),
        "gi0_scores": _np(s0).reshape(-1, cases.FW_C4["mem_topk"]),
        "gi0_indices": i0.numpy().astype(np.int32).reshape(-1, cases.FW_C4["mem_topk"]),
        "indices": res["indices"].numpy().astype(np.int32),
        "scores": _np(res["scores"]),
        "losses": _np(res["losses"]),
        "addr_loss": np.array(res["addr_loss"].item()),
        "grad_norms": np.array([g.item() for g in res["grad_norms"]]),
        "grad_norms_f64": np.array(norms64).mean(axis=0),
        "output": _np(res["output"]),
        "loss": np.array(loss.item()),
    }
    _put_summary(out, "final_keys", m.keys.detach())
    _put_summary(out, "values_delta", m.values.detach() - values, nonzero_rows=True, f32=True)
    _put_summary(out, "q_grad", q.grad.view(T, -1))
    _put_summary(out, "ref_v_grad", ref_v.grad.view(T, -1))
    _put_summary(out, "keys_grad", m.keys.grad)
    _put_summary(out, "values_grad", m.values.grad, nonzero_rows=True, f32=True)
    np.savez_compressed(os.path.join(HERE, name), **out)
    print("wrote", name)


def gen_addr_stats(name):
    """``compute_addr_stats`` of the reference's decoder layer
    (``modeling_qwen3pkm.py:447-471``) on ``cases.addr_case`` inputs; the
    method only reads ``config.fwpkm_n_subkeys`` and ``config.fwpkm_addr_loss``."""
    import refmodel
    model = refmodel.load("refmodel_golden", ours=False)
    out = {}
    for cname in cases.ADDR_CASES:
        idx, K, loss = cases.addr_case(cname)
        n = int(round(K ** 0.5))
        assert n * n == K
        stub = types.SimpleNamespace(config=types.SimpleNamespace(fwpkm_n_subkeys=n, fwpkm_addr_loss="me"))
        st = model.Qwen3PKMDecoderLayer.compute_addr_stats(stub, idx, loss)
        out[cname + "_idx_checksum"] = cases.checksum(idx)
        out[cname + "_stats"] = np.array([st["collision_ratio"], st["coverage_ratio"], st["kld"],
                                          st["addressing_loss/me"]], dtype=np.float64)
    np.savez_compressed(os.path.join(HERE, name), **out)
    print("wrote", name)


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    mem, xeb, fw, gw, leg = _import_ref()
    gen_pkm(mem, cases.CONFIG0, "c0_pkm.npz", (2, 128, 512), torch.float32)
    gen_indices_seeds(mem, "c0_indices_seeds.npz")
    gen_ties(mem, "ties.npz")
    gen_embbag(xeb, gw, leg, "embbag.npz")
    gen_fwpkm(fw, "fwpkm_dot.npz", "dot_product")
    gen_fwpkm(fw, "fwpkm_idw.npz", "idw")
    c2 = dict(cases.CONFIG2)
    c2.update(mem_n_keys=64)  # same layer, smaller table so the fixture stays small
    gen_pkm(mem, c2, "c2_small_bf16.npz", (2, 32, 1024), torch.bfloat16)
    gen_addr_stats("addr_stats.npz")
    for sname in cases.STREAM_FIXTURES:
        gen_fwpkm_stream(fw, sname)
    gen_c2_full(mem, "c2_full_bf16.npz")
    gen_fwpkm_c4(fw, "fwpkm_c4_dot.npz", "dot_product")
    gen_fwpkm_c4(fw, "fwpkm_c4_idw.npz", "idw")
    for vname in cases.FW_VARIANTS:
        gen_fwpkm_variant(fw, gw, vname)
    for vname in cases.PKM_VARIANTS:
        gen_pkm_variant(mem, vname)


if __name__ == "__main__":
    if len(sys.argv) > 1:  # regenerate named fixtures only, e.g. ``addr_stats``
        for arg in sys.argv[1:]:
            if arg == "addr_stats":
                gen_addr_stats("addr_stats.npz")
            elif arg == "c2_full":
                gen_c2_full(_import_ref()[0], "c2_full_bf16.npz")
            elif arg == "pkm_var":
                mem = _import_ref()[0]
                for vname in cases.PKM_VARIANTS:
                    gen_pkm_variant(mem, vname)
            elif arg == "fwpkm_var":
                ref = _import_ref()
                for vname in cases.FW_VARIANTS:
                    gen_fwpkm_variant(ref[2], ref[3], vname)
            elif arg == "fwpkm_c4":
                fw = _import_ref()[2]
                gen_fwpkm_c4(fw, "fwpkm_c4_dot.npz", "dot_product")
                gen_fwpkm_c4(fw, "fwpkm_c4_idw.npz", "idw")
            elif arg == "fwpkm_stream":
                fw = _import_ref()[2]
                for sname in cases.STREAM_FIXTURES:
                    gen_fwpkm_stream(fw, sname)
            else:
                raise SystemExit(f"unknown fixture {arg}")
    else:
        main()
