"""Seeded input generators shared by the golden-fixture script and the tests.

Every tensor is drawn from an explicit ``torch.Generator`` in a fixed order,
so the GPU box (same torch build) regenerates bit-identical parameters and
inputs without the reference tree; the fixtures store checksums of what was
generated so a drift in torch's CPU generator is caught instead of silently
changing the case.
"""
from __future__ import annotations

import math

import numpy as np
import torch

# Benchmark config 0 (``pkm/memory.py:41-68`` argument names).
CONFIG0 = dict(input_dim=512, output_dim=512, mem_k_dim=256, mem_v_dim=512, mem_heads=4,
               mem_knn=32, mem_n_keys=128)
# Benchmark config 2 geometry (bf16, query BatchNorm).
CONFIG2 = dict(input_dim=1024, output_dim=1024, mem_k_dim=512, mem_v_dim=1024, mem_heads=4,
               mem_knn=32, mem_n_keys=512, mem_query_batchnorm=True, mem_query_rmsnorm=False)


def _u(g, shape, bound):
    return (torch.rand(shape, generator=g, dtype=torch.float32) * 2 - 1) * bound


def _n(g, shape, std):
    return torch.randn(shape, generator=g, dtype=torch.float32) * std


def pkm_state(cfg: dict, seed: int = 0) -> dict:
    """Parameters of a ``HashingMemory`` built with ``cfg``.

    Init follows ``HashingMemory.reset_parameters`` (``pkm/memory.py:169-188``)
    for keys (U(+-1/sqrt(k_dim))), values (N(0, v_dim^-1/2)) and the SwiLU /
    value projections (N(0, output_dim^-1/2)); the query Linear and all biases
    keep nn.Linear's default U(+-1/sqrt(fan_in)), as benchmark config 0 states.
    """
    g = torch.Generator().manual_seed(seed)
    C = cfg["input_dim"]
    O = cfg["output_dim"]
    kd = cfg["mem_k_dim"]
    H = cfg["mem_heads"]
    n = cfg["mem_n_keys"]
    v = cfg["mem_v_dim"] if cfg.get("mem_v_dim", -1) > 0 else O
    st = {}
    st["keys"] = _u(g, (2 * H * n, kd // 2), 1 / math.sqrt(kd))
    st["values.weight"] = _n(g, (n * n, v), v ** -0.5)
    st["value_proj.weight"] = _n(g, (O, v), O ** -0.5)
    st["value_proj.bias"] = _u(g, (O,), 1 / math.sqrt(v))
    st["swilu_projection.weight"] = _n(g, (v, C), O ** -0.5)
    st["swilu_projection.bias"] = _u(g, (v,), 1 / math.sqrt(C))
    st["query_proj.query_mlps.0.weight"] = _u(g, (H * kd, C), 1 / math.sqrt(C))
    st["query_proj.query_mlps.0.bias"] = _u(g, (H * kd,), 1 / math.sqrt(C))
    if cfg.get("mem_query_batchnorm", False):
        st["query_proj.norm.weight"] = torch.ones(H * kd)
        st["query_proj.norm.bias"] = torch.zeros(H * kd)
        st["query_proj.norm.running_mean"] = torch.zeros(H * kd)
        st["query_proj.norm.running_var"] = torch.ones(H * kd)
        st["query_proj.norm.num_batches_tracked"] = torch.tensor(0, dtype=torch.int64)
    elif cfg.get("mem_query_rmsnorm", True):
        st["query_proj.norm.weight"] = torch.ones(H * kd)
    return st


# ``HashingMemory`` option sets beyond the benchmark configs, on a small
# geometry: the gate, no query bias, no query norm, the value projection
# without the SwiLU branch, no projection at all, three heads, eval mode
# (``last_indices`` / ``last_scores``).  Each entry: options, training mode.
PKM_VARIANT_BASE = dict(input_dim=64, output_dim=64, mem_k_dim=32, mem_v_dim=-1, mem_heads=2, mem_knn=4,
                        mem_n_keys=16)
PKM_VARIANTS = {
    "pkm_var_gated.npz": (dict(mem_gated=True, mem_v_dim=48, mem_query_bias=False), True),
    "pkm_var_plain.npz": (dict(swilu_projection=False, mem_query_rmsnorm=False, mem_gated=True, mem_heads=3,
                               mem_knn=8), True),
    "pkm_var_vproj.npz": (dict(swilu_projection=False, mem_v_dim=48), True),
    "pkm_var_eval.npz": (dict(), False),
}


def pkm_variant_state(shapes: dict, seed: int = 0) -> dict:
    """Parameters for a ``PKM_VARIANTS`` module from its state-dict names and
    shapes, filled in sorted-name order from one seeded generator: keys
    U(+-1/sqrt(2·cols)), weight matrices N(0, cols^-1/2), biases
    U(+-1/sqrt(64)), the RMS-norm scale 1 + N(0, 0.1)."""
    g = torch.Generator().manual_seed(50_000 + seed)
    st = {}
    for name in sorted(shapes):
        shape = tuple(shapes[name])
        if name == "keys":
            st[name] = _u(g, shape, 1 / math.sqrt(2 * shape[1]))
        elif name.endswith("norm.weight"):
            st[name] = 1 + _n(g, shape, 0.1)
        elif len(shape) == 2:
            st[name] = _n(g, shape, shape[1] ** -0.5)
        else:
            st[name] = _u(g, shape, 0.125)
    return st


def run_pkm_variant(module, name, seed=0, device="cpu"):
    """Load ``pkm_variant_state`` into ``module`` (built with the variant's
    options), run one forward + backward of loss = sum(out^2) on a seeded
    [2, 8, input_dim] input and return every output: out, indices, the input
    gradient, each parameter's gradient (``g_<name>``) and, in eval mode,
    ``last_indices`` / ``last_scores``."""
    kw, train = PKM_VARIANTS[name]
    module.load_state_dict(pkm_variant_state({k: v.shape for k, v in module.state_dict().items()}, seed))
    module = module.to(device).train(train)
    g = torch.Generator().manual_seed(60_000 + seed)
    x = torch.randn((2, 8, module.input_dim), generator=g).to(device).requires_grad_(True)
    y, idx = module(x)
    (y ** 2).sum().backward()
    out = {"out": y, "indices": idx, "x_grad": x.grad}
    out.update({"g_" + k: p.grad for k, p in module.named_parameters() if p.grad is not None})
    if not train:
        out["last_indices"] = module.last_indices
        out["last_scores"] = module.last_scores
    return out


def pkm_input(shape, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(10_000 + seed)
    return torch.randn(shape, generator=g, dtype=torch.float32)


def embbag_case(B: int, L: int, K: int, D: int, seed: int = 0, heads: int = 1,
                w_std: float = 0.03):
    """Embedding-bag inputs in the style of benchmark config 1.

    Indices uniform in [0, K) with replacement, per-bag weights the softmax of
    N(0,1) logits normalised per head (``heads`` groups of L/heads), table
    N(0, w_std), upstream gradient N(0,1).  All fp32; callers cast.
    """
    g = torch.Generator().manual_seed(20_000 + seed)
    idx = torch.randint(0, K, (B, L), generator=g, dtype=torch.int64)
    logits = torch.randn((B, heads, L // heads if heads > 1 else L), generator=g)
    psw = torch.softmax(logits, dim=-1).reshape(B, L)
    W = torch.randn((K, D), generator=g) * w_std
    gout = torch.randn((B, D), generator=g)
    return idx, psw, W, gout


# The small FwPKM geometry of ``fwpkm_case`` (module options).
FW_KW = dict(mem_k_dim=16, mem_v_dim=32, mem_heads=2, mem_topk=4, mem_n_subkeys=16, lookahead=1,
             learning_rate=0.1)


def fwpkm_case(seed: int = 0, B=2, T=16, heads=2, k_dim=16, v_dim=32, n_sub=16, topk=4):
    """Tiny FwPKM inputs: q [B,T,H*k_dim], ref_v [B,T,v_dim], keys, values."""
    g = torch.Generator().manual_seed(30_000 + seed)
    keys = _u(g, (2 * heads * n_sub, k_dim // 2), 1 / math.sqrt(k_dim))
    values = _n(g, (n_sub * n_sub, v_dim), v_dim ** -0.5)
    q = torch.randn((B, T, heads * k_dim), generator=g)
    ref_v = torch.randn((B, T, v_dim), generator=g)
    return keys, values, q, ref_v


# Non-default module options, each fixture a combination the defaults
# leave untested: the transform (silu / relu, temperature), the keys trained
# by the memorisation loss too, gradient clipping, weight decay, no
# look-ahead, no addressing loss, per-token gates and a loss mask.  Each
# entry: module options, with gates, with a loss mask, and the dtype of the
# module and its inputs ("bf16": the model's setting, bf16 parameters with
# the fast weights in fp32 copies, ``fp32_fw``).
FW_VARIANTS = {
    "fwpkm_var_silu.npz": (dict(qk_score_type="idw", score_nonlinear="silu", score_temperature=0.5,
                                mem_grad_to_values_only=False, grad_clip=True, weight_decay=0.01),
                           True, True, "f32"),
    "fwpkm_var_relu.npz": (dict(qk_score_type="dot_product", score_nonlinear="relu", lookahead=0, addr_loss=None,
                                mem_grad_to_values_only=False),
                           False, True, "f32"),
    "fwpkm_var_keys.npz": (dict(qk_score_type="dot_product", mem_grad_to_values_only=False), False, False, "f32"),
    "fwpkm_var_bf16.npz": (dict(qk_score_type="dot_product", addr_loss_weight=0.5), True, False, "bf16"),
}
# normwise tolerance by variant dtype: fp32, and one bf16 rounding of
# results computed in fp32 on both sides
FW_VARIANT_TOL = {"f32": 1e-5, "bf16": 1e-2}


def fw_variant_inputs(B, T, with_gates, with_mask, seed=5):
    """Per-token gates in (0, 1) and a 0/1 loss mask for a variant run."""
    g = torch.Generator().manual_seed(40_000 + seed)
    gates = torch.rand((B, T), generator=g) if with_gates else None
    mask = (torch.rand((B, T), generator=g) > 0.25).float() if with_mask else None
    return gates, mask


# Benchmark config 4 geometry (FwPKM): k_dim 512, v_dim 1024, 4 heads x top-32
# over 512^2 fp32 fast-weight slots; the module's other defaults (idw,
# softmax, addressing loss "me", lookahead 1, fp32 fast weights).
FW_C4 = dict(mem_k_dim=512, mem_v_dim=1024, mem_heads=4, mem_topk=32, mem_n_subkeys=512, learning_rate=0.1)
# A config-4 slice small enough for the reference on CPU: one sequence of
# 512 positions in two chunks of 256 (two inner updates).
FW_C4_T, FW_C4_CHUNK = 512, 256


def fwpkm_c4_case(seed: int = 0, T: int = FW_C4_T):
    """Config-4-geometry FwPKM inputs: keys U(+-1/sqrt(k_dim)) and values
    N(0, v_dim^-1/2) as ``reset_parameters`` (``fwpkm/fwpkm.py:91-96``);
    q [1, T, H*k_dim] and ref_v [1, T, v_dim] N(0,1), rounded to bf16 (the
    config's input dtype) and kept in fp32, the dtype the fast-weight path
    computes in (``fp32_fw``, ``fwpkm/fwpkm.py:406-409``)."""
    kw = FW_C4
    H, kd, D, n = kw["mem_heads"], kw["mem_k_dim"], kw["mem_v_dim"], kw["mem_n_subkeys"]
    g = torch.Generator().manual_seed(31_000 + seed)
    keys = _u(g, (2 * H * n, kd // 2), 1 / math.sqrt(kd))
    values = _n(g, (n * n, D), D ** -0.5)
    q = torch.randn((1, T, H * kd), generator=g).bfloat16().float()
    ref_v = torch.randn((1, T, D), generator=g).bfloat16().float()
    return keys, values, q, ref_v


SUMMARY_SAMPLE = 64


def summarize(t: torch.Tensor, rows_idx=None, nsample: int = SUMMARY_SAMPLE, seed: int = 0,
              nonzero_rows: bool = False) -> dict:
    """Size-independent fingerprint of a 2-D (or flattened-to-2-D) tensor.

    Per row, in float64 on the tensor's device: the L2 norm and the product
    with one fixed random vector; plus ``nsample`` full rows.  The generator
    picks the rows (among the nonzero rows when ``nonzero_rows``: sparse
    gradients) and stores their indices; a checker passes those indices back
    as ``rows_idx``.  Comparing the three parts normwise bounds every row's
    size and direction and samples its elements.
    """
    t2 = t.detach().reshape(t.shape[0], -1).double()
    cols = t2.shape[1]
    r = torch.randn(cols, generator=torch.Generator().manual_seed(77_000), dtype=torch.float64).to(t2.device)
    out = {"rownorm": t2.norm(dim=1).cpu().numpy(), "proj": (t2 @ r).cpu().numpy()}
    if rows_idx is None:
        g = np.random.default_rng(seed)
        pool = np.arange(t2.shape[0])
        if nonzero_rows:
            pool = torch.nonzero(t2.abs().amax(dim=1) > 0).flatten().cpu().numpy()
        rows_idx = np.sort(g.choice(pool, size=min(nsample, len(pool)), replace=False))
    out["rows_idx"] = np.asarray(rows_idx, dtype=np.int64)
    out["rows"] = t2[torch.from_numpy(out["rows_idx"]).to(t2.device)].cpu().numpy()
    return out


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns (half the bytes of a float32 copy)."""
    return t.detach().to(torch.bfloat16).cpu().view(torch.int16).numpy().view(np.uint16)


def from_bf16_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def checksum(t: torch.Tensor) -> np.ndarray:
    """(sum, sum|x|, sum x*i) in float64: a cheap fingerprint of a tensor."""
    a = t.detach().double().reshape(-1)
    w = torch.arange(a.numel(), dtype=torch.float64) / max(1, a.numel())
    return np.array([a.sum().item(), a.abs().sum().item(), (a * w).sum().item()])


# Addressing-statistics cases: name -> (slots K, generator).  ``c4_chunk`` is
# one FwPKM chunk of benchmark config 4 (8 x 512 tokens, 4 heads x top-32
# over 512^2 slots); ``clamped`` has a total count above 1/eps(fp32), so both
# of torch's probability clamps act (the lone slot's p < eps, the hot
# slot's p > 1 - eps).
ADDR_CASES = ("c4_chunk", "hot", "single_slot", "permutation", "tiny", "clamped")


def addr_case(name: str, seed: int = 0):
    """``(indices int64, K, addr_loss [n] fp32)`` of one addressing case."""
    g = torch.Generator().manual_seed(40_000 + seed)
    if name == "c4_chunk":
        K = 512 * 512
        idx = torch.randint(0, K, (4096, 128), generator=g)
    elif name == "hot":
        K = 4096
        idx = torch.randint(0, K, (20000,), generator=g)
        hot = torch.rand(20000, generator=g) < 0.6
        idx[hot] = torch.randint(0, 8, (int(hot.sum()),), generator=g) * 37
    elif name == "single_slot":
        K = 64
        idx = torch.full((1000,), 5, dtype=torch.long)
    elif name == "permutation":
        K = 1024
        idx = torch.randperm(K, generator=g)
    elif name == "tiny":
        K = 16
        idx = torch.tensor([2, 2, 9], dtype=torch.long)
    elif name == "clamped":
        K = 64
        idx = torch.zeros(9_000_000, dtype=torch.long)
        idx[4_500_000] = 1
    else:
        raise KeyError(name)
    loss = torch.rand((max(1, idx.shape[0]),), generator=g)
    return idx, K, loss


# Token ranges of three successive ``forward_w_past`` calls over one
# ``fwpkm_case`` (T = 16, chunk 8, lookahead 1): the first only queues, the
# second updates once and queues the rest, the third updates again.
STREAM_CALLS = ((0, 4), (4, 13), (13, 16))


# Streaming fixtures: module options, with gates, with a loss mask.  The
# variant carries gates and a mask through the queues, with a look-ahead of
# 2, the silu transform and the clipped, decayed update.
STREAM_FIXTURES = {
    "fwpkm_stream_dot.npz": (dict(qk_score_type="dot_product"), False, False),
    "fwpkm_stream_idw.npz": (dict(qk_score_type="idw"), False, False),
    "fwpkm_stream_var.npz": (dict(qk_score_type="dot_product", score_nonlinear="silu", score_temperature=0.5,
                                  lookahead=2, grad_clip=True, weight_decay=0.01), True, True),
}


def stream_calls(m, q, ref_v, gates=None, mask=None):
    """Drive ``m`` through ``STREAM_CALLS`` under ``no_grad`` (as generation
    does), with token ids and the calls' slices of ``gates`` / ``mask``;
    yields ``(call, result, past_key_values)``."""
    B, T = q.shape[:2]
    ids = torch.arange(B * T, device=q.device).view(B, T)
    past = (None,) * 6
    with torch.no_grad():
        for c, (t0, t1) in enumerate(STREAM_CALLS):
            res = m(q[:, t0:t1], ref_v[:, t0:t1], None if gates is None else gates[:, t0:t1], 8,
                    loss_mask=None if mask is None else mask[:, t0:t1], past_key_values=past,
                    token_ids=ids[:, t0:t1])
            past = res["past_key_values"]
            yield c, res, past


def stream_inputs(name, seed=1, device="cpu"):
    """``(q, ref_v, gates, mask)`` of a ``STREAM_FIXTURES`` entry; keys and
    values are ``fwpkm_case(seed)``'s."""
    _, with_gates, with_mask = STREAM_FIXTURES[name]
    _, _, q, ref_v = fwpkm_case(seed)
    gates, mask = fw_variant_inputs(q.shape[0], q.shape[1], with_gates, with_mask)
    return tuple(None if t is None else t.to(device) for t in (q, ref_v, gates, mask))


def run_stream(m, q, ref_v, d, rel_err, tol=1e-5, gates=None, mask=None):
    """``stream_calls`` compared call by call with the fixture ``d``:
    indices and queued ids exactly; outputs, scores, queues, losses and the
    fast weights after every call to ``tol``."""
    for c, res, past in stream_calls(m, q, ref_v, gates, mask):
        np.testing.assert_array_equal(res["indices"].cpu().numpy(), d[f"c{c}_indices"])
        assert (res["losses"] is not None) == bool(d[f"c{c}_updated"]), c
        pairs = [(res["output"], "output"), (res["scores"], "scores"), (past[0], "past_q"),
                 (past[1], "past_hyp"), (past[2], "past_ref"), (m.keys, "keys"), (m.values, "values")]
        for t, key in ((past[3], "past_gates"), (past[4], "past_mask")):
            assert (t is None) == (f"c{c}_{key}" not in d), (c, key)
            if t is not None:
                pairs.append((t, key))
        if res["losses"] is not None:
            pairs.append((res["losses"], "losses"))
            got_addr = res["addr_loss"].item()
            ref_addr = float(d[f"c{c}_addr_loss"])
            assert abs(got_addr - ref_addr) <= tol * abs(ref_addr) + 1e-7, c
        for got, key in pairs:
            assert rel_err(got.detach().float().cpu().numpy(), d[f"c{c}_{key}"]) < tol, (c, key)
        np.testing.assert_array_equal(past[5].cpu().numpy(), d[f"c{c}_past_ids"])


def run_fw_variant(cls, fw_kw, name, d, rel_err, tol=1e-5, device="cpu"):
    """One training call of a ``FW_VARIANTS`` module on ``fwpkm_case(2)``
    (gates, loss mask and dtype as the variant asks), loss = sum(output^2) plus the
    addressing loss when there is one, checked against the fixture ``d``:
    indices exactly, outputs, losses, updated fast weights and every
    gradient to ``tol``."""
    kw, with_gates, with_mask, dt = FW_VARIANTS[name]
    dt = torch.bfloat16 if dt == "bf16" else torch.float32
    m = cls(**dict(fw_kw, **kw)).to(device=device, dtype=dt).train()
    keys, values, q, ref_v = (t.to(dt) for t in fwpkm_case(2))
    gates, mask = (None if t is None else t.to(dt)
                   for t in fw_variant_inputs(q.shape[0], q.shape[1], with_gates, with_mask))
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    q = q.to(device).requires_grad_(True)
    ref_v = ref_v.to(device).requires_grad_(True)
    gates = None if gates is None else gates.to(device)
    mask = None if mask is None else mask.to(device)
    res = m(q, ref_v, gates, 8, loss_mask=mask)
    loss = (res["output"] ** 2).sum()
    assert (res["addr_loss"] is None) == ("addr_loss" not in d)
    if res["addr_loss"] is not None:
        loss = loss + res["addr_loss"]
        ref_addr = float(d["addr_loss"])
        assert abs(res["addr_loss"].item() - ref_addr) <= tol * abs(ref_addr) + 1e-7
    loss.backward()
    np.testing.assert_array_equal(res["indices"].cpu().numpy(), d["indices"])
    assert (m.keys.grad is None) == ("keys_grad" not in d)
    pairs = [(res["output"], "output"), (res["losses"], "losses"), (m.keys, "final_keys"),
             (m.values, "final_values"), (q.grad, "q_grad"), (ref_v.grad, "ref_v_grad"),
             (m.values.grad, "values_grad")]
    if m.keys.grad is not None:
        pairs.append((m.keys.grad, "keys_grad"))
    for got, key in pairs:
        assert rel_err(got.detach().float().cpu().numpy(), d[key]) < tol, key


def check_pkm_variant(res, d, rel_err, tol=1e-5):
    """``run_pkm_variant`` results against the reference's fixture ``d``:
    the same set of outputs and gradients, indices exactly, the rest to
    ``tol`` of each tensor's largest magnitude."""
    assert sorted(res) == sorted(d), (sorted(res), sorted(d))
    for key, got in res.items():
        got = got.detach().cpu()
        if got.dtype == torch.long:
            np.testing.assert_array_equal(got.numpy(), d[key], err_msg=key)
        else:
            assert rel_err(got.float().numpy(), d[key]) < tol, key
