"""Worker of the multi-process CPU tests (gloo): one rank of a data-parallel
HashingMemory step with the kernels replaced by the CPU stand-in."""
from __future__ import annotations

import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

CFG = dict(input_dim=64, output_dim=64, mem_k_dim=32, mem_v_dim=64, mem_heads=2, mem_knn=4, mem_n_keys=16)


def install_cpu_kernels(set_attr=setattr):
    """Swap the kernels for the CPU stand-in (``set_attr`` may be pytest's
    ``monkeypatch.setattr`` so that the swap is undone after a test)."""
    import fake_native
    from modelos_b200 import _native
    from modelos_b200.pkm import colwise_embedding_bag, xformer_embeddingbag
    for name in ("bag_fwd", "bag_bwd", "bag_bwd2", "subkey_scores", "product_topk", "score_grad_dense", "swiglu_fwd",
                 "swiglu_bwd", "colsum", "segment_sum", "bag_bwd_ragged", "route_pack", "route_segments",
                 "route_combine", "read_device_errors"):
        set_attr(_native, name, getattr(fake_native, name))

    def bag(indices, weight, per_sample_weights, mode="sum", bw_algo="reverse_indices"):
        return xformer_embeddingbag.xFormersEmbeddingBag.apply(indices, weight, per_sample_weights, bw_algo)

    set_attr(xformer_embeddingbag, "xformers_embedding_bag", bag)
    set_attr(colwise_embedding_bag, "xformers_embedding_bag", bag)


def layer_grads(rank_input_seed: int, reducer_world=None):
    """Gradients of sum(out^2) for one rank's batch (single process)."""
    import torch

    import cases
    from modelos_b200.pkm.memory import HashingMemory
    m = HashingMemory(**CFG)
    m.load_state_dict(cases.pkm_state(CFG, 0))
    x = cases.pkm_input((2, 8, 64), rank_input_seed)
    y, _ = m(x)
    (y ** 2).sum().backward()
    return m, {n: p.grad.clone() for n, p in m.named_parameters()}


def run(rank: int, world: int, port: int, out_dir: str, mode: str):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        install_cpu_kernels()
        import cases
        from modelos_b200.dist import GradReducer
        from modelos_b200.pkm.memory import HashingMemory
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before its first collective")
        m = HashingMemory(**CFG)
        m.load_state_dict(cases.pkm_state(CFG, 0))
        red = GradReducer(m.parameters(), early=[m.values.weight])
        x = cases.pkm_input((2, 8, 64), 100 + rank)
        y, _ = m(x)
        (y ** 2).sum().backward()
        red.finish()
        torch.save({n: p.grad for n, p in m.named_parameters()}, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


SHARD_K, SHARD_D, SHARD_B, SHARD_L = 50, 16, 5, 7


def sharded_case(rank: int):
    """Table, this rank's bags and upstream gradient (seeded; the full table is
    the same on every rank)."""
    import torch
    g = torch.Generator().manual_seed(7)
    table = torch.randn(SHARD_K, SHARD_D, generator=g)
    g = torch.Generator().manual_seed(100 + rank)
    idx = torch.randint(0, SHARD_K, (SHARD_B, SHARD_L), generator=g)
    idx[0, :3] = 0  # a repeated row inside one bag
    psw = torch.rand(SHARD_B, SHARD_L, generator=g)
    d_out = torch.randn(SHARD_B, SHARD_D, generator=g)
    return table, idx, psw, d_out


def run_sharded(rank: int, world: int, port: int, out_dir: str, bad_rank=None):
    """One rank of the row-sharded bag on gloo with the CPU stand-in kernels;
    with ``bad_rank``, that rank's first index lies outside the table and
    every rank records the IndexError it raised."""
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        install_cpu_kernels()
        from modelos_b200.sharded import RowShardedEmbeddingBag
        table, idx, psw, d_out = sharded_case(rank)
        m = RowShardedEmbeddingBag(SHARD_K, SHARD_D)
        m.load_full(table)
        p = psw.clone().requires_grad_()
        if bad_rank is not None:
            if rank == bad_rank:
                idx[0, 0] = SHARD_K + 3
            try:
                m(idx, p)
                msg = None
            except IndexError as e:
                msg = str(e)
            torch.save({"raised": msg}, os.path.join(out_dir, f"bad{rank}.pt"))
            return
        out = m(idx, p)
        out.backward(d_out)
        torch.save({"out": out.detach(), "dpsw": p.grad, "dW": m.weight.grad, "rows": m.shard_rows},
                   os.path.join(out_dir, f"shard{rank}.pt"))
    finally:
        dist.destroy_process_group()


FW_DP_KW = dict(mem_k_dim=16, mem_v_dim=32, mem_heads=2, mem_topk=4, mem_n_subkeys=16, lookahead=1,
                learning_rate=0.1)


def fwpkm_dp_case():
    import cases
    return cases.fwpkm_case(0, B=4, T=16)


FW_VARIANT_KW = dict(mem_grad_to_values_only=False, weight_decay=0.01, grad_clip=True)


def fwpkm_run(q, ref_v, keys, values, group=None, sharded=False, extra_kw=None):
    """``forward_wo_past`` and the outer backward of ``sum(out^2)`` for the
    sequences given (all of them, or one rank's share with ``group``; with
    ``sharded`` the value table is split by rows over the group, and the
    returned values and value gradient are the gathered whole tables)."""
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    import torch
    m = FastWeightProductKeyMemory(**dict(FW_DP_KW, **(extra_kw or {}))).train()
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    if group is not None:
        if sharded:
            m.row_sharded(group)
        else:
            m.data_parallel(group)
    q = q.clone().requires_grad_(True)
    ref_v = ref_v.clone().requires_grad_(True)
    res = m(q, ref_v, None, 8)
    (res["output"] ** 2).sum().backward()
    m.reduce_grads()
    vals, vgrad = m.values.detach(), m.values.grad
    if sharded:
        import torch.distributed as dist
        world = dist.get_world_size(group)

        def gather(t):
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t.contiguous(), group=group)
            return torch.cat(parts)[: m.size]
        vals, vgrad = gather(vals), gather(vgrad)
    return {"out": res["output"].detach(), "q_grad": q.grad, "ref_v_grad": ref_v.grad, "keys": m.keys.detach(),
            "values": vals, "keys_grad": m.keys.grad, "values_grad": vgrad,
            "losses": res["losses"], "addr_loss": res["addr_loss"], "indices": res["indices"],
            "grad_norms": torch.stack(res["grad_norms"])}


def run_fwpkm_dp(rank: int, world: int, port: int, out_dir: str, sharded: bool = False, variant: bool = False):
    """One rank of the data-parallel fast-weight memory (gloo, CPU stand-ins),
    with a replicated or a row-split value table."""
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import fake_native

        class _Set:
            setattr = staticmethod(setattr)
        fake_native.install(_Set())
        install_cpu_kernels()
        keys, values, q, ref_v = fwpkm_dp_case()
        per = q.shape[0] // world
        sl = slice(rank * per, (rank + 1) * per)
        out = fwpkm_run(q[sl], ref_v[sl], keys, values, dist.group.WORLD, sharded=sharded,
                        extra_kw=FW_VARIANT_KW if variant else None)
        torch.save(out, os.path.join(out_dir, f"{'fwsh' if sharded else 'fwdp'}{rank}.pt"))
    finally:
        dist.destroy_process_group()
