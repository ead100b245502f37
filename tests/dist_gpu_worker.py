"""Worker of the two-GPU data-parallel test: one NCCL rank per GPU runs a
HashingMemory step with the fused table-gradient exchange and with the plain
NCCL all-reduce, and saves both table gradients."""
from __future__ import annotations

import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

CFG = dict(input_dim=256, output_dim=256, mem_k_dim=128, mem_v_dim=256, mem_heads=4, mem_knn=16, mem_n_keys=64,
           mem_query_batchnorm=False, mem_query_rmsnorm=True)


def run(rank: int, world: int, port: int, out_dir: str, dtype_name: str, mode: str = "p2p"):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from modelos_b200.dist import GradReducer, ShardedTableGrad
        from modelos_b200.pkm.memory import HashingMemory

        dtype = getattr(torch, dtype_name)
        torch.manual_seed(0)
        m = HashingMemory(**CFG)
        m.reset_parameters()
        m = m.to(dev, dtype)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        x = torch.randn((2, 300, CFG["input_dim"]), generator=g, device=dev).to(dtype)
        params = list(m.parameters())

        def step():
            for p in params:
                p.grad = None
            y, _ = m(x)
            (y.float() ** 2).sum().backward()

        # plain: local gradient + NCCL all-reduce
        step()
        ref = m.values.weight.grad.clone()
        dist.all_reduce(ref)
        ref_keys = m.keys.grad.clone()
        dist.all_reduce(ref_keys)
        # fused exchange, two steps (the buffers are reused)
        try:
            ex = ShardedTableGrad(m.values.weight, mode=mode)
        except RuntimeError as e:  # no NVLink multicast on this machine
            torch.save({"skip": str(e)}, os.path.join(out_dir, f"rank{rank}.pt"))
            return
        red = GradReducer(params, sharded=[ex])
        for _ in range(2):
            step()
            red.finish()
        torch.cuda.synchronize()
        got = m.values.weight.grad
        torch.save({"ref": ref.cpu(), "got": got.cpu(), "ref_keys": ref_keys.cpu(), "got_keys": m.keys.grad.cpu(),
                    "aliased": got.data_ptr() == ex.full.data_ptr(), "mode": ex.mode},
                   os.path.join(out_dir, f"rank{rank}.pt"))
        ex.close()
        del ex, red
    finally:
        dist.destroy_process_group()


def sharded_inputs(rank: int, dtype, dev):
    import torch
    K, D, B, L = 4096, 256, 512, 32
    g = torch.Generator().manual_seed(11)
    table = (torch.randn(K, D, generator=g) * 0.1).to(dtype)
    g = torch.Generator().manual_seed(200 + rank)
    idx = torch.randint(0, K, (B, L), generator=g)
    psw = torch.softmax(torch.randn(B, L, generator=g), -1).to(dtype)
    d_out = torch.randn(B, D, generator=g).to(dtype)
    return table.to(dev), idx.to(dev), psw.to(dev), d_out.to(dev)


def run_sharded(rank: int, world: int, port: int, out_dir: str, dtype_name: str, backend: str = "nccl"):
    """Row-sharded bag against the dense kernels over the full table: NCCL
    with one GPU per rank, or gloo with every rank on GPU 0 (the collectives
    then move host copies; no kernel of one rank waits on another)."""
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    gpu = rank if backend == "nccl" else 0
    torch.cuda.set_device(gpu)
    dev = torch.device("cuda", gpu)
    if backend == "nccl":
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
    else:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from modelos_b200 import _native
        from modelos_b200.sharded import RowShardedEmbeddingBag
        dtype = getattr(torch, dtype_name)
        table, idx, psw, d_out = sharded_inputs(rank, dtype, dev)
        m = RowShardedEmbeddingBag(table.shape[0], table.shape[1], dtype=dtype, device=dev)
        m.load_full(table)
        p = psw.clone().requires_grad_()
        out = m(idx, p)
        out.backward(d_out)
        torch.cuda.synchronize()
        # dense references: this rank's bags, and every rank's bags for dW
        ref_out = _native.bag_fwd(idx, table, psw)
        _, ref_dpsw, _ = _native.bag_bwd(idx, table, psw, d_out)
        all_idx, all_psw, all_d = [], [], []
        for r in range(world):
            _, i_r, p_r, d_r = sharded_inputs(r, dtype, dev)
            all_idx.append(i_r)
            all_psw.append(p_r)
            all_d.append(d_r)
        ref_dW, _, _ = _native.bag_bwd(torch.cat(all_idx), table, torch.cat(all_psw), torch.cat(all_d))
        S = m.shard_rows
        torch.save({"out": out.detach().cpu(), "ref_out": ref_out.cpu(), "dpsw": p.grad.cpu(),
                    "ref_dpsw": ref_dpsw.cpu(), "dW": m.weight.grad.cpu(),
                    "ref_dW": ref_dW[rank * S:(rank + 1) * S].cpu()},
                   os.path.join(out_dir, f"shard{rank}.pt"))
        _native.check_device_errors(dev)
    finally:
        dist.destroy_process_group()


def run_owner(rank: int, world: int, port: int, out_dir: str, dtype_name: str):
    """RowOwnerSGD (reduce-scatter in the bag backward, owner SGD, all-gather
    of the rows) against NCCL all-reduce of the table gradient plus
    torch.optim.SGD on every rank, over two steps."""
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from modelos_b200.dist import RowOwnerSGD
        from modelos_b200.pkm.memory import HashingMemory

        dtype = getattr(torch, dtype_name)
        lr, wd = 0.05, 0.01

        def make():
            torch.manual_seed(0)
            m = HashingMemory(**CFG)
            m.reset_parameters()
            return m.to(dev, dtype)

        ref, m = make(), make()
        owner = RowOwnerSGD(m.values.weight, lr=lr, weight_decay=wd)
        opt = torch.optim.SGD([ref.values.weight], lr=lr, weight_decay=wd, foreach=True)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        tables = []
        for _ in range(2):
            x = torch.randn((2, 300, CFG["input_dim"]), generator=g, device=dev).to(dtype)
            for mod in (ref, m):
                for p in mod.parameters():
                    p.grad = None
                y, _ = mod(x)
                (y.float() ** 2).sum().backward()
            dist.all_reduce(ref.values.weight.grad)
            opt.step()
            assert m.values.weight.grad is None
            owner.step()
            torch.cuda.synchronize()
            tables.append((ref.values.weight.detach().cpu().clone(), m.values.weight.detach().cpu().clone()))
        torch.save({"tables": tables, "aliased": m.values.weight.data_ptr() == owner.table.data_ptr()},
                   os.path.join(out_dir, f"owner{rank}.pt"))
        owner.close()
        del owner
    finally:
        dist.destroy_process_group()


def run_fwpkm_dp(rank: int, world: int, port: int, out_dir: str, backend: str = "nccl", sharded: bool = False,
                 variant: bool = False):
    """One rank of the data-parallel fast-weight memory on the GPU kernels
    (fp32, tiny geometry): half of the batch, fast weights replicated or the
    value table split by rows; ``variant`` adds ``FW_VARIANT_KW`` (keys
    trained by the memorisation loss, weight decay, clipping)."""
    import datetime

    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank if backend == "nccl" else 0)
    torch.cuda.set_device(dev)
    kw = dict(rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    if backend == "nccl":
        kw["device_id"] = dev
    dist.init_process_group(backend, **kw)
    try:
        import dist_worker
        keys, values, q, ref_v = dist_worker.fwpkm_dp_case()
        per = q.shape[0] // world
        sl = slice(rank * per, (rank + 1) * per)
        out = fwpkm_gpu_run(q[sl], ref_v[sl], keys, values, dev, dist.group.WORLD, sharded=sharded,
                            extra_kw=dist_worker.FW_VARIANT_KW if variant else None)
        torch.save(out, os.path.join(out_dir, f"{'fwsh' if sharded else 'fwdp'}{rank}.pt"))
    finally:
        dist.destroy_process_group()


def fwpkm_gpu_run(q, ref_v, keys, values, dev, group=None, sharded=False, extra_kw=None):
    import torch

    import dist_worker
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    m = FastWeightProductKeyMemory(**dict(dist_worker.FW_DP_KW, **(extra_kw or {}))).to(dev).train()
    with torch.no_grad():
        m.keys.copy_(keys)
        m.values.copy_(values)
    if group is not None:
        if sharded:
            m.row_sharded(group)
        else:
            m.data_parallel(group)
    q = q.to(dev).requires_grad_(True)
    ref_v = ref_v.to(dev).requires_grad_(True)
    res = m(q, ref_v, None, 8)
    (res["output"] ** 2).sum().backward()
    m.reduce_grads()
    vals, vgrad = m.values.detach(), m.values.grad
    if sharded:
        import torch.distributed as dist
        world = dist.get_world_size(group)

        def gather(t):
            parts = [torch.empty_like(t) for _ in range(world)]
            if dist.get_backend(group) == "nccl":
                dist.all_gather(parts, t.contiguous(), group=group)
            else:
                host = [torch.empty_like(t, device="cpu") for _ in range(world)]
                dist.all_gather(host, t.detach().cpu().contiguous(), group=group)
                parts = [h.to(t.device) for h in host]
            return torch.cat(parts)[: m.size]
        vals, vgrad = gather(vals), gather(vgrad)
    torch.cuda.synchronize()
    return {k: v.detach().cpu() for k, v in (("out", res["output"]), ("q_grad", q.grad), ("ref_v_grad", ref_v.grad),
                                             ("keys", m.keys), ("values", vals), ("keys_grad", m.keys.grad),
                                             ("values_grad", vgrad), ("indices", res["indices"]))}
