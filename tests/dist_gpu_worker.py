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
