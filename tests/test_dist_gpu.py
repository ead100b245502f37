"""Multi-rank GPU paths.

Fused data-parallel exchanges of the value-table gradient on two GPUs
(NVLink stores to the row owners, and the in-switch multimem all-reduce):
the table gradient equals the NCCL all-reduce of the ranks' local
gradients, bit for bit at two ranks (one addition per element, rounded
once) in fp32 and for the NVLink-store exchange in bf16, and within one
bf16 ulp for the in-switch reduction in bf16.

Row-sharded table: on two GPUs over NCCL, and with 2 or 3 ranks sharing
GPU 0 over gloo (runs on a one-GPU machine)."""
from __future__ import annotations

import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode", ["p2p", "nvls"])
@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
def test_sharded_table_grad_two_ranks(tmp_path, dtype_name, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    sys.path.insert(0, HERE)
    import dist_gpu_worker
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=dist_gpu_worker.run, args=(r, 2, port, str(tmp_path), dtype_name, mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in procs] == [0, 0]
    for r in range(2):
        d = torch.load(os.path.join(tmp_path, f"rank{r}.pt"))
        if "skip" in d:
            pytest.skip(d["skip"])
        assert d["mode"] == mode and d["aliased"]
        if mode == "nvls" and dtype_name == "bfloat16":
            # the switch's bf16 reduction (fp32 accumulation, its own final
            # rounding) may differ from NCCL's by one bf16 ulp
            got, ref = d["got"].float(), d["ref"].float()
            assert torch.all((got - ref).abs() <= ref.abs() * 2.0 ** -7)
            assert ((got - ref).abs().max() / ref.abs().max()).item() < 2e-2
        else:
            assert torch.equal(d["got"], d["ref"])
        assert torch.equal(d["got_keys"], d["ref_keys"])


def _run_row_sharded(tmp_path, dtype_name, tol, world, backend):
    import torch.multiprocessing as mp
    sys.path.insert(0, HERE)
    import dist_gpu_worker
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=dist_gpu_worker.run_sharded, args=(r, world, port, str(tmp_path), dtype_name, backend))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in procs] == [0] * world

    def rel(a, b):
        a, b = a.double(), b.double()
        return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()

    for r in range(world):
        d = torch.load(os.path.join(tmp_path, f"shard{r}.pt"))
        assert rel(d["out"], d["ref_out"]) < tol
        assert rel(d["dpsw"], d["ref_dpsw"]) < tol
        assert torch.equal(d["dW"][: d["ref_dW"].shape[0]], d["ref_dW"])


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("dtype_name,tol", [("float32", 1e-5), ("bfloat16", 2e-2)])
def test_row_sharded_bag_ranks_on_one_gpu(tmp_path, dtype_name, tol, world):
    """The row-sharded table with every rank on GPU 0 over gloo: the routing
    kernels (pack, segments, combine) and the ragged bag kernels for 2 and 3
    owners, against the dense kernels over the full table."""
    _run_row_sharded(tmp_path, dtype_name, tol, world, "gloo")


@pytest.mark.parametrize("dtype_name,tol", [("float32", 1e-5), ("bfloat16", 2e-2)])
def test_row_sharded_bag_two_ranks(tmp_path, dtype_name, tol):
    """Row-sharded table on two GPUs (NCCL all-to-all routing, ragged bag
    kernels) against the dense bag kernels over the full table: outputs and
    per-sample gradients of each rank's bags, and each owner's table rows of
    the gradient over every rank's bags (those bit for bit: the same rows
    are summed in the same order)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_row_sharded(tmp_path, dtype_name, tol, 2, "nccl")


def test_shard_sgd_kernel_against_torch_sgd():
    """pkm_grad_shard_sgd in one process, the "peer" tables being local
    buffers: the owner rows of every table get torch.optim.SGD's update of
    the summed gradient copies; other rows stay untouched."""
    from modelos_b200 import _native
    g = torch.Generator(device="cuda").manual_seed(3)
    for dtype in (torch.float32, torch.bfloat16):
        K, D, world, rank = 1000, 96, 3, 1
        S = -(-K // world)
        recv = torch.randn(world, S, D, generator=g, device="cuda").to(dtype)
        tables = [torch.randn(world * S, D, generator=g, device="cuda").to(dtype) for _ in range(world)]
        before = [t.clone() for t in tables]
        lr, wd = 0.1, 0.01
        _native.grad_shard_sgd(recv, K, rank, S, [t.data_ptr() for t in tables], lr, wd)
        torch.cuda.synchronize()
        gsum = recv[0].clone()
        for s_ in range(1, world):
            gsum = gsum + recv[s_]  # in the table dtype, source order
        p = torch.nn.Parameter(before[rank][rank * S:(rank + 1) * S].clone())
        p.grad = gsum
        torch.optim.SGD([p], lr=lr, weight_decay=wd, foreach=True).step()
        own = slice(rank * S, (rank + 1) * S)
        for t, b in zip(tables, before):
            got = t[own].float()
            exp = p.detach().float()
            ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -22
            assert ((got - exp).abs() <= exp.abs() * ulp + 1e-30).all()
            keep = torch.ones(world * S, dtype=torch.bool)
            keep[own] = False
            assert torch.equal(t[keep.cuda()], b[keep.cuda()])


@pytest.mark.parametrize("world", [1, 2])
@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
def test_row_owner_sgd(tmp_path, dtype_name, world):
    """RowOwnerSGD over two training steps equals NCCL all-reduce of the
    table gradient plus torch.optim.SGD on every rank: the first update
    within one rounding elementwise, both within the fp32 / bf16 tolerance
    normwise (the second step's gradient comes from the updated tables)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    sys.path.insert(0, HERE)
    import dist_gpu_worker
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=dist_gpu_worker.run_owner, args=(r, world, port, str(tmp_path), dtype_name))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in procs] == [0] * world
    ulp = 2.0 ** -7 if dtype_name == "bfloat16" else 2.0 ** -22
    tol = 2e-2 if dtype_name == "bfloat16" else 1e-5
    for r in range(world):
        d = torch.load(os.path.join(tmp_path, f"owner{r}.pt"))
        assert d["aliased"]
        for i, (ref, got) in enumerate(d["tables"]):
            ref, got = ref.float(), got.float()
            if i == 0:  # the first update: same gradient, one rounding apart at most
                assert ((got - ref).abs() <= ref.abs() * ulp + 1e-30).all()
            assert ((got - ref).abs().max() / ref.abs().max()).item() < tol


@pytest.mark.parametrize("sharded,variant", [(False, False), (True, False), (True, True)],
                         ids=["replicated", "row_sharded", "row_sharded_variant"])
@pytest.mark.parametrize("backend,world", [("gloo", 2), ("nccl", 2)])
def test_fwpkm_data_parallel_equals_one_gpu(tmp_path, backend, world, sharded, variant):
    """The fast-weight memory with its batch split over ranks on the GPU
    kernels equals one GPU running the whole batch: outputs, indices, final
    fast weights and outer gradients (fp32, 1e-5), with the value table
    replicated (``data_parallel``) or split by rows (``row_sharded``: the
    route, segment-sum and ragged-backward kernels, the owners' double
    backward; ``variant``: keys trained by the memorisation loss, weight
    decay and clipping as well).  gloo: the ranks share GPU 0; nccl: one GPU
    per rank."""
    if backend == "nccl" and torch.cuda.device_count() < world:
        pytest.skip("needs two GPUs")
    import numpy as np
    import torch.multiprocessing as mp
    sys.path.insert(0, HERE)
    import dist_gpu_worker
    import dist_worker
    torch.backends.cuda.matmul.allow_tf32 = False
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=dist_gpu_worker.run_fwpkm_dp,
                         args=(r, world, port, str(tmp_path), backend, sharded, variant))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in procs] == [0] * world
    keys, values, q, ref_v = dist_worker.fwpkm_dp_case()
    full = dist_gpu_worker.fwpkm_gpu_run(q, ref_v, keys, values, torch.device("cuda", 0),
                                         extra_kw=dist_worker.FW_VARIANT_KW if variant else None)

    def rel(a, b):
        a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
        return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))

    parts = [torch.load(os.path.join(tmp_path, f"{'fwsh' if sharded else 'fwdp'}{r}.pt")) for r in range(world)]
    for key in ("out", "q_grad", "ref_v_grad", "indices"):
        got = torch.cat([p[key] for p in parts], 0)
        if key == "indices":
            assert torch.equal(got, full[key])
        else:
            assert rel(got.numpy(), full[key].numpy()) < 1e-5, key
    for p in parts:
        for key in ("keys", "values", "keys_grad", "values_grad"):
            assert rel(p[key].numpy(), full[key].numpy()) < 1e-5, key
