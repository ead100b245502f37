"""Data-parallel gradient reduction across processes (gloo, world size 2,
CPU): the all-reduced gradients equal the sum of the single-process
gradients of every rank's batch; a rank that dies makes the others fail on
the process-group timeout instead of hanging."""
from __future__ import annotations

import os
import socket

import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(world, mode, tmp_path):
    os.environ["PYTHONPATH"] = os.pathsep.join([HERE, os.path.dirname(HERE), os.environ.get("PYTHONPATH", "")])
    import dist_worker
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=dist_worker.run, args=(r, world, port, str(tmp_path), mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    codes = []
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
        codes.append(p.exitcode)
    return codes


def test_grad_reducer_sums_rank_gradients(tmp_path, monkeypatch):
    codes = _spawn(2, "ok", tmp_path)
    assert codes == [0, 0], codes
    import dist_worker
    dist_worker.install_cpu_kernels(monkeypatch.setattr)
    ref = None
    for r in range(2):
        _, g = dist_worker.layer_grads(100 + r)
        ref = g if ref is None else {k: ref[k] + g[k] for k in ref}
    for r in range(2):
        got = torch.load(os.path.join(tmp_path, f"rank{r}.pt"))
        for k, v in ref.items():
            den = max(v.abs().max().item(), 1e-30)
            assert (got[k] - v).abs().max().item() <= 1e-5 * den, k


def test_dead_rank_fails_fast(tmp_path):
    codes = _spawn(2, "fail", tmp_path)
    assert codes[1] != 0
    assert codes[0] != 0  # the surviving rank errors out (connection closed or timeout)


def test_row_sharded_bag_matches_dense(tmp_path):
    """Row-sharded table (gloo, 2 ranks, CPU stand-in kernels): outputs, weight
    gradients and each owner's table-gradient rows equal the dense bag over
    the full table with all ranks' bags."""
    import dist_worker
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=dist_worker.run_sharded, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in procs] == [0, 0]
    dW_full = torch.zeros(dist_worker.SHARD_K, dist_worker.SHARD_D)
    for r in range(2):
        table, idx, psw, d_out = dist_worker.sharded_case(r)
        got = torch.load(os.path.join(tmp_path, f"shard{r}.pt"))
        ref = (table[idx] * psw[..., None]).sum(1)
        assert torch.allclose(got["out"], ref, atol=1e-5, rtol=1e-5)
        ref_dpsw = (table[idx] * d_out[:, None, :]).sum(-1)
        assert torch.allclose(got["dpsw"], ref_dpsw, atol=1e-5, rtol=1e-5)
        dW_full.index_add_(0, idx.reshape(-1), (d_out[:, None, :] * psw[..., None]).reshape(-1, dist_worker.SHARD_D))
    for r in range(2):
        got = torch.load(os.path.join(tmp_path, f"shard{r}.pt"))
        S = got["rows"]
        rows = dW_full[r * S:(r + 1) * S]
        assert torch.allclose(got["dW"][: rows.shape[0]], rows, atol=1e-5, rtol=1e-5)


def test_row_sharded_bad_index_raises_on_every_rank(tmp_path):
    """An index outside the table on one rank: every rank raises IndexError
    at the same step (the validity of each sender's indices travels with
    the counts), so no rank is left waiting in a collective."""
    import dist_worker
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=dist_worker.run_sharded, args=(r, 2, port, str(tmp_path), 1)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in procs] == [0, 0]
    msgs = [torch.load(os.path.join(tmp_path, f"bad{r}.pt"))["raised"] for r in range(2)]
    assert msgs[1] == "row index outside the sharded table"
    assert msgs[0] is not None and "rank(s) [1]" in msgs[0]


def _fwpkm_dp_check(tmp_path, monkeypatch, sharded, variant=False):
    import numpy as np

    import dist_worker
    import fake_native
    os.environ["PYTHONPATH"] = os.pathsep.join([HERE, os.path.dirname(HERE), os.environ.get("PYTHONPATH", "")])
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=dist_worker.run_fwpkm_dp, args=(r, 2, port, str(tmp_path), sharded, variant))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in procs] == [0, 0]
    fake_native.install(monkeypatch)
    dist_worker.install_cpu_kernels(monkeypatch.setattr)
    keys, values, q, ref_v = dist_worker.fwpkm_dp_case()
    full = dist_worker.fwpkm_run(q, ref_v, keys, values, extra_kw=dist_worker.FW_VARIANT_KW if variant else None)

    def rel(a, b):
        a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
        return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))

    tag = "fwsh" if sharded else "fwdp"
    parts = [torch.load(os.path.join(tmp_path, f"{tag}{r}.pt")) for r in range(2)]
    for key in ("out", "q_grad", "ref_v_grad", "losses", "indices"):
        got = torch.cat([p[key] for p in parts], 0)
        if key == "indices":
            assert torch.equal(got, full[key])
        else:
            assert rel(got.numpy(), full[key].numpy()) < 1e-5, key
    for p in parts:
        for key in ("keys", "values", "keys_grad", "values_grad", "grad_norms"):
            assert rel(p[key].numpy(), full[key].numpy()) < 1e-5, key
        assert abs(p["addr_loss"].item() - full["addr_loss"].item()) <= 1e-5 * abs(full["addr_loss"].item())


def test_fwpkm_data_parallel_equals_one_process(tmp_path, monkeypatch):
    """The fast-weight memory with its batch split over two gloo ranks
    (``data_parallel``): outputs, losses, indices, final fast weights and
    every outer gradient equal one process running the whole batch (fp32,
    1e-5; the sums only change order)."""
    _fwpkm_dp_check(tmp_path, monkeypatch, sharded=False)


def test_fwpkm_row_sharded_equals_one_process(tmp_path, monkeypatch):
    """The same with the value table split by rows over the two ranks
    (``row_sharded``: lookups served by the rows' owners, the value update
    and its double backward on the owners): outputs, losses, indices, the
    final fast weights (the shards gathered), every outer gradient and the
    gradient norms equal one process on the whole table."""
    _fwpkm_dp_check(tmp_path, monkeypatch, sharded=True)


def test_fwpkm_row_sharded_variant_equals_one_process(tmp_path, monkeypatch):
    """The row-split table with the memorisation loss reaching the keys too
    (``mem_grad_to_values_only=False``), weight decay (the value update's
    backward then scales the incoming gradient rather than passing it on)
    and gradient clipping: the same comparison with one process."""
    _fwpkm_dp_check(tmp_path, monkeypatch, sharded=True, variant=True)
