"""Benchmark: PKM layer forward + backward tokens/s (the headline benchmark's config 2).

One step = forward + backward of ``HashingMemory`` at the config-2 shape
(x [8, 2048, 1024] bf16, heads 4, knn 32, k_dim 512, n_keys 512 -> 262144
slots, v_dim 1024, query BatchNorm) with loss ``sum(out**2)``; at N GPUs
every rank runs that step on its own batch (weak scaling) and the gradients
are summed over the ranks inside the step: the value table's through the
fused NVLink exchange of ``modelos_b200.dist.ShardedTableGrad``, the others
through NCCL.  Inputs are synthetic (seeded normal draws; there is no dataset).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--grad-exchange fused|nccl|owner] [--optimizer none|sgd]

``--optimizer sgd`` adds an SGD step of every parameter to each timed step
(a different metric, named in the line); with ``--grad-exchange owner`` the
table's step is sharded by rows (``modelos_b200.dist.RowOwnerSGD``).

Prints one JSON line on rank 0.  ``--impl reference`` times the CPU port of
the reference's path (``oracle/pkm_layer.py``) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "PKM layer tokens/s (fwd+bwd)"
METRIC_SGD = "PKM layer tokens/s (fwd+bwd+SGD step)"
UNIT = "tokens/s"
B, T, C = 8, 2048, 1024
CFG = dict(input_dim=1024, output_dim=1024, mem_k_dim=512, mem_v_dim=1024, mem_heads=4, mem_knn=32,
           mem_n_keys=512, mem_query_batchnorm=True, mem_query_rmsnorm=False)


def config_obj(n):
    return {"workload": "c2: HashingMemory fwd+bwd, x[8,2048,1024] bf16, H=4 knn=32 k_dim=512 "
                        "n_keys=512 (262144 slots) v_dim=1024, query BatchNorm, loss sum(out^2)",
            "tokens_per_rank_step": B * T, "global_batch": B * n, "seq_len": T,
            "parallelism": f"dp{n}" if n > 1 else "single",
            "l2": "inputs larger than L2 (value table 512 MiB, dense value grad 512 MiB per step)"}


# ---------------------------------------------------------------------------
# CPU port (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------
def cpu_port_rate(sample_tokens=256, steps=2, warmup=1):
    import numpy as np

    from oracle.pkm_layer import layer_step, make_params

    try:
        from threadpoolctl import threadpool_info
        cores = max([i.get("num_threads", 1) for i in threadpool_info()] + [1])
    except Exception:  # pragma: no cover
        cores = os.cpu_count() or 1
    P = make_params(CFG, 0)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((1, sample_tokens, C), dtype=np.float32)
    for _ in range(warmup):
        layer_step(P, x, CFG["mem_heads"], CFG["mem_knn"], norm="bn")
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        layer_step(P, x, CFG["mem_heads"], CFG["mem_knn"], norm="bn")
        ts.append(time.perf_counter() - t0)
    t = statistics.median(ts)
    cpu = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                cpu = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"value": sample_tokens / t, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{sample_tokens} tokens of the c2 layer (fwd+bwd, fp32 numpy port of "
                      f"oracle/pkm_layer.py, BLAS threads={cores}, host {os.cpu_count()} cpus {cpu}), "
                      f"median of {steps} after {warmup} warm-up; s/step={t:.3f}"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    cb = cpu_port_rate()
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * B * T / cb["value"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config_obj(world),
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# clocks sampler
# ---------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=5)
            except Exception:
                self.p.kill()
                self.out = ""
        else:
            self.out = ""

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_from_profiles():
    """Per-launch DRAM bytes from the committed ncu summary, if present."""
    out = {}
    p = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    try:
        for line in open(p):
            if "=" in line and not line.startswith("#"):
                k, v = line.split("=", 1)
                out[k.strip()] = float(v.split()[0])
    except OSError:
        pass
    return out


def bag_bytes(N, L, D, K, s_v=2, s_idx=8, s_w=2, s_out=2):
    fwd = N * L * (D * s_v + s_idx + s_w) + N * D * s_out
    kt = K * (1.0 - math.exp(-N * L / K))
    bwd = N * L * (D * s_v + s_idx + s_w + s_w) + kt * D * s_v + K * D * s_v
    return fwd, bwd


def count_launches(step, x):
    """Kernels of libpkm_b200 launched by one step (profiled outside timing)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    try:
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step(x)
            torch.cuda.synchronize()
        n = 0
        for ev in prof.events():
            if getattr(ev, "device_type", None) is not None and "CUDA" in str(ev.device_type):
                if "pkm::" in ev.name:
                    n += 1
        return n
    except Exception:
        return None


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from modelos_b200 import _native
    from modelos_b200.pkm.memory import HashingMemory

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    torch.manual_seed(1234 + rank)
    m = HashingMemory(**CFG)
    torch.manual_seed(0)  # identical parameters on every rank
    m.reset_parameters()
    m = m.to(dev, torch.bfloat16).train()
    params = [p for p in m.parameters()]
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn((B, T, C), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    x_host = x.cpu().pin_memory()
    reducer = None
    owner = None
    exchange = "none"
    if world > 1:
        from modelos_b200.dist import GradReducer, RowOwnerSGD, ShardedTableGrad
        if args.grad_exchange == "owner":
            # the table's gradient is reduce-scattered inside the bag backward;
            # its owner applies SGD to its rows and stores them into every
            # rank's table (the optimizer step below)
            owner = RowOwnerSGD(m.values.weight, lr=args.lr)
            reducer = GradReducer(params, sharded=[owner])
            exchange = "owner sgd: segment-pass stores to row owners + owner SGD and all-gather of the updated rows"
        elif args.grad_exchange == "fused":
            # the value-table gradient goes to its row owners over NVLink while
            # the bag backward computes it; owners reduce and all-gather beside
            # the rest of the backward
            ex = ShardedTableGrad(m.values.weight)
            reducer = GradReducer(params, sharded=[ex])
            exchange = {"nvls": "fused nvls: in-switch multimem all-reduce of the table gradient beside the backward",
                        "p2p": "fused p2p: segment-pass stores to row owners + owner reduce/all-gather"}[ex.mode]
        else:
            # NCCL all-reduce started as soon as the bag backward produced it
            reducer = GradReducer(params, early=[m.values.weight])
            exchange = "nccl all-reduce from a post-accumulate hook"

    opt = None
    if args.optimizer == "sgd":
        dense = [p for p in params if owner is None or p is not m.values.weight]
        opt = torch.optim.SGD(dense, lr=args.lr, foreach=True)

    def step(xin):
        for p in params:
            p.grad = None
        y, _ = m(xin)
        loss = (y.float() ** 2).sum()
        loss.backward()
        if reducer is not None:
            reducer.finish()
        if opt is not None:
            opt.step()
        if owner is not None:
            owner.step()
        return loss

    for _ in range(args.warmup):
        step(x)
    torch.cuda.synchronize()
    _native.check_device_errors(dev)

    # ---- timed region (device time, CUDA events), probes on the bag kernels
    probe = _native.EventProbe(["pkm_bag_fwd", "pkm_bag_bwd"], min_rows=m.values.weight.shape[0])
    _native.set_probe(probe)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with Clocks(local_rank) as clk:
        e0.record()
        for _ in range(args.steps):
            step(x)
        e1.record()
        torch.cuda.synchronize()
    _native.set_probe(None)
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = B * T * world / (ms / 1000.0)

    # ---- end to end: every step copies its batch from pinned host memory and
    # reads its loss back, the way a training loop with a prefetching loader
    # runs: the next batch's host-to-device copy (side stream, two device
    # buffers) overlaps the current step, and a step's loss is read once the
    # next step has been queued
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    copy_stream = torch.cuda.Stream(dev)
    bufs = [torch.empty_like(x), torch.empty_like(x)]
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    free = [torch.cuda.Event(), torch.cuda.Event()]
    compute = torch.cuda.current_stream(dev)
    for ev in free:
        ev.record(compute)
    t0 = time.perf_counter()

    def h2d(b):
        copy_stream.wait_event(free[b])
        with torch.cuda.stream(copy_stream):
            bufs[b].copy_(x_host, non_blocking=True)
            ready[b].record(copy_stream)

    h2d(0)
    pending = None
    for i in range(args.steps):
        b = i & 1
        compute.wait_event(ready[b])
        if i + 1 < args.steps:
            h2d(b ^ 1)
        loss = step(bufs[b])
        free[b].record(compute)
        if pending is not None:
            lv = pending.item()
        pending = loss
    lv = pending.item()
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / args.steps
    t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    assert math.isfinite(lv)

    # every rank runs the counted step: it holds the gradient all-reduce
    launches_per_step = count_launches(step, x)
    _native.check_device_errors(dev)

    if rank != 0:
        return
    hbm, src = peaks()
    N, L, D, K = B * T, CFG["mem_heads"] * CFG["mem_knn"], CFG["mem_v_dim"], CFG["mem_n_keys"] ** 2
    fwd_b, bwd_b = bag_bytes(N, L, D, K)
    tr = traffic_from_profiles()
    rl = {}
    for name, nbytes in (("pkm_bag_fwd", fwd_b), ("pkm_bag_bwd", bwd_b)):
        k_ms = probe.mean_ms(name)
        ach = nbytes / (k_ms / 1000.0) / 1e9
        traffic = tr.get(f"{name}.c2")
        rl[name] = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                    "frac": round(ach / hbm, 4), "traffic": traffic,
                    "kernel_ms": round(k_ms, 4), "algorithmic_bytes": int(nbytes),
                    "launches_timed": probe.count(name), "peak_source": src}
        if traffic:
            # DRAM bytes actually moved (ncu) over the live kernel time: where
            # the algorithmic rate exceeds it, the difference is served by L2
            rl[name]["dram_achieved"] = round(traffic / (k_ms / 1000.0) / 1e9, 1)
            rl[name]["dram_frac"] = round(traffic / (k_ms / 1000.0) / 1e9 / hbm, 4)
    dom = max(rl, key=lambda k: rl[k]["kernel_ms"])
    roof = dict(rl[dom])
    roof["kernel"] = dom
    other = [k for k in rl if k != dom][0]
    line = {
        "metric": METRIC if opt is None else METRIC_SGD, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded normal x, reset_parameters init)",
        "config": dict(config_obj(world), grad_exchange=exchange,
                       **({} if opt is None else {"optimizer": f"sgd lr {args.lr} (foreach; table rows by owner "
                                                                f"with --grad-exchange owner)"})),
        "e2e": {"value": round(B * T * world / (e2e_ms / 1000.0), 1), "unit": UNIT,
                "h2d_bytes_per_step": x.numel() * x.element_size(), "d2h_bytes_per_step": 4,
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": None if launches_per_step is None else launches_per_step * args.steps,
        "gpu_launches_per_step": launches_per_step,
        "roofline": roof,
        "roofline_other": dict(rl[other], kernel=other),
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_port_rate()
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--grad-exchange", default="fused", choices=["fused", "nccl", "owner"],
                    help="data-parallel exchange of the value-table gradient (N > 1); owner: the table's "
                         "optimizer sharded by rows (needs --optimizer sgd)")
    ap.add_argument("--optimizer", default="none", choices=["none", "sgd"],
                    help="add an SGD step of every parameter to each timed step")
    ap.add_argument("--lr", type=float, default=1e-6,
                    help="SGD learning rate (the loss sums 16.7 M squares: larger rates diverge)")
    args = ap.parse_args()
    if args.grad_exchange == "owner" and args.optimizer != "sgd":
        ap.error("--grad-exchange owner updates the table in the optimizer step: add --optimizer sgd")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
