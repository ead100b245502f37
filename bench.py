"""Benchmark: PKM layer forward + backward tokens/s (the headline benchmark's
config 2), and the embedding bag's HBM GB/s (config 1).

One step of the default workload (``--workload c2``) = forward + backward of
``HashingMemory`` at the config-2 shape (x [8, 2048, 1024] bf16, heads 4,
knn 32, k_dim 512, n_keys 512 -> 262144 slots, v_dim 1024, query BatchNorm)
with loss ``sum(out**2)``; at N GPUs every rank runs that step on its own batch
(weak scaling) and the gradients are summed over the ranks inside the step:
the value table's through the fused NVLink exchange of
``modelos_b200.dist.ShardedTableGrad``, the others through NCCL.  The same
line carries ``emb_bag``: config 1 (bag forward + backward over a bf16
[262144, 1024] table, 16384 bags of 128 uniform indices) measured in the
same run.  ``--workload c1`` prints that measurement as its own line.
Inputs are synthetic (seeded draws with the configs' distributions; there is
no dataset).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c1] [--grad-exchange fused|nccl|owner]
                    [--optimizer none|sgd]

``--optimizer sgd`` adds an SGD step of every parameter to each timed step
(a different metric, named in the line); with ``--grad-exchange owner`` the
table's step is sharded by rows (``modelos_b200.dist.RowOwnerSGD``).

``--impl reference`` times the reference's CPU path on the host cores
instead: ``oracle/ref_torch.py``, the reference's layer step on torch's CPU
operators (bit-identical to the reference on the fixtures), in bf16 on a
2048-token slice of the workload per step; for config 1, ``F.embedding_bag``
forward + backward on 2048 of the 16384 bags.  Prints one JSON line on rank 0.
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
METRIC_C1 = "emb-bag fwd+bwd HBM GB/s (algorithmic bytes)"
UNIT = "tokens/s"
B, T, C = 8, 2048, 1024
CFG = dict(input_dim=1024, output_dim=1024, mem_k_dim=512, mem_v_dim=1024, mem_heads=4, mem_knn=32,
           mem_n_keys=512, mem_query_batchnorm=True, mem_query_rmsnorm=False)
# config 1: bags, bag size, table rows, row width
C1_N, C1_L, C1_K, C1_D = 16384, 128, 262144, 1024
# config 4: FwPKM on [8, 4096, 1024] in chunks of 512 (fp32 fast weights)
C4_B, C4_T, C4_CHUNK = 8, 4096, 512
C4_FW = dict(mem_k_dim=512, mem_v_dim=1024, mem_heads=4, mem_topk=32, mem_n_subkeys=512, learning_rate=0.1)
METRIC_C4 = "FwPKM layer tokens/s (fwd+bwd)"
METRIC_C3 = "Qwen3-PKM train tokens/s (fwd+bwd)"
C3_B, C3_T, C3_DECODE = 8, 2048, 256
REF_TOKENS = 2048   # tokens per reference-arm step (one sequence of the c2 batch)
REF_BAGS = 2048     # bags per reference-arm step at config 1


def config_obj(n, workload="c2"):
    if workload == "c3":
        return {"workload": "c3: Qwen3-0.6B-shaped decoder (hidden 1024, 28 layers, 16/8 heads, head_dim 128, "
                            "FFN 3072, vocab 151936, RoPE 1e6, tied embeddings) with HashingMemory (config-2 "
                            "geometry, query RMSNorm) in place of the MLP at layers 6, 12, 18; bf16 random init; "
                            "training step = fwd + bwd of the next-token loss on [8, 2048] uniform token ids; "
                            "prefill = [8, 2048] with KV cache; decode = 256 greedy tokens per sequence",
                "tokens_per_rank_step": C3_B * C3_T, "global_batch": C3_B * n, "seq_len": C3_T,
                "parallelism": "single", "l2": "inputs larger than L2 (PKM tables 3 x 512 MiB, logits 5 GB)"}
    if workload == "c4":
        return {"workload": "c4: FastWeightProductKeyMemory fwd (8 chunks of 512 positions, inner SGD update "
                            "lr 0.1 with create_graph) + outer bwd, x[8,4096,1024] bf16 -> q = Linear(1024->2048), "
                            "ref_v = Linear(1024->1024), k_dim 512, 4 heads x top-32 over 512^2 fp32 fast-weight "
                            "slots of 1024, idw scores, joint softmax, addressing loss me, loss sum(out^2)",
                "tokens_per_rank_step": C4_B * C4_T, "global_batch": C4_B * n, "seq_len": C4_T,
                "parallelism": "single" if n == 1 else f"dp{n}",
                "l2": "inputs larger than L2 (fp32 fast-weight table 1 GiB, updated per chunk)"}
    if workload == "c1":
        return {"workload": "c1: embedding bag fwd+bwd, table bf16 [262144,1024] N(0,0.03), 16384 bags x 128 "
                            "int64 indices uniform with replacement, fp32 per-head softmax weights, bf16 dOut",
                "bags_per_rank_step": C1_N, "parallelism": f"replicas{n}" if n > 1 else "single",
                "l2": "inputs larger than L2 (table 512 MiB, dense table gradient 512 MiB per step)"}
    return {"workload": "c2: HashingMemory fwd+bwd, x[8,2048,1024] bf16, H=4 knn=32 k_dim=512 "
                        "n_keys=512 (262144 slots) v_dim=1024, query BatchNorm, loss sum(out^2)",
            "tokens_per_rank_step": B * T, "global_batch": B * n, "seq_len": T,
            "parallelism": f"dp{n}" if n > 1 else "single",
            "l2": "inputs larger than L2 (value table 512 MiB, dense value grad 512 MiB per step)"}


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# the reference's CPU path (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------
def _timed(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return ts


def ref_layer_rate(steps=5, warmup=2, tokens=REF_TOKENS):
    """The reference's layer step (``oracle/ref_torch.py``: its torch CPU
    operators in its order, bf16) on ``tokens`` tokens of the c2 workload."""
    import torch

    from oracle import ref_torch as rt

    torch.set_num_threads(os.cpu_count() or 1)
    P = rt.make_params(CFG, 0, torch.bfloat16)
    g = torch.Generator().manual_seed(1)
    x = torch.randn((1, tokens, C), generator=g).to(torch.bfloat16)
    ts = _timed(lambda: rt.layer_step(P, x, CFG["mem_heads"], CFG["mem_knn"], CFG["mem_k_dim"], "bn"), steps, warmup)
    t = statistics.median(ts)
    cores = torch.get_num_threads()
    return {"value": tokens / t, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{tokens} tokens of the c2 layer per step (fwd+bwd, bf16, the reference's torch CPU operators "
                      f"via oracle/ref_torch.py, torch threads={cores}, host {os.cpu_count()} cpus {cpu_model()}), "
                      f"median of {steps} after {warmup} warm-up; s/step median {t:.4f} mean "
                      f"{statistics.mean(ts):.4f}",
            "ms_per_step": 1000.0 * t, "steps": steps, "warmup": warmup, "tokens_per_step": tokens}


def ref_bag_rate(steps=5, warmup=2, bags=REF_BAGS):
    """Config 1 on the reference's CPU branch (``F.embedding_bag`` forward and
    its autograd backward, ``pkm/xformer_embeddingbag.py:436-437``) over
    ``bags`` of the 16384 bags, bf16 table and weights (PKM semantics)."""
    import torch
    import torch.nn.functional as F

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    W = (torch.randn((C1_K, C1_D), generator=g) * 0.03).to(torch.bfloat16).requires_grad_(True)
    idx = torch.randint(0, C1_K, (bags, C1_L), generator=g)
    psw = torch.softmax(torch.randn((bags, 4, C1_L // 4), generator=g), -1).reshape(bags, C1_L)
    psw = psw.to(torch.bfloat16).requires_grad_(True)
    dout = torch.randn((bags, C1_D), generator=g).to(torch.bfloat16)

    def step():
        W.grad = None
        psw.grad = None
        F.embedding_bag(idx, W, per_sample_weights=psw, mode="sum").backward(dout)

    ts = _timed(step, steps, warmup)
    t = statistics.median(ts)
    fwd, bwd = bag_bytes(bags, C1_L, C1_D, C1_K, s_w=2)
    cores = torch.get_num_threads()
    return {"value": (fwd + bwd) / t / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{bags} of the {C1_N} config-1 bags per step (F.embedding_bag fwd + autograd bwd, bf16, "
                      f"torch threads={cores}, host {os.cpu_count()} cpus {cpu_model()}), median of {steps} after "
                      f"{warmup} warm-up; s/step {t:.4f}; algorithmic bytes of the sample (dense table gradient "
                      f"counted in full)",
            "ms_per_step": 1000.0 * t, "steps": steps, "warmup": warmup}


REF_C4_TOKENS = 512  # positions of one sequence per reference-arm step at config 4 (one chunk)


def ref_fw_rate(steps=3, warmup=1, tokens=REF_C4_TOKENS):
    """Config 4 on the reference's CPU path (``oracle/ref_torch.fw_step``: the
    fast-weight layer's torch CPU operators in its order, fp32 fast weights)
    on one sequence of ``tokens`` positions (one chunk of 512) per step."""
    import torch

    from oracle import ref_torch as rt

    torch.set_num_threads(os.cpu_count() or 1)
    P = rt.fw_make_params(C4_FW, 0)
    g = torch.Generator().manual_seed(1)
    q = torch.randn((1, tokens, 2048), generator=g).to(torch.bfloat16)
    v = torch.randn((1, tokens, 1024), generator=g).to(torch.bfloat16)
    keys0, values0 = P["keys"].detach().clone(), P["values"].detach().clone()

    def step():
        with torch.no_grad():
            P["keys"].copy_(keys0)
            P["values"].copy_(values0)
        rt.fw_step(P, q, v, C4_FW, C4_CHUNK, "idw")

    ts = _timed(step, steps, warmup)
    t = statistics.median(ts)
    cores = torch.get_num_threads()
    return {"value": tokens / t, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{tokens} positions (one chunk of {C4_CHUNK}) of the c4 layer per step (fwd with inner "
                      f"update + outer bwd, fp32 fast weights, the reference's torch CPU operators via "
                      f"oracle/ref_torch.py, torch threads={cores}, host {os.cpu_count()} cpus {cpu_model()}), "
                      f"median of {steps} after {warmup} warm-up; s/step {t:.3f}",
            "ms_per_step": 1000.0 * t, "steps": steps, "warmup": warmup, "tokens_per_step": tokens}


def run_reference(args, rank, world):
    if rank != 0:
        return
    steps, warmup = max(args.steps, 1), max(args.warmup, 0)
    if args.workload == "gemm":
        print(json.dumps({"impl": "reference", "unavailable": "the GEMM comparison times torch's cuBLAS beside "
                          "this library's kernel in the same line", "metric": "dense GEMM TFLOP/s"}), flush=True)
        return
    if args.workload == "c3":
        print(json.dumps({"impl": "reference", "unavailable": "config 3 runs the reference's model file "
                          "(modeling_qwen3pkm.py), which is not on the benchmark machine; the PKM layer it "
                          "calls is the default workload (c2)", "metric": METRIC_C3}), flush=True)
        return
    if args.workload == "c1":
        cb = ref_bag_rate(steps, warmup)
        metric, unit = METRIC_C1, "GB/s"
    elif args.workload == "c4":
        # a step of the CPU path takes seconds: at most 3 after 1 warm-up
        steps, warmup = min(steps, 3), min(warmup, 1)
        cb = ref_fw_rate(steps, warmup)
        metric, unit = METRIC_C4, UNIT
    else:
        cb = ref_layer_rate(steps, warmup)
        metric, unit = METRIC, UNIT
    line = {"impl": "reference", "metric": metric, "value": round(cb["value"], 3), "unit": unit,
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": round(cb["ms_per_step"], 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": config_obj(world, args.workload), "cpu_baseline": dict(cb),
            "e2e": {"value": round(cb["value"], 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    line["cpu_baseline"]["value"] = line["value"]
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# clocks: NVML sampled in a child process over the whole run, summarised over
# the samples taken inside the timed region
# ---------------------------------------------------------------------------
_SAMPLER = r"""
import sys, time
import pynvml
pynvml.nvmlInit()
try:
    h = pynvml.nvmlDeviceGetHandleByUUID(sys.argv[1])
except Exception:
    h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[2]))
print("max", pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), flush=True)
period = float(sys.argv[3])
while True:
    t = time.time()
    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
    try:
        r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
    except Exception:
        r = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h)
    print("%.6f %d %d" % (t, sm, r), flush=True)
    time.sleep(period)
"""
_REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown"}


class Clocks:
    def __init__(self, dev_index: int, period_s: float = 0.005):
        self.dev_index = dev_index
        self.period = period_s
        self.p = None
        self.window = None

    def start(self):
        import torch
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(self.dev_index).uuid)
            self.p = subprocess.Popen([sys.executable, "-c", _SAMPLER, uuid, str(self.dev_index), str(self.period)],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
        return self

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def stop(self):
        self.out = ""
        if self.p is not None:
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=10)
            except Exception:
                self.p.kill()

    def summary(self):
        mx, samples = None, []
        for line in (self.out or "").splitlines():
            f = line.split()
            if len(f) == 2 and f[0] == "max":
                mx = float(f[1])
            elif len(f) == 3:
                samples.append((float(f[0]), float(f[1]), int(f[2])))
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": ["unsampled"]}
        t0, t1 = self.window or (samples[0][0], samples[-1][0])
        inside = [s for s in samples if t0 <= s[0] <= t1]
        scope = "timed region"
        if len(inside) < 3:  # a region shorter than a few sampling periods: add the run around it
            inside = [s for s in samples if t0 - 2.0 <= s[0] <= t1 + 0.1]
            scope = "timed region and the 2 s of warm-up before it"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": ["unsampled"], "samples": 0}
        reasons = sorted({name for _, _, r in inside for bit, name in _REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(inside), "scope": scope, "source": "NVML, %.0f ms period" % (1000 * self.period)}


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
    """Algorithmic bytes of one bag forward and one bag backward (the logical
    bytes of the reference's kernels: every entry's table / upstream row read,
    the indices and weights, every touched table row read once for the weight
    gradient, the dense table gradient written in full)."""
    fwd = N * L * (D * s_v + s_idx + s_w) + N * D * s_out
    kt = K * (1.0 - math.exp(-N * L / K))
    bwd = N * L * (D * s_v + s_idx + s_w + s_w) + kt * D * s_v + K * D * s_v
    return fwd, bwd


def e2e_graph(step, x, x_host, steps, dev):
    """The end-to-end loop (c2, c4) with the step (the layer's forward and
    backward and the loss, all through the public modules) captured once in
    a CUDA graph and replayed: every step still copies its batch from
    pinned host memory (side stream, two device buffers, then a
    device-to-device copy into the graph's input) and reads its loss back.
    Returns ``(ms_per_step, None)``, or ``(None, reason)`` when the capture
    fails or its first replay does not give the eager step's loss bit for
    bit (the eager loop's number then stands)."""
    import torch
    compute = torch.cuda.current_stream(dev)
    try:
        static_x = torch.empty_like(x)
        static_x.copy_(x)
        # the reference step and the warm-up on a side stream, so that the
        # leaves' gradient accumulators are recreated off the default stream
        # (an accumulator made there would sync with it inside the capture)
        side = torch.cuda.Stream(dev)
        side.wait_stream(compute)
        with torch.cuda.stream(side):
            ref = step(static_x).detach().clone()
            for _ in range(2):
                step(static_x)
        compute.wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_loss = step(static_x)
        graph.replay()
        torch.cuda.synchronize(dev)
        if not torch.equal(static_loss, ref):
            return None, "the graph's loss differs from the eager step's"
    except Exception as e:  # the eager loop's number stands
        return None, f"capture failed ({type(e).__name__}: {str(e).splitlines()[0][:160] if str(e) else ''})"
    copy_stream = torch.cuda.Stream(dev)
    bufs = [torch.empty_like(x), torch.empty_like(x)]
    slots = [torch.empty_like(static_loss), torch.empty_like(static_loss)]
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    free = [torch.cuda.Event(), torch.cuda.Event()]
    for ev in free:
        ev.record(compute)
    torch.cuda.synchronize(dev)

    def h2d(b):
        copy_stream.wait_event(free[b])
        with torch.cuda.stream(copy_stream):
            bufs[b].copy_(x_host, non_blocking=True)
            ready[b].record(copy_stream)

    w0 = time.perf_counter()
    h2d(0)
    pending = None
    lv = None
    for i in range(steps):
        b = i & 1
        compute.wait_event(ready[b])
        static_x.copy_(bufs[b])
        free[b].record(compute)
        if i + 1 < steps:
            h2d(b ^ 1)
        graph.replay()
        slots[b].copy_(static_loss)  # the next replay overwrites the graph's loss
        if pending is not None:
            lv = pending.item()
        pending = slots[b]
    lv = pending.item()
    torch.cuda.synchronize(dev)
    ms = (time.perf_counter() - w0) * 1000.0 / steps
    del graph
    if not math.isfinite(lv):
        return None, "non-finite loss in the graph loop"
    return ms, None


def count_launches(step, *a):
    """Kernels of libpkm_b200 launched by one step (profiled outside timing)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    try:
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step(*a)
            torch.cuda.synchronize()
        n = 0
        for ev in prof.events():
            if getattr(ev, "device_type", None) is not None and "CUDA" in str(ev.device_type):
                if "pkm::" in ev.name:
                    n += 1
        return n
    except Exception:
        return None


def _roof(nbytes, k_ms, hbm, src, traffic, launches):
    if k_ms is None or not (k_ms > 0):
        return None
    ach = nbytes / (k_ms / 1000.0) / 1e9
    r = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s", "frac": round(ach / hbm, 4),
         "traffic": traffic, "kernel_ms": round(k_ms, 4), "algorithmic_bytes": int(nbytes),
         "launches_timed": launches, "peak_source": src}
    if traffic:
        # DRAM bytes actually moved (ncu) over the live kernel time: where
        # the algorithmic rate exceeds it, the difference is served by L2
        r["dram_achieved"] = round(traffic / (k_ms / 1000.0) / 1e9, 1)
        r["dram_frac"] = round(traffic / (k_ms / 1000.0) / 1e9 / hbm, 4)
    return r


def c1_inputs(dev, seed=0):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    W = (torch.randn((C1_K, C1_D), generator=g, device=dev) * 0.03).to(torch.bfloat16)
    idx = torch.randint(0, C1_K, (C1_N, C1_L), generator=g, device=dev)
    psw = torch.softmax(torch.randn((C1_N, 4, C1_L // 4), generator=g, device=dev), -1).reshape(C1_N, C1_L)
    dout = torch.randn((C1_N, C1_D), generator=g, device=dev).to(torch.bfloat16)
    return W, idx, psw.contiguous(), dout


def measure_c1(dev, steps, warmup):
    """Config 1 on this library's kernels: one step = K3 (bag forward) + K4
    (bag backward: dense table gradient and weight gradient), inputs resident,
    device time by CUDA events.  Returns the timing and roofline fields."""
    import torch

    from modelos_b200 import _native
    W, idx, psw, dout = c1_inputs(dev)
    dW = torch.empty_like(W)
    probe = _native.EventProbe(["pkm_bag_fwd", "pkm_bag_bwd"], min_rows=C1_K)

    def step():
        _native.bag_fwd(idx, W, psw)
        _native.bag_bwd(idx, W, psw, dout, out=dW)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    _native.set_probe(probe)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    _native.set_probe(None)
    _native.check_device_errors(dev)
    ms = e0.elapsed_time(e1) / steps
    fwd, bwd = bag_bytes(C1_N, C1_L, C1_D, C1_K, s_w=4)
    hbm, src = peaks()
    tr = traffic_from_profiles()
    res = {"ms_per_step": round(ms, 4), "gbs": round((fwd + bwd) / (ms / 1000.0) / 1e9, 1),
           "algorithmic_bytes_per_step": int(fwd + bwd), "peak": hbm, "peak_source": src,
           "frac": round((fwd + bwd) / (ms / 1000.0) / 1e9 / hbm, 4),
           "roofline_60pct_ms": round((fwd + bwd) / (0.6 * hbm * 1e9) * 1000.0, 4)}
    for name, nb in (("pkm_bag_fwd", fwd), ("pkm_bag_bwd", bwd)):
        res[name] = _roof(nb, probe.mean_ms(name), hbm, src, tr.get(f"{name}.c1"), probe.count(name))
    return res, (W, idx, psw, dout, dW, step)


def run_ours_c1(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from modelos_b200 import _native
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    clk = Clocks(local_rank).start()
    res, (W, idx, psw, dout, dW, step) = measure_c1(dev, 1, args.warmup)  # warm-up run
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.time()
    res, _ = measure_c1(dev, args.steps, 0)
    clk.mark(t0, time.time())
    t = torch.tensor([res["ms_per_step"]], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # end to end: each step copies its indices, weights and upstream gradient
    # from pinned host memory and reads the weight gradient back
    h_idx, h_psw, h_dout = idx.cpu().pin_memory(), psw.cpu().pin_memory(), dout.cpu().pin_memory()
    h_dpsw = torch.empty(psw.shape, dtype=psw.dtype).pin_memory()
    d_idx, d_psw, d_dout = torch.empty_like(idx), torch.empty_like(psw), torch.empty_like(dout)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        d_idx.copy_(h_idx, non_blocking=True)
        d_psw.copy_(h_psw, non_blocking=True)
        d_dout.copy_(h_dout, non_blocking=True)
        _native.bag_fwd(d_idx, W, d_psw)
        _, dpsw, _ = _native.bag_bwd(d_idx, W, d_psw, d_dout, out=dW)
        h_dpsw.copy_(dpsw, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    e2e_ms = (time.perf_counter() - w0) * 1000.0 / args.steps
    t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    launches = count_launches(step)
    clk.stop()
    if rank != 0:
        return
    nbytes = res["algorithmic_bytes_per_step"]
    roof = res["pkm_bag_bwd"] if (res["pkm_bag_bwd"] or {}).get("kernel_ms", 0) >= \
        (res["pkm_bag_fwd"] or {}).get("kernel_ms", 0) else res["pkm_bag_fwd"]
    dom = "pkm_bag_bwd" if roof is res["pkm_bag_bwd"] else "pkm_bag_fwd"
    line = {"metric": METRIC_C1, "value": round(nbytes * world / (ms / 1000.0) / 1e9, 1), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded: table N(0,0.03), uniform indices, softmax weights, N(0,1) dOut)",
            "config": config_obj(world, "c1"),
            "e2e": {"value": round(nbytes * world / (e2e_ms / 1000.0) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": idx.numel() * 8 + psw.numel() * 4 + dout.numel() * 2,
                    "d2h_bytes_per_step": psw.numel() * 4, "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": None if launches is None else launches * args.steps,
            "gpu_launches_per_step": launches,
            "roofline": dict(roof, kernel=dom), "frac_of_step": res["frac"],
            "roofline_60pct_ms": res["roofline_60pct_ms"], "kernels": {k: res[k] for k in ("pkm_bag_fwd",
                                                                                         "pkm_bag_bwd")},
            "clocks": clk.summary()}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = ref_bag_rate()
    print(json.dumps(line), flush=True)


def run_ours_c4(args, rank, world, local_rank):
    """Config 4: the fast-weight memory's chunked forward with its inner
    updates, then the outer backward through them; at N GPUs every rank runs
    its own 8 sequences (weak scaling) and the inner updates use the whole
    batch, with the value table split by rows over the ranks
    (``row_sharded``, the default) or replicated (``data_parallel``,
    ``--fw-table replicated``)."""
    import torch

    from modelos_b200 import _native
    from modelos_b200.fwpkm.fwpkm import FastWeightProductKeyMemory
    from modelos_b200.pkm.memory import LinearColsumBias

    import torch.distributed as dist

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    clk = Clocks(local_rank).start()
    torch.manual_seed(0)  # identical parameters on every rank
    m = FastWeightProductKeyMemory(**C4_FW).to(dev).train()
    m.reset_parameters()
    wq = torch.nn.Linear(1024, 2048).to(dev, torch.bfloat16)
    wv = torch.nn.Linear(1024, 1024).to(dev, torch.bfloat16)
    proj = list(wq.parameters()) + list(wv.parameters())
    if world > 1:
        if args.fw_table == "sharded":
            # batch split over the ranks, value rows split over the ranks:
            # lookups and their gradients travel to the rows' owners
            m.row_sharded(dist.group.WORLD)
        else:
            # batch split over the ranks, fast weights replicated, every inner
            # update from the whole batch's gradient (differentiable all-reduces)
            m.data_parallel(dist.group.WORLD)
    keys0, values0 = m.keys.detach().clone(), m.values.detach().clone()
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn((C4_B, C4_T, 1024), generator=g, device=dev).to(torch.bfloat16)
    x_host = x.cpu().pin_memory()

    def step(xin):
        # every step starts from the same fast weights (the layer writes the
        # final ones back into its parameters)
        with torch.no_grad():
            m.keys.copy_(keys0)
            m.values.copy_(values0)
        for p in list(m.parameters()) + list(wq.parameters()) + list(wv.parameters()):
            p.grad = None
        xf = xin.view(-1, 1024)
        q = LinearColsumBias.apply(xf, wq.weight, wq.bias).view(C4_B, C4_T, -1)
        ref_v = LinearColsumBias.apply(xf, wv.weight, wv.bias).view(C4_B, C4_T, -1)
        res = m(q, ref_v, None, C4_CHUNK)
        loss = (res["output"].float() ** 2).sum()
        loss.backward()
        if world > 1:
            m.reduce_grads()
            for p in proj:
                dist.all_reduce(p.grad)
        return loss

    for _ in range(args.warmup):
        step(x)
    torch.cuda.synchronize()
    _native.check_device_errors(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.time()
    e0.record()
    for _ in range(args.steps):
        step(x)
    e1.record()
    torch.cuda.synchronize()
    clk.mark(t0, time.time())
    if world > 1:
        dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    d_x = torch.empty_like(x)
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        d_x.copy_(x_host, non_blocking=True)
        lv = step(d_x).item()
    e2e_ms = (time.perf_counter() - w0) * 1000.0 / args.steps
    t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    assert math.isfinite(lv)
    launches = count_launches(step, x)
    _native.check_device_errors(dev)
    clk.stop()
    # last, so that a capture that went wrong can cost nothing else
    graph_ms, graph_note = (None, "not attempted (N > 1 or --no-graph)")
    if world == 1 and not args.no_graph:
        lv = None
        graph_ms, graph_note = e2e_graph(step, x, x_host, args.steps, dev)
        _native.check_device_errors(dev)
    if rank != 0:
        return
    tokens = C4_B * C4_T * world
    line = {"metric": METRIC_C4, "value": round(tokens / (ms / 1000.0), 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 inputs, fp32 fast weights",
            "data": "synthetic (seeded normal x, reset_parameters init, default nn.Linear projections)",
            "config": config_obj(world, "c4"),
            "e2e": ({"value": round(tokens / (graph_ms / 1000.0), 1), "unit": UNIT,
                     "h2d_bytes_per_step": x.numel() * x.element_size(), "d2h_bytes_per_step": 4,
                     "ms_per_step": round(graph_ms, 4),
                     "graph": "the step captured once in a CUDA graph, replayed per step (its first replay's loss "
                              "equals the eager step's bit for bit)",
                     "eager": {"value": round(tokens / (e2e_ms / 1000.0), 1), "ms_per_step": round(e2e_ms, 4)}}
                    if graph_ms is not None else
                    {"value": round(tokens / (e2e_ms / 1000.0), 1), "unit": UNIT,
                     "h2d_bytes_per_step": x.numel() * x.element_size(), "d2h_bytes_per_step": 4,
                     "ms_per_step": round(e2e_ms, 4), "graph": graph_note}),
            "gpu_launches": None if launches is None else launches * args.steps, "gpu_launches_per_step": launches,
            "clocks": clk.summary()}
    if world > 1 and args.fw_table == "sharded":
        line["config"]["fw_table"] = "value rows split over the ranks (row_sharded)"
        line["config"]["exchange"] = ("per chunk: all-to-alls of the lookups to the rows' owners and of the owners' "
                                      "partial bag sums back, in the backward of the upstream rows to the owners "
                                      "and of the weight gradients back (twice more for the double backward); "
                                      "differentiable all-reduces of the key gradients and of the addressing "
                                      "loss's row sums; no value-table gradient crosses the links; after the "
                                      "step, all-reduce of the keys' and the projections' gradients")
    elif world > 1:
        line["config"]["fw_table"] = "replicated (data_parallel)"
        line["config"]["exchange"] = ("per chunk: differentiable all-reduces of the fast-weight gradients (fp32 "
                                      "values 1 GiB, keys) and of the addressing loss's row sums, all-gather of the "
                                      "slot indices; after the step, all-reduce of the parameters' gradients")
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = ref_fw_rate()
    print(json.dumps(line), flush=True)


def run_ours_c3(args, rank, world, local_rank):
    """Config 3 on one GPU: the model's training step (forward + backward),
    then a prefill and a decode loop in evaluation mode."""
    import torch

    from modelos_b200 import _native
    from modelos_b200.qwen3pkm import build_qwen3_pkm

    if world > 1:
        raise SystemExit("--workload c3 runs on one GPU")
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    clk = Clocks(local_rank).start()
    model = build_qwen3_pkm(device=dev, dtype=torch.bfloat16).train()
    g = torch.Generator(device=dev).manual_seed(0)
    ids = torch.randint(0, model.config.vocab_size, (C3_B, C3_T), generator=g, device=dev)
    ids_host = ids.cpu().pin_memory()
    params = [p for p in model.parameters()]

    def step(x):
        for p in params:
            p.grad = None
        out = model(input_ids=x, labels=x, use_cache=False)
        out.loss.backward()
        return out.loss

    for _ in range(args.warmup):
        step(ids)
    torch.cuda.synchronize()
    _native.check_device_errors(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    e0.record()
    for _ in range(args.steps):
        step(ids)
    e1.record()
    torch.cuda.synchronize()
    clk.mark(t0, time.time())
    ms = e0.elapsed_time(e1) / args.steps
    d_ids = torch.empty_like(ids)
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        d_ids.copy_(ids_host, non_blocking=True)
        lv = step(d_ids).item()
    e2e_ms = (time.perf_counter() - w0) * 1000.0 / args.steps
    assert math.isfinite(lv)
    launches = count_launches(step, ids)
    for p in params:
        p.grad = None

    # prefill and decode (evaluation mode, KV cache)
    model.eval()
    with torch.no_grad():
        for _ in range(2):
            model(input_ids=ids, use_cache=True)
        torch.cuda.synchronize()
        e0.record()
        out = model(input_ids=ids, use_cache=True)
        e1.record()
        torch.cuda.synchronize()
        prefill_ms = e0.elapsed_time(e1)
        cache = out.past_key_values
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        # cuDNN's attention plans every new KV length on the host
        # (milliseconds a decode step); decode on the flash backend
        torch.backends.cuda.enable_cudnn_sdp(False)
        e0.record()
        for _ in range(C3_DECODE):
            out = model(input_ids=nxt, past_key_values=cache, use_cache=True)
            cache = out.past_key_values
            nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        e1.record()
        torch.cuda.synchronize()
        decode_ms = e0.elapsed_time(e1)
    _native.check_device_errors(dev)
    clk.stop()
    tokens = C3_B * C3_T
    line = {"metric": METRIC_C3, "value": round(tokens / (ms / 1000.0), 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform token ids, random init)", "config": config_obj(world, "c3"),
            "prefill": {"tokens_per_s": round(tokens / (prefill_ms / 1000.0), 1), "ms": round(prefill_ms, 3),
                        "tokens": tokens},
            "decode": {"tokens_per_s": round(C3_B * C3_DECODE / (decode_ms / 1000.0), 1),
                       "ms_per_token_step": round(decode_ms / C3_DECODE, 4), "batch": C3_B, "steps": C3_DECODE},
            "e2e": {"value": round(tokens / (e2e_ms / 1000.0), 1), "unit": UNIT,
                    "h2d_bytes_per_step": ids.numel() * ids.element_size(), "d2h_bytes_per_step": 4,
                    "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": None if launches is None else launches * args.steps, "gpu_launches_per_step": launches,
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


GEMM_SHAPES = (  # the dense GEMMs of one c2 step: name, M, N, K, A MN-major, B MN-major
    ("query fwd", 16384, 2048, 1024, False, False), ("swilu/value fwd", 16384, 1024, 1024, False, False),
    ("query dgrad", 16384, 1024, 2048, False, True), ("swilu/value dgrad", 16384, 1024, 1024, False, True),
    ("query wgrad", 2048, 1024, 16384, True, True), ("swilu/value wgrad", 1024, 1024, 16384, True, True))


def run_ours_gemm(args, rank, world, local_rank):
    """The dense GEMM shapes of one c2 step on this library's tensor-core
    GEMM and on torch's matmul (cuBLAS), device-timed; one line with the
    per-shape times and rates."""
    import torch

    from modelos_b200 import _native
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    bf = torch.bfloat16
    torch.manual_seed(0)

    def timed(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps * 1000.0

    rows, ours_total, torch_total, flops = [], 0.0, 0.0, 0.0
    for name, M, N, K, amn, bmn in GEMM_SHAPES:
        a = torch.randn((K, M) if amn else (M, K), device=dev, dtype=bf)
        b = torch.randn((K, N) if bmn else (N, K), device=dev, dtype=bf)
        A, Bt = (a.t() if amn else a), (b if bmn else b.t())
        uo = timed(lambda: _native.gemm(a, b, a_mn=amn, b_mn=bmn))
        ut = timed(lambda: A @ Bt)
        f = 2.0 * M * N * K
        rows.append({"gemm": name, "M": M, "N": N, "K": K, "ours_us": round(uo, 1), "torch_us": round(ut, 1),
                     "ours_tflops": round(f / uo / 1e6, 1), "torch_tflops": round(f / ut / 1e6, 1)})
        ours_total += uo
        torch_total += ut
        flops += f
    T, G, n, half = 16384, 8, 512, 256
    dS = torch.randn(T, G * n, device=dev, dtype=bf)
    keys = torch.randn(G * n, half, device=dev, dtype=bf)
    q = torch.randn(T, G * half, device=dev, dtype=bf)
    dq = torch.empty(T, G * half, device=dev, dtype=bf)
    dk = torch.empty(G * n, half, device=dev, dtype=bf)
    u1 = timed(lambda: _native.gemm(dS, keys, b_mn=True, batch=G, M=T, N=half, K=n, a_batch=(n, 0), b_batch=(0, n),
                                    out=dq, c_batch_stride=half))
    u2 = timed(lambda: _native.gemm(dS, q, a_mn=True, b_mn=True, batch=G, M=n, N=half, K=T, a_batch=(n, 0),
                                    b_batch=(half, 0), out=dk, c_batch_stride=n * half))
    dSv = dS.view(T, G, n)
    dqv = torch.empty(T, G, half, device=dev, dtype=bf)
    t1 = timed(lambda: torch.bmm(dSv.transpose(0, 1), keys.view(G, n, half), out=dqv.transpose(0, 1)))
    t2 = timed(lambda: torch.bmm(dSv.permute(1, 2, 0), q.view(T, G, half).transpose(0, 1)))
    fb = 2.0 * T * G * n * half
    rows.append({"gemm": "score dq (batched 8)", "ours_us": round(u1, 1), "torch_us": round(t1, 1),
                 "ours_tflops": round(fb / u1 / 1e6, 1), "torch_tflops": round(fb / t1 / 1e6, 1)})
    rows.append({"gemm": "score dk (batched 8)", "ours_us": round(u2, 1), "torch_us": round(t2, 1),
                 "ours_tflops": round(fb / u2 / 1e6, 1), "torch_tflops": round(fb / t2 / 1e6, 1)})
    _native.check_device_errors(dev)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        peak = 1590.0
    rate = flops / ours_total / 1e6
    print(json.dumps({"metric": "dense GEMM TFLOP/s over the c2 step's projection shapes", "value": round(rate, 1),
                      "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "higher_is_better": True, "dtype": "bf16",
                      "roofline": {"bound": "tensor", "achieved": round(rate, 1), "peak": peak, "unit": "TFLOP/s",
                                   "frac": round(rate / peak, 4), "peak_source": "measured cuBLAS bf16 burst"},
                      "torch_cublas_tflops": round(flops / torch_total / 1e6, 1), "shapes": rows}), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from modelos_b200 import _native
    from modelos_b200.pkm.memory import HashingMemory

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    clk = Clocks(local_rank).start()
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
    exchanges = []
    waits = []  # (before, after) events around the caller's wait for the gradient exchange
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
            exchanges.append(ex)
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

    timing_on = [False]

    def step(xin):
        for p in params:
            p.grad = None
        y, _ = m(xin)
        loss = (y.float() ** 2).sum()
        loss.backward()
        if reducer is not None:
            if timing_on[0]:
                a = torch.cuda.Event(enable_timing=True)
                a.record()
            reducer.finish()
            if timing_on[0]:
                b = torch.cuda.Event(enable_timing=True)
                b.record()
                waits.append((a, b))
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
    names = ["pkm_bag_fwd", "pkm_bag_bwd", "pkm_bag_bwd_sort", "pkm_bag_bwd_rows"]
    probe = _native.EventProbe(names, min_rows=m.values.weight.shape[0])
    _native.set_probe(probe)
    timing_on[0] = True
    for ex in exchanges:
        ex.timing = True
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    e0.record()
    for _ in range(args.steps):
        step(x)
    e1.record()
    torch.cuda.synchronize()
    clk.mark(t0, time.time())
    _native.set_probe(None)
    timing_on[0] = False
    for ex in exchanges:
        ex.timing = False
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    ex_ms = [e.exchange_ms() for e in exchanges]
    ex_ms = ex_ms[0] if ex_ms and ex_ms[0] is not None else None
    wait_ms = sum(a.elapsed_time(b) for a, b in waits) / len(waits) if waits else None
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
    w0 = time.perf_counter()

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
    e2e_ms = (time.perf_counter() - w0) * 1000.0 / args.steps
    t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    assert math.isfinite(lv)

    # every rank runs the counted step: it holds the gradient all-reduce
    launches_per_step = count_launches(step, x)
    _native.check_device_errors(dev)

    # config 1 in the same run (rank 0 of a single-GPU run: the replicated
    # bag microbenchmark has no data-parallel form)
    emb = None
    if world == 1:
        del bufs
        emb, _ = measure_c1(dev, max(args.steps, 20), max(args.warmup, 3))
    clk.stop()
    # last, so that a capture that went wrong can cost nothing else
    graph_ms, graph_note = (None, "not attempted (N > 1 or --no-graph)")
    if world == 1 and not args.no_graph:
        # no loss of an earlier step may keep its autograd graph, and with it
        # the gradient accumulators made on the default stream, alive
        loss = pending = None
        graph_ms, graph_note = e2e_graph(step, x, x_host, args.steps, dev)

    if rank != 0:
        return
    hbm, src = peaks()
    N, L, D, K = B * T, CFG["mem_heads"] * CFG["mem_knn"], CFG["mem_v_dim"], CFG["mem_n_keys"] ** 2
    fwd_b, bwd_b = bag_bytes(N, L, D, K)
    tr = traffic_from_profiles()
    # the bag backward is one launch, or (in-switch exchange) a sort launch
    # followed by row-range launches: time per backward = their sum per step
    n_bwd = probe.count("pkm_bag_bwd") or probe.count("pkm_bag_bwd_sort")
    bwd_ms = None
    if n_bwd:
        bwd_ms = (probe.total_ms("pkm_bag_bwd") + probe.total_ms("pkm_bag_bwd_sort")
                  + probe.total_ms("pkm_bag_bwd_rows")) / n_bwd
    rl = {"pkm_bag_fwd": _roof(fwd_b, probe.mean_ms("pkm_bag_fwd"), hbm, src, tr.get("pkm_bag_fwd.c2"),
                               probe.count("pkm_bag_fwd")),
          "pkm_bag_bwd": _roof(bwd_b, bwd_ms, hbm, src, tr.get("pkm_bag_bwd.c2"), n_bwd)}
    if probe.count("pkm_bag_bwd_sort"):
        rl["pkm_bag_bwd"]["phases"] = "pkm_bag_bwd_sort + pkm_bag_bwd_rows (row ranges beside the exchange)"
    timed = {k: v for k, v in rl.items() if v is not None}
    dom = max(timed, key=lambda k: timed[k]["kernel_ms"]) if timed else None
    line = {
        "metric": METRIC if opt is None else METRIC_SGD, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded normal x, reset_parameters init)",
        "config": dict(config_obj(world), grad_exchange=exchange,
                       **({} if opt is None else {"optimizer": f"sgd lr {args.lr} (foreach; table rows by owner "
                                                                f"with --grad-exchange owner)"})),
        "e2e": ({"value": round(B * T * world / (graph_ms / 1000.0), 1), "unit": UNIT,
                 "h2d_bytes_per_step": x.numel() * x.element_size(), "d2h_bytes_per_step": 4,
                 "ms_per_step": round(graph_ms, 4),
                 "graph": "the step captured once in a CUDA graph, replayed per step (its first replay's loss "
                          "equals the eager step's bit for bit)",
                 "eager": {"value": round(B * T * world / (e2e_ms / 1000.0), 1), "ms_per_step": round(e2e_ms, 4)}}
                if graph_ms is not None else
                {"value": round(B * T * world / (e2e_ms / 1000.0), 1), "unit": UNIT,
                 "h2d_bytes_per_step": x.numel() * x.element_size(), "d2h_bytes_per_step": 4,
                 "ms_per_step": round(e2e_ms, 4), "graph": graph_note}),
        "gpu_launches": None if launches_per_step is None else launches_per_step * args.steps,
        "gpu_launches_per_step": launches_per_step,
        "roofline": dict(rl[dom], kernel=dom) if dom else None,
        "roofline_other": {k: v for k, v in rl.items() if k != dom},
        "clocks": clk.summary(),
    }
    if world > 1:
        # the table gradient's exchange on its side stream, and the part of
        # it (with the small gradients' NCCL all-reduce) the step waits for
        line["exchange_ms"] = None if ex_ms is None else round(ex_ms, 4)
        line["exchange_exposed_ms"] = None if wait_ms is None else round(wait_ms, 4)
    if emb is not None:
        line["emb_bag"] = dict(emb, metric=METRIC_C1, config=config_obj(1, "c1")["workload"])
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = ref_layer_rate()
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c2", "c1", "c3", "c4", "gemm"],
                    help="c2: the PKM layer (default); c1: the embedding bag alone; c3: the Qwen3-PKM model "
                         "(train step, prefill, decode); c4: the fast-weight memory; gemm: the c2 step's GEMM "
                         "shapes on this library's GEMM and on cuBLAS")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="c2 at N=1: the end-to-end loop without the CUDA-graph replay")
    ap.add_argument("--fw-table", default="sharded", choices=["sharded", "replicated"],
                    help="c4 at N > 1: the fast-weight value table split by rows over the ranks, or replicated")
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
    if args.warmup < 3 and args.impl == "ours":
        ap.error("--warmup must be at least 3")
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
        if args.workload == "c1":
            run_ours_c1(args, rank, world, local_rank)
        elif args.workload == "c4":
            run_ours_c4(args, rank, world, local_rank)
        elif args.workload == "c3":
            run_ours_c3(args, rank, world, local_rank)
        elif args.workload == "gemm":
            run_ours_gemm(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
