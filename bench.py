"""Benchmark: GQA decode attention, KV GB/s and tokens/s (BASELINE metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl molot|reference]
                    [--config cfg2|cfg1|cfg3|cfg4|cfg5]

Default workload ("cfg2"): one decode step of a 32-layer
Llama-shaped model at 16k context -- Hq=32, Hkv=8, head_dim=128, 16384 cached
slots + the new token (n=16385), RoPE theta=5e5.  Per layer the step runs
the library's public call molot_attn_step: QK-norm/RoPE of the raw q/k, the
append of the new row and split-KV decode over the HBM-resident cache, in
one launch (--path split: molot_attn_append_rope + molot_attn_decode, two
launches).  K/V and
q/k/v are seeded N(0,1) synthetic data generated on the device.  The 4.3 GB
of KV is far larger than L2 (126 MB), so no flush is needed.

value  : unique KV bytes (2*Hkv*n*d*4 per layer, all layers, all ranks)
         / max-over-ranks device time of the K timed steps, inputs resident.
e2e    : the same metric through the same public API with the step's inputs
         (raw q/k/v of every layer) copied host->device from pinned memory
         and the attention outputs copied back, inside the timed region.
With N>1 every rank runs its own replica (one sequence per GPU, weak
scaling, no collective on the data path).

--impl reference times the reference's own CPU implementation
(attn_decode_gqa_cache from attn.h, compiled unchanged into
oracle/_ref/libmolot_ref.so, AVX-512 + its ThreadPool over all host cores)
on a bounded sample of the same workload; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (layers, nq, nkv, d, n_cached, rope_theta, window, scale)
    "cfg1": dict(layers=32, nq=32, nkv=8, d=128, ctx=4096, theta=1e4, window=0,
                 desc="single-sequence GQA decode, ctx 4096 (bench.cc shape)"),
    "cfg2": dict(layers=32, nq=32, nkv=8, d=128, ctx=16384, theta=5e5, window=0,
                 desc="single-sequence GQA decode, ctx 16384, 32-layer sweep"),
}
METRIC = "GQA decode attn KV GB/s (% of HBM peak) and tok/s at ctx 16k, 1/2/4/8 GPU"


def hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def read_traffic(kernel: str, workload: str):
    """dram bytes per launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 3 and parts[0] == kernel and parts[1] == workload:
                return float(parts[2])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------------ reference arm

def run_reference(args, cfg):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    import oracle
    lib = oracle.ref()
    kind = "reference"
    if lib is None:
        kind = "port"
    cores = os.cpu_count() or 1
    nq, nkv, d, n = cfg["nq"], cfg["nkv"], cfg["d"], cfg["ctx"] + 1
    scale = 1.0 / math.sqrt(d)
    rng = np.random.default_rng(7)
    nbuf = 2  # distinct layer buffers, each 134 MB >> any CPU cache
    bufs = [(rng.standard_normal((nq, d), dtype=np.float32),
             rng.standard_normal((n, nkv * d), dtype=np.float32),
             rng.standard_normal((n, nkv * d), dtype=np.float32)) for _ in range(nbuf)]

    def one(i):
        Q, K, V = bufs[i % nbuf]
        if kind == "reference":
            oracle.attn_decode_gqa_cache(Q, K, V, nq, nkv, n, d, scale, n - 1, 0, impl="ref",
                                         nthreads=cores)
        else:
            oracle.attn_decode_gqa_cache(Q, K, V, nq, nkv, n, d, scale, n - 1, 0)

    layers_per_step = 2
    for i in range(args.warmup):
        one(i)
    t0 = time.perf_counter()
    for i in range(args.steps * layers_per_step):
        one(i)
    dt = (time.perf_counter() - t0) / (args.steps * layers_per_step)  # s per layer
    kv_bytes = 2 * nkv * n * d * 4
    value = kv_bytes / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * cfg["layers"] * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.config}: {cfg['desc']} (reference CPU, per-layer sample)",
                   "layers": cfg["layers"], "nq": nq, "nkv": nkv, "head_dim": d, "n": n},
        "tok_per_s": round(1.0 / (dt * cfg["layers"]), 3),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": f"{args.steps * layers_per_step} layer calls of "
                                   f"attn_decode_gqa_cache (n={n}) over {nbuf} buffers; "
                                   "per-step time = 32 x mean layer time"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def cpu_baseline_sample(cfg):
    """A bounded reference sample for the GPU arm's cpu_baseline key."""
    import oracle
    lib = oracle.ref()
    kind = "reference" if lib is not None else "port"
    cores = (os.cpu_count() or 1) if kind == "reference" else 1
    nq, nkv, d, n = cfg["nq"], cfg["nkv"], cfg["d"], cfg["ctx"] + 1
    rng = np.random.default_rng(11)
    Q = rng.standard_normal((nq, d), dtype=np.float32)
    K = rng.standard_normal((n, nkv * d), dtype=np.float32)
    V = rng.standard_normal((n, nkv * d), dtype=np.float32)
    scale = 1.0 / math.sqrt(d)
    calls, t_total = 0, 0.0
    budget = 10.0 if kind == "reference" else 6.0
    while t_total < budget and calls < 400:
        t0 = time.perf_counter()
        if kind == "reference":
            oracle.attn_decode_gqa_cache(Q, K, V, nq, nkv, n, d, scale, n - 1, 0, impl="ref",
                                         nthreads=cores)
        else:
            oracle.attn_decode_gqa_cache(Q, K, V, nq, nkv, n, d, scale, n - 1, 0)
        t_total += time.perf_counter() - t0
        calls += 1
    dt = t_total / calls
    return {"value": round(2 * nkv * n * d * 4 / dt / 1e9, 3), "unit": "GB/s", "cores": cores,
            "kind": kind,
            "sample": f"{calls} calls of attn_decode_gqa_cache (one layer, n={n}, "
                      f"{nq}/{nkv}/{d}) ~{t_total:.1f}s"}


# ------------------------------------------------------------------ molot arm

def run_molot(args, cfg):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    torch.cuda.set_device(local)
    import molot_b200 as mb

    L, nq, nkv, d = cfg["layers"], cfg["nq"], cfg["nkv"], cfg["d"]
    ctx = cfg["ctx"]
    n = ctx + 1
    scale = 1.0 / math.sqrt(d)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()

    cache = mb.KVCache(L, nkv, d, n)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    for layer in range(L):
        kt, vt = cache.layer_tensors(layer)  # head-major [nkv][cap][hd]
        kt[:, :ctx].normal_(generator=gen)
        vt[:, :ctx].normal_(generator=gen)
    q_raw = torch.randn((L, nq * d), device=dev, generator=gen)
    k_raw = torch.randn((L, nkv * d), device=dev, generator=gen)
    v_raw = torch.randn((L, nkv * d), device=dev, generator=gen)
    q_norm = (1 + 0.1 * torch.randn(d, device=dev, generator=gen)).contiguous()
    k_norm = (1 + 0.1 * torch.randn(d, device=dev, generator=gen)).contiguous()
    freq = torch.tensor([1.0 / cfg["theta"] ** (2.0 * i / d) for i in range(d // 2)],
                        dtype=torch.float32, device=dev)
    q_rot = torch.randn((L, nq * d), device=dev, generator=gen)
    out = torch.empty((L, nq * d), device=dev)
    torch.cuda.synchronize()

    fused = args.path == "fused"

    def step(qr, kr, vr, o, decode_only=False):
        st = torch.cuda.current_stream()
        for layer in range(L):
            if decode_only:
                cache.decode(layer, q_rot[layer], o[layer], scale, ctx, cfg["window"], nq, st)
                continue
            cache.set_length(layer, ctx)
            if fused:
                cache.step(layer, qr[layer], kr[layer], vr[layer], o[layer], scale, ctx,
                           cfg["window"], q_norm, k_norm, False, 1e-6, freq, nq, st)
            else:
                cache.append_rope(layer, qr[layer], kr[layer], vr[layer], q_rot[layer], q_norm,
                                  k_norm, False, 1e-6, freq, ctx, nq, st)
                cache.decode(layer, q_rot[layer], o[layer], scale, ctx, cfg["window"], nq, st)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, iters):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    # ---- warm-up through the eager API (also sizes the scratch workspace)
    for _ in range(args.warmup):
        step(q_raw, k_raw, v_raw, out)
    cache.check(stream)

    # ---- device-resident step: the 2*L launches captured once, replayed
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step(q_raw, k_raw, v_raw, out)  # warm the side stream
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        step(q_raw, k_raw, v_raw, out)
    dgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(dgraph):
        step(q_raw, k_raw, v_raw, out, decode_only=True)
    for _ in range(args.warmup):
        graph.replay()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ms = max_over_ranks(timed(graph.replay, args.steps))
    clk = clocks.stop()
    cache.check(stream)
    # dominant kernel: with the fused path every launch of the step is one
    # (prologue + append + decode) kernel, so the step graph times it; the
    # split path replays L back-to-back decode launches alone.
    if fused:
        dec_avg_ms = ms / L
    else:
        for _ in range(args.warmup):
            dgraph.replay()
        dec_avg_ms = timed(dgraph.replay, args.steps) / L
        cache.check(stream)

    # ---- end-to-end through the public API with host copies (eager calls)
    h_q = torch.randn((L, nq * d), generator=torch.Generator().manual_seed(5)).pin_memory()
    h_k = torch.randn((L, nkv * d), generator=torch.Generator().manual_seed(6)).pin_memory()
    h_v = torch.randn((L, nkv * d), generator=torch.Generator().manual_seed(7)).pin_memory()
    h_o = torch.empty((L, nq * d)).pin_memory()
    d_q, d_k, d_v = torch.empty_like(q_raw), torch.empty_like(k_raw), torch.empty_like(v_raw)
    d_o = torch.empty_like(out)

    def e2e_step():
        d_q.copy_(h_q, non_blocking=True)
        d_k.copy_(h_k, non_blocking=True)
        d_v.copy_(h_v, non_blocking=True)
        step(d_q, d_k, d_v, d_o)
        h_o.copy_(d_o, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    e2e_ms = max_over_ranks(timed(e2e_step, args.steps))
    cache.check(stream)
    del graph, dgraph

    kv_bytes_layer = 2 * nkv * n * d * 4
    total_bytes = kv_bytes_layer * L * world
    value = total_bytes / (ms * 1e-3) / 1e9
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e9
    peak, peak_kind = hbm_peak()
    achieved = kv_bytes_layer / (dec_avg_ms * 1e-3) / 1e9
    traffic = read_traffic("gqa_decode_kernel", args.config)

    result = None
    if rank == 0:
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) K/V and q/k/v generated on device)",
            "config": {"workload": f"{args.config}: {cfg['desc']}", "layers": L, "nq": nq,
                       "nkv": nkv, "head_dim": d, "n": n, "rope_theta": cfg["theta"],
                       "parallelism": f"replicas x{world} (one sequence per GPU)",
                       "l2": "inputs larger than L2 (4.3 GB KV per GPU)"},
            "tok_per_s": round(world * 1000.0 / ms, 2),
            "pct_hbm_peak": round(100.0 * value / world / peak, 2),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": int(4 * L * (nq + 2 * nkv) * d),
                    "d2h_bytes_per_step": int(4 * L * nq * d),
                    "ms_per_step": round(e2e_ms, 4),
                    "path": (("molot_attn_step" if fused else
                              "molot_attn_append_rope + molot_attn_decode")
                             + " per layer, pinned H2D/D2H")},
            "gpu_launches": (1 if fused else 2) * L * args.steps,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "kernel": "gqa_decode_kernel<128,4,1>",
                         "timed": ("fused step launches (prologue + append + decode)" if fused
                                   else "decode launches alone"),
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "bytes_per_launch": kv_bytes_layer,
                         "avg_launch_ms": round(dec_avg_ms, 5)},
            "clocks": clk,
        }
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline_sample(cfg)
        print(json.dumps(result), flush=True)
    cache.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["molot", "reference"], default="molot")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--path", choices=["fused", "split"], default="fused",
                    help="fused: molot_attn_step (one launch per layer); split: "
                         "molot_attn_append_rope + molot_attn_decode")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (small cases for profiler captures)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.layers > 0:
        cfg["layers"] = args.layers
    if args.impl == "reference":
        return run_reference(args, cfg)
    return run_molot(args, cfg)


if __name__ == "__main__":
    sys.exit(main())
