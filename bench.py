"""Benchmark: GQA decode attention, KV GB/s and tokens/s (BASELINE metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl molot|reference]
                    [--config cfg2|cfg1|cfg3|cfg4|cfg5] [--path fused|split]

Default workload ("cfg2"): one decode step of a 32-layer
Llama-shaped model at 16k context -- Hq=32, Hkv=8, head_dim=128, 16384 cached
slots + the new token (n=16385), RoPE theta=5e5.  Per layer the step runs
the library's public call molot_attn_step: QK-norm/RoPE of the raw q/k, the
append of the new row and split-KV decode over the HBM-resident cache, in
one launch (--path split: molot_attn_append_rope + molot_attn_decode, two
launches).  K/V and q/k/v are seeded N(0,1) synthetic data generated on the
device.  The 4.3 GB of KV is far larger than L2 (126 MB), so no flush is
needed.  With N>1 every rank runs its own replica (one sequence per GPU,
weak scaling, no collective on the data path).

Other BASELINE configs (parity cases, also benchable):
  cfg1  the same at ctx 4096 (bench.cc shape);
  cfg3  Gemma-3-4B shape: 34 layers, Hq=8, Hkv=4, d=256, QK-norm + V-norm,
        every 6th layer global (theta 1e6, full 32769 slots), the rest
        sliding-window (1024 slots, theta 1e4), scale 1, one launch per layer;
  cfg4  continuous batching, Llama-3-8B shape, 64 sequences with lengths
        U[512, 32768] (seeded), 16-slot pages with a shuffled block table;
        sequences split over the ranks by LPT on their lengths (strong
        scaling, no collective), batched append + paged decode per layer;
  cfg5  Llama-3-70B shape (80 layers, Hq=64, Hkv=8), 32 sequences with
        lengths U[8192, 131072]; kv heads split over the ranks, each
        layer's outputs all-gathered over NCCL on a second stream.
  cfg4/cfg5 hold more KV than one GPU: --resident-gb of distinct layer pools
  stay resident and the step cycles through them (each pool is far larger
  than L2, so every layer still streams from HBM).

value  : unique KV bytes read per step (2*Hkv*slots*d*4 per layer and
         sequence, all ranks) / max-over-ranks device time of the K timed
         steps, inputs resident.
e2e    : the same metric through the same public API with the step's inputs
         (raw q/k/v of every layer) copied host->device from pinned memory
         and the attention outputs copied back, inside the timed region.

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
    "cfg1": dict(kind="single", layers=32, nq=32, nkv=8, d=128, ctx=4096, theta=1e4, window=0,
                 desc="single-sequence GQA decode, ctx 4096 (bench.cc shape)"),
    "cfg2": dict(kind="single", layers=32, nq=32, nkv=8, d=128, ctx=16384, theta=5e5, window=0,
                 desc="single-sequence GQA decode, ctx 16384, 32-layer sweep"),
    "cfg3": dict(kind="gemma", layers=34, nq=8, nkv=4, d=256, ctx=32768, swa_window=1024,
                 swa_theta=1e4, global_theta=1e6, global_every=6, scale=1.0,
                 desc="Gemma-3-4B shape, 5:1 SWA(1024)/global at ctx 32768, QK-norm + V-norm"),
    "cfg4": dict(kind="paged_seq", layers=32, nq=32, nkv=8, d=128, batch=64, len_lo=512,
                 len_hi=32768, page=16, theta=5e5, seed=4,
                 desc="paged continuous batching, Llama-3-8B shape, B=64, n~U[512,32768]"),
    "prefill": dict(kind="prefill", layers=32, nq=32, nkv=8, d=128, prompt=4096, theta=5e5,
                    window=0, desc="prefill of a 4096-token prompt, Llama-3-8B attention shape "
                                   "(not a BASELINE config: the next row after decode)"),
    "gemv": dict(kind="gemv", layers=32, hidden=4096, nq=32, nkv=8, d=128,
                 desc="Q4 projections around attention per decode token, Llama-3-8B: fused "
                      "QKV (6144x4096) and O (4096x4096) GEMVs per layer, 32 layers (not a "
                      "BASELINE config: item 3 after decode)"),
    "cfg5": dict(kind="paged_head", layers=80, nq=64, nkv=8, d=128, batch=32, len_lo=8192,
                 len_hi=131072, page=16, theta=5e5, seed=5,
                 desc="Llama-3-70B shape, B=32, n~U[8192,131072], kv-head sharded"),
}
for _name, _cfg in CONFIGS.items():
    _cfg["name"] = _name
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


# ------------------------------------------------------------------ workloads

def paged_lengths(cfg):
    """Cached context length of each sequence (seeded U[len_lo, len_hi])."""
    rng = np.random.default_rng(cfg["seed"])
    return [int(x) for x in rng.integers(cfg["len_lo"], cfg["len_hi"] + 1, size=cfg["batch"])]


def gemma_layers(cfg):
    """(window, rope theta) per layer: every global_every-th layer is global."""
    k = cfg["global_every"]
    return [(0, cfg["global_theta"]) if l % k == k - 1 else (cfg["swa_window"], cfg["swa_theta"])
            for l in range(cfg["layers"])]


def attended(n, window):
    """Slots a decode at position n-1 attends (attn.h:137)."""
    return min(n, window) if window > 0 else n


def prefill_flops(cfg):
    """Attention FLOPs of one prefill layer: 2 (QK) + 2 (PV) multiply-adds
    per attended (query, slot, head, dim)."""
    M, w = cfg["prompt"], cfg["window"]
    pairs = sum(min(m + 1, w) if w > 0 else m + 1 for m in range(M))
    return 4 * cfg["nq"] * cfg["d"] * pairs


PREFILL_METRIC = "prefill attention TFLOP/s (FP32 results), 4096-token prompt"


GEMV_METRIC = "Q4 projection GEMV GB/s (weights streamed per decode token)"


def gemv_shapes(cfg):
    """(rows, cols) of the per-layer GEMVs: fused QKV, then O."""
    h, d = cfg["hidden"], cfg["d"]
    return [((cfg["nq"] + 2 * cfg["nkv"]) * d, h), (h, cfg["nq"] * d)]


def gemv_bytes(rows, cols):
    """HBM bytes of one Q4 GEMV: nibbles, FP32 scales, int8 zeros, x, y."""
    return rows * cols // 2 + rows * (cols // 32) * 5 + cols * 4 + rows * 4


def step_work(cfg):
    """(metric, unit, amount per step, divisor to the unit's base) of a config."""
    if cfg["kind"] == "gemv":
        return (GEMV_METRIC, "GB/s",
                cfg["layers"] * sum(gemv_bytes(r, c) for r, c in gemv_shapes(cfg)), 1e9)
    if cfg["kind"] == "prefill":
        return PREFILL_METRIC, "TFLOP/s", cfg["layers"] * prefill_flops(cfg), 1e12
    return METRIC, "GB/s", step_bytes(cfg), 1e9


def kv_row_bytes(kv, d):
    """Bytes of one cached row of one kv head in a storage type."""
    if kv == "q8":
        return (d + d // 8 + 15) & ~15
    return d * (2 if kv == "bf16" else 4)


def step_bytes(cfg, kv="f32"):
    """Unique KV bytes one decode step reads (all layers, all sequences)."""
    kind, nkv, d = cfg["kind"], cfg["nkv"], cfg["d"]
    rb = kv_row_bytes(kv, d)
    if kind == "single":
        return cfg["layers"] * 2 * nkv * (cfg["ctx"] + 1) * rb
    if kind == "gemma":
        n = cfg["ctx"] + 1
        return sum(2 * nkv * attended(n, w) * rb for w, _ in gemma_layers(cfg))
    return cfg["layers"] * sum(2 * nkv * (x + 1) * rb for x in paged_lengths(cfg))


class RefWorkload:
    """Representative calls of the reference's attn_decode_gqa_cache for a
    config (the reference is single-sequence and unpaged: a paged config is
    per-sequence calls on contiguous [n][nkv*d] caches, page gather excluded).
    call(i) runs the i-th call; step_seconds() extrapolates one step of the
    GPU arm's workload from the per-call means."""

    def __init__(self, cfg, impl, cores):
        import oracle
        self.oracle, self.impl, self.cores, self.cfg = oracle, impl, cores, cfg
        kind, nq, nkv, d = cfg["kind"], cfg["nq"], cfg["nkv"], cfg["d"]
        if kind == "gemv":
            self.items = [(0, 0, 0)]
            self.q4 = []
            rng0 = np.random.default_rng(3)
            for r, c in gemv_shapes(cfg):
                self.q4.append((rng0.uniform(1e-3, 1e-2, (r, c // 32)).astype(np.float32),
                                rng0.integers(0, 16, (r, c // 32), dtype=np.int8),
                                rng0.integers(0, 256, (r, c // 2), dtype=np.uint8),
                                np.zeros((r, c // 32), np.int16),
                                rng0.standard_normal(c).astype(np.float32)))
            self.t = [0.0]
            self.c = [0]
            self.bytes = 0
            self.seconds = 0.0
            return
        if kind == "prefill":
            self.items = [(cfg["prompt"], 0, cfg["window"])]
        elif kind == "single":
            n = cfg["ctx"] + 1
            self.items = [(n, n - 1, 0)]
        elif kind == "gemma":
            n = cfg["ctx"] + 1
            self.items = [(n, n - 1, 0), (n, n - 1, cfg["swa_window"])]
        else:
            lens = paged_lengths(cfg)
            order = np.random.default_rng(cfg["seed"] + 100).permutation(len(lens))
            self.items = [(lens[i] + 1, lens[i], 0) for i in order]
        nmax = max(x[0] for x in self.items)
        rng = np.random.default_rng(7)
        nbuf = 2 if kind in ("single", "gemma") else 1  # distinct buffers >> CPU caches
        self.Q = rng.standard_normal((nq, d), dtype=np.float32)
        if kind == "prefill":
            self.Qm = rng.standard_normal((cfg["prompt"], nq, d), dtype=np.float32)
        self.K = [rng.standard_normal((nmax, nkv * d), dtype=np.float32) for _ in range(nbuf)]
        self.V = [rng.standard_normal((nmax, nkv * d), dtype=np.float32) for _ in range(nbuf)]
        self.t = [0.0] * len(self.items)
        self.c = [0] * len(self.items)
        self.bytes = 0
        self.seconds = 0.0

    def call(self, i, record=True, item=None):
        cfg = self.cfg
        nq, nkv, d = cfg["nq"], cfg["nkv"], cfg["d"]
        j = i % len(self.items) if item is None else item
        n, pos, w = self.items[j]
        scale = 1.0 / math.sqrt(d)
        if cfg["kind"] == "gemv":  # one layer's GEMVs per call
            t0 = time.perf_counter()
            for sc, z, data, ws, x in self.q4:
                self.oracle.gemv_q4((sc, z, data, ws), x,
                                    impl="ref" if self.impl == "reference" else "port",
                                    nthreads=self.cores)
            dt = time.perf_counter() - t0
            if record:
                self.t[0] += dt
                self.c[0] += 1
                self.bytes += sum(gemv_bytes(r, c) for r, c in gemv_shapes(cfg))
                self.seconds += dt
            return dt
        buf = i % len(self.K)
        K, V = self.K[buf][:n], self.V[buf][:n]
        if cfg["kind"] == "prefill":  # n = prompt length, pos0 = 0
            Qm = self.Qm
            t0 = time.perf_counter()
            self.oracle.attn_prefill_gqa(Qm, K, V, nq, nkv, n, n, d, scale, 0, w,
                                         impl="ref" if self.impl == "reference" else "port",
                                         nthreads=self.cores)
            dt = time.perf_counter() - t0
            if record:
                self.t[j] += dt
                self.c[j] += 1
                self.bytes += prefill_flops(cfg)  # FLOPs for this kind
                self.seconds += dt
            return dt
        t0 = time.perf_counter()
        if self.impl == "reference":
            self.oracle.attn_decode_gqa_cache(self.Q, K, V, nq, nkv, n, d, scale, pos, w,
                                              impl="ref", nthreads=self.cores)
        else:
            self.oracle.attn_decode_gqa_cache(self.Q, K, V, nq, nkv, n, d, scale, pos, w)
        dt = time.perf_counter() - t0
        if record:
            self.t[j] += dt
            self.c[j] += 1
            self.bytes += 2 * nkv * attended(n, w) * d * 4
            self.seconds += dt
        return dt

    def step_seconds(self):
        cfg = self.cfg
        mean = [t / c if c else 0.0 for t, c in zip(self.t, self.c)]
        if cfg["kind"] in ("single", "prefill", "gemv"):
            return cfg["layers"] * mean[0]
        if cfg["kind"] == "gemma":
            ng = sum(1 for w, _ in gemma_layers(cfg) if w == 0)
            return ng * mean[0] + (cfg["layers"] - ng) * mean[1]
        return step_bytes(cfg) / (self.bytes / self.seconds)

    def describe(self, what):
        fn = {"prefill": "attn_prefill_gqa", "gemv": "gemv_q4"}.get(self.cfg["kind"],
                                                                    "attn_decode_gqa_cache")
        return (f"{sum(self.c)} calls of {fn} ({what}), "
                f"{self.seconds:.1f}s; per-step time extrapolated from per-call means")


def ref_kind_and_cores():
    import oracle
    if oracle.ref() is not None:
        return "reference", os.cpu_count() or 1
    return "port", 1


# ------------------------------------------------------------------ reference arm

def run_reference(args, cfg):
    """The reference's own attn_decode_gqa_cache on the host cores.  For the
    single-sequence configs (cfg1 / cfg2) and cfg3 every step is timed in
    full: one call per layer, each on its own layer-sized cache (two cycled
    buffers, far larger than the CPU caches), exactly --steps steps after
    --warmup untimed ones.  The reference times attention only: its per-token
    norm / RoPE / append (about 1 % of its step) are outside the timed calls,
    while the GPU arm's step includes them.  The paged, prefill and GEMV
    configs would take minutes per step on the host: there the line times a
    bounded sample of calls and extrapolates the step, and says so."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    kind, cores = ref_kind_and_cores()
    wl = RefWorkload(cfg, kind, cores)
    metric, unit, amount, div = step_work(cfg)
    batch = cfg.get("batch", cfg.get("prompt", 1) if cfg["kind"] == "prefill" else 1)
    full = cfg["kind"] in ("single", "gemma")
    if full:
        items = ([0] * cfg["layers"] if cfg["kind"] == "single" else
                 [0 if w == 0 else 1 for w, _ in gemma_layers(cfg)])
        i = 0
        for _ in range(args.warmup):
            for j in items:
                wl.call(i, record=False, item=j)
                i += 1
        t0 = time.perf_counter()
        for _ in range(args.steps):
            for j in items:
                wl.call(i, item=j)
                i += 1
        sec = (time.perf_counter() - t0) / args.steps
        config = (single_config(args, cfg, world) if cfg["kind"] == "single"
                  else gemma_config(args, cfg, world))
        sample = (f"{args.steps} full steps timed ({len(items)} attn_decode_gqa_cache calls "
                  f"each, one per layer) after {args.warmup} untimed; attention only (the "
                  "reference's norm / RoPE / append are not in the timed calls)")
        timed_s = sec * args.steps
    else:
        per_step = 2
        for i in range(args.warmup):
            wl.call(i, record=False)
        for i in range(args.steps * per_step):
            wl.call(i)
        sec = wl.step_seconds()
        what = {"prefill": f"one layer's attn_prefill_gqa over a {cfg.get('prompt')}-token "
                           "prompt",
                "gemv": "one layer's fused-QKV and O gemv_q4",
                }.get(cfg["kind"], "one sequence per call, lengths from the config's seeded "
                                   "draw")
        config = {"workload": f"{args.config}: {cfg['desc']}", "layers": cfg["layers"],
                  "nq": cfg["nq"], "nkv": cfg["nkv"], "head_dim": cfg["d"],
                  "kv_dtype": args.kv}
        sample = wl.describe(what) + (f"; {args.steps * per_step} calls timed in all, not "
                                      f"{args.steps} full steps")
        timed_s = wl.seconds
    value = amount / sec / div
    line = {
        "impl": "reference", "metric": metric, "value": round(value, 3), "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True,
        "scaling": "weak" if cfg["kind"] in ("single", "gemma", "prefill", "gemv") else "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": config,
        "tok_per_s": round(batch / sec, 3),
        "timed_region_s": round(timed_s, 3),
        "steps_timed_in_full": bool(full),
        "cpu_baseline": {"value": round(value, 3), "unit": unit, "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def cpu_baseline_sample(cfg):
    """A bounded reference sample (~10 s) for the GPU arm's cpu_baseline key."""
    kind, cores = ref_kind_and_cores()
    wl = RefWorkload(cfg, kind, cores)
    budget = 10.0 if kind == "reference" else 6.0
    wl.call(0, record=False)
    i = 0
    while wl.seconds < budget and i < 400:
        wl.call(i)
        i += 1
    sec = wl.step_seconds()
    _, unit, amount, div = step_work(cfg)
    return {"value": round(amount / sec / div, 3), "unit": unit, "cores": cores,
            "kind": kind, "sample": wl.describe(f"{cfg['kind']} workload")}


# ------------------------------------------------------------------ molot arm

def single_config(args, cfg, world):
    """`config` of a single-sequence line; the reference arm emits the same."""
    n = cfg["ctx"] + 1
    per_gpu = step_bytes(cfg, args.kv)
    return {"workload": f"{args.config}: {cfg['desc']}", "layers": cfg["layers"],
            "nq": cfg["nq"], "nkv": cfg["nkv"], "head_dim": cfg["d"], "n": n,
            "rope_theta": cfg["theta"], "kv_dtype": args.kv,
            "parallelism": f"replicas x{world} (one sequence per GPU)",
            "l2": f"inputs larger than L2 ({per_gpu / 1e9:.1f} GB KV per GPU)"}


def timed_repeats(rt, fn, steps, repeats):
    """ms per step over `repeats` windows of exactly `steps` calls of fn, each
    window timed with CUDA events (barrier + synchronize on both sides) and
    taken as the max over ranks; returns (median, windows)."""
    vals = [rt.max(rt.timed(fn, steps)) for _ in range(max(1, repeats))]
    return statistics.median(vals), vals


def capture(torch, fn):
    """fn() captured into a CUDA graph after one run on a side stream."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


class SingleSeq:
    """KV cache, per-layer inputs and the step of a single-sequence config
    (cfg1 / cfg2): per layer molot_attn_step (fused) or
    molot_attn_append_rope + molot_attn_decode (split)."""

    def __init__(self, rt, args, cfg):
        import molot_b200 as mb
        torch = rt.torch
        self.rt, self.cfg, self.torch = rt, cfg, torch
        L, nq, nkv, d = cfg["layers"], cfg["nq"], cfg["nkv"], cfg["d"]
        self.L, self.nq, self.nkv, self.d = L, nq, nkv, d
        ctx = self.ctx = cfg["ctx"]
        self.n = ctx + 1
        self.scale = 1.0 / math.sqrt(d)
        self.fused = args.path == "fused"
        dev = rt.dev
        self.cache = mb.KVCache(L, nkv, d, self.n, dtype=args.kv)
        gen = torch.Generator(device=dev)
        gen.manual_seed(1234 + rt.rank)
        for layer in range(L):
            if args.kv == "q8":  # rows enter through the library's quantizing write
                rows_k = torch.randn((ctx, nkv * d), device=dev, generator=gen)
                rows_v = torch.randn((ctx, nkv * d), device=dev, generator=gen)
                self.cache.write(layer, 0, rows_k, rows_v)
                del rows_k, rows_v
                continue
            kt, vt = self.cache.layer_tensors(layer)  # head-major [nkv][cap][hd]
            kt[:, :ctx].normal_(generator=gen)
            vt[:, :ctx].normal_(generator=gen)
        self.q_raw = torch.randn((L, nq * d), device=dev, generator=gen)
        self.k_raw = torch.randn((L, nkv * d), device=dev, generator=gen)
        self.v_raw = torch.randn((L, nkv * d), device=dev, generator=gen)
        self.q_norm = (1 + 0.1 * torch.randn(d, device=dev, generator=gen)).contiguous()
        self.k_norm = (1 + 0.1 * torch.randn(d, device=dev, generator=gen)).contiguous()
        self.freq = rope_freq(torch, cfg["theta"], d, dev)
        self.q_rot = torch.randn((L, nq * d), device=dev, generator=gen)
        self.out = torch.empty((L, nq * d), device=dev)
        torch.cuda.synchronize()

    def step(self, qr=None, kr=None, vr=None, o=None, decode_only=False):
        qr = self.q_raw if qr is None else qr
        kr = self.k_raw if kr is None else kr
        vr = self.v_raw if vr is None else vr
        o = self.out if o is None else o
        st = self.torch.cuda.current_stream()
        c, cfg = self.cache, self.cfg
        for layer in range(self.L):
            if decode_only:
                c.decode(layer, self.q_rot[layer], o[layer], self.scale, self.ctx, cfg["window"],
                         self.nq, st)
                continue
            c.set_length(layer, self.ctx)
            if self.fused:
                c.step(layer, qr[layer], kr[layer], vr[layer], o[layer], self.scale, self.ctx,
                       cfg["window"], self.q_norm, self.k_norm, False, 1e-6, self.freq, self.nq,
                       st)
            else:
                c.append_rope(layer, qr[layer], kr[layer], vr[layer], self.q_rot[layer],
                              self.q_norm, self.k_norm, False, 1e-6, self.freq, self.ctx,
                              self.nq, st)
                c.decode(layer, self.q_rot[layer], o[layer], self.scale, self.ctx,
                         cfg["window"], self.nq, st)

    def close(self):
        self.cache.close()


def single_sub(rt, args, name):
    """A BASELINE single-sequence config measured beside the headline one
    (N = 1 line): device time per token of the fused step (CUDA graph)."""
    cfg = dict(CONFIGS[name])
    s = SingleSeq(rt, args, cfg)
    for _ in range(args.warmup):
        s.step()
    s.cache.check()
    g = capture(rt.torch, s.step)
    for _ in range(args.warmup):
        g.replay()
    ms, reps = timed_repeats(rt, g.replay, args.steps, args.repeats)
    s.cache.check()
    del g
    s.close()
    peak, _ = hbm_peak()
    layer_bytes = 2 * cfg["nkv"] * (cfg["ctx"] + 1) * kv_row_bytes(args.kv, cfg["d"])
    achieved = layer_bytes / (ms / cfg["layers"] * 1e-3) / 1e9
    return {"workload": f"{name}: {cfg['desc']}", "ms_per_token": round(ms, 4),
            "tok_per_s": round(1000.0 / ms, 1), "value": round(achieved, 1), "unit": "GB/s",
            "frac": round(achieved / peak, 4), "avg_launch_ms": round(ms / cfg["layers"], 5),
            "bytes_per_launch": layer_bytes, "repeats_ms": [round(x, 4) for x in reps],
            "path": "molot_attn_step per layer (CUDA graph)"}


def run_single(args, cfg):
    rt = Rt()
    torch = rt.torch
    world, rank = rt.world, rt.rank
    L, nq, nkv, d = cfg["layers"], cfg["nq"], cfg["nkv"], cfg["d"]
    n = cfg["ctx"] + 1
    s = SingleSeq(rt, args, cfg)
    fused = s.fused

    # ---- warm-up through the eager API (also sizes the scratch workspace)
    for _ in range(args.warmup):
        s.step()
    s.cache.check()

    # ---- device-resident step: the step's launches captured once, replayed
    graph = capture(torch, s.step)
    dgraph = capture(torch, lambda: s.step(decode_only=True))
    for _ in range(args.warmup):
        graph.replay()
    clocks = ClockSampler(rt.local)
    clocks.start()
    time.sleep(0.3)
    ms, reps = timed_repeats(rt, graph.replay, args.steps, args.repeats)
    clk = clocks.stop()
    s.cache.check()
    # dominant kernel: with the fused path every launch of the step is one
    # (prologue + append + decode) kernel, so the step graph times it; the
    # split path replays L back-to-back decode launches alone.
    if fused:
        dec_avg_ms = ms / L
    else:
        for _ in range(args.warmup):
            dgraph.replay()
        dec_avg_ms = rt.timed(dgraph.replay, args.steps) / L
        s.cache.check()

    # ---- end-to-end through the public API with host copies (eager calls)
    h_q = pinned_like(torch, s.q_raw, 5)
    h_k = pinned_like(torch, s.k_raw, 6)
    h_v = pinned_like(torch, s.v_raw, 7)
    h_o = torch.empty(s.out.shape).pin_memory()
    d_q, d_k, d_v = (torch.empty_like(t) for t in (s.q_raw, s.k_raw, s.v_raw))
    d_o = torch.empty_like(s.out)

    def e2e_step():
        d_q.copy_(h_q, non_blocking=True)
        d_k.copy_(h_k, non_blocking=True)
        d_v.copy_(h_v, non_blocking=True)
        s.step(d_q, d_k, d_v, d_o)
        h_o.copy_(d_o, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    e2e_ms = rt.max(rt.timed(e2e_step, args.steps))
    s.cache.check()
    del graph, dgraph
    s.close()
    torch.cuda.empty_cache()

    # ---- the other BASELINE configs, measured in the same run
    extras = {}
    if args.extras and args.config == "cfg2" and args.kv == "f32" and fused:
        if world == 1:
            extras["configs"] = {"cfg1": single_sub(rt, args, "cfg1"),
                                 "cfg3": gemma_sub(rt, args)}
            torch.cuda.empty_cache()
        extras["batched"] = {}
        for name in ("cfg4", "cfg5"):
            extras["batched"][name] = paged_measure(rt, args, dict(CONFIGS[name]), brief=True)
            torch.cuda.empty_cache()

    row_bytes = kv_row_bytes(args.kv, d)
    kv_bytes_layer = 2 * nkv * n * row_bytes
    total_bytes = kv_bytes_layer * L * world
    value = total_bytes / (ms * 1e-3) / 1e9
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e9
    peak, peak_kind = hbm_peak()
    achieved = kv_bytes_layer / (dec_avg_ms * 1e-3) / 1e9
    traffic = read_traffic("gqa_decode_kernel",
                           args.config + ("-" + args.kv if args.kv != "f32" else ""))
    if rank == 0:
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) K/V and q/k/v generated on device)",
            "config": single_config(args, cfg, world),
            "repeats": {"windows": len(reps), "steps_each": args.steps,
                        "ms_per_step": [round(x, 4) for x in reps],
                        "spread_pct": round(100.0 * (max(reps) - min(reps)) / ms, 2),
                        "reported": "median window (each window: max over ranks)"},
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
                         "traffic": traffic,
                         "kernel": "gqa_decode_kernel<128,4,1%s>" % (
                             "," + args.kv if args.kv != "f32" else ""),
                         "timed": ("fused step launches (prologue + append + decode)" if fused
                                   else "decode launches alone"),
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "bytes_per_launch": kv_bytes_layer,
                         "avg_launch_ms": round(dec_avg_ms, 5)},
            "clocks": clk,
        }
        result.update(extras)
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline_sample(cfg)
        print(json.dumps(result), flush=True)
    rt.close()
    return 0


class Rt:
    """Process group, device and device-timing helpers of the molot arm."""

    def __init__(self):
        import datetime
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.world, self.rank, self.local = dist_env()
        torch.cuda.set_device(self.local)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        self.dev = torch.device("cuda", self.local)

    def barrier(self):
        self.torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def reduce(self, x, op):
        if self.world == 1:
            return x
        t = self.torch.tensor([float(x)], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=op)
        return float(t.item())

    def max(self, x):
        return self.reduce(x, self.dist.ReduceOp.MAX)

    def sum(self, x):
        return self.reduce(x, self.dist.ReduceOp.SUM)

    def timed(self, fn, iters):
        """Mean ms per call of fn over `iters` calls, CUDA events on the
        current stream, bracketed by barrier + synchronize."""
        torch = self.torch
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        self.barrier()
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def rope_freq(torch, theta, d, dev):
    return torch.tensor([1.0 / theta ** (2.0 * i / d) for i in range(d // 2)],
                        dtype=torch.float32, device=dev)


def pinned_like(torch, t, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(t.shape, generator=g).pin_memory()


def emit(rt, args, cfg, ms, e2e_ms, clk, h2d, d2h, launches, roof, config, scaling, extra=None):
    """The bench JSON line (rank 0)."""
    # weak scaling = replicas (every rank runs the whole step); strong = the
    # step's sequences or kv heads are split over the ranks
    total = step_bytes(cfg, args.kv) * (rt.world if scaling == "weak" else 1)
    peak, peak_kind = hbm_peak()
    value = total / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": rt.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) K/V and q/k/v generated on device)",
        "config": dict(config, kv_dtype=args.kv),
        "tok_per_s": round(cfg.get("batch", 1) * (rt.world if scaling == "weak" else 1)
                           * 1000.0 / ms, 2),
        "pct_hbm_peak": round(100.0 * value / rt.world / peak, 2),
        "e2e": {"value": round(total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": int(launches),
        "roofline": dict(roof, peak=peak, unit="GB/s", frac=round(roof["achieved"] / peak, 4),
                         peak_source=f"{peak_kind} hbm_gbs"),
        "clocks": clk,
    }
    if extra:
        line.update(extra)
    if rt.world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(cfg)
    print(json.dumps(line), flush=True)


def gemma_config(args, cfg, world):
    """`config` of a cfg3 line; the reference arm emits the same."""
    layers = gemma_layers(cfg)
    return {"workload": f"{args.config}: {cfg['desc']}", "layers": cfg["layers"],
            "nq": cfg["nq"], "nkv": cfg["nkv"], "head_dim": cfg["d"], "n": cfg["ctx"] + 1,
            "global_layers": [l for l, (w, _) in enumerate(layers) if w == 0],
            "swa_window": cfg["swa_window"], "scale": cfg["scale"], "kv_dtype": args.kv,
            "parallelism": f"replicas x{world} (one sequence per GPU)",
            "l2": "inputs larger than L2 (1.585 GB KV read per step)"}


class GemmaSeq:
    """cfg3 (Gemma-3-4B shape): KV cache, inputs and the step, one
    molot_attn_step launch per layer; SWA layers attend 1024 slots."""

    def __init__(self, rt, args, cfg):
        import molot_b200 as mb
        torch = rt.torch
        self.torch, self.cfg = torch, cfg
        L, nq, nkv, d = cfg["layers"], cfg["nq"], cfg["nkv"], cfg["d"]
        self.L, self.nq, self.nkv, self.d = L, nq, nkv, d
        ctx = self.ctx = cfg["ctx"]
        self.n = ctx + 1
        self.layers = gemma_layers(cfg)
        dev = rt.dev
        self.cache = mb.KVCache(L, nkv, d, self.n, dtype=args.kv)
        gen = torch.Generator(device=dev)
        gen.manual_seed(1234 + rt.rank)
        for l, (w, _) in enumerate(self.layers):
            lo = max(0, ctx - w + 1) if w else 0
            if args.kv == "q8":  # rows enter through the library's quantizing write
                rows = torch.randn((2, ctx - lo, nkv * d), device=dev, generator=gen)
                self.cache.write(l, lo, rows[0], rows[1])
                del rows
                continue
            kt, vt = self.cache.layer_tensors(l)  # head-major [nkv][cap][hd]
            kt[:, lo:ctx].normal_(generator=gen)
            vt[:, lo:ctx].normal_(generator=gen)
        self.q_raw = torch.randn((L, nq * d), device=dev, generator=gen)
        self.k_raw = torch.randn((L, nkv * d), device=dev, generator=gen)
        self.v_raw = torch.randn((L, nkv * d), device=dev, generator=gen)
        self.q_norm = (1 + 0.1 * torch.randn(d, device=dev, generator=gen)).contiguous()
        self.k_norm = (1 + 0.1 * torch.randn(d, device=dev, generator=gen)).contiguous()
        self.freq = {th: rope_freq(torch, th, d, dev) for _, th in self.layers}
        self.out = torch.empty((L, nq * d), device=dev)
        self.glob = [l for l, (w, _) in enumerate(self.layers) if w == 0]
        self.swa = [l for l, (w, _) in enumerate(self.layers) if w != 0]
        torch.cuda.synchronize()

    def step(self, qr=None, kr=None, vr=None, o=None, only=None):
        qr = self.q_raw if qr is None else qr
        kr = self.k_raw if kr is None else kr
        vr = self.v_raw if vr is None else vr
        o = self.out if o is None else o
        st = self.torch.cuda.current_stream()
        for l in (range(self.L) if only is None else only):
            w, th = self.layers[l]
            self.cache.set_length(l, self.ctx)
            self.cache.step(l, qr[l], kr[l], vr[l], o[l], self.cfg["scale"], self.ctx, w,
                            self.q_norm, self.k_norm, True, 1e-6, self.freq[th], self.nq, st)

    def close(self):
        self.cache.close()


def gemma_sub(rt, args):
    """cfg3 beside the headline config (N = 1 line): time per token of the
    34-launch step, and per launch of its global and SWA layers."""
    cfg = dict(CONFIGS["cfg3"])
    g3 = GemmaSeq(rt, args, cfg)
    for _ in range(args.warmup):
        g3.step()
    g3.cache.check()
    g = capture(rt.torch, g3.step)
    gg = capture(rt.torch, lambda: g3.step(only=g3.glob))
    gs = capture(rt.torch, lambda: g3.step(only=g3.swa))
    for _ in range(args.warmup):
        g.replay()
    ms, reps = timed_repeats(rt, g.replay, args.steps, args.repeats)
    for _ in range(args.warmup):
        gg.replay()
    glob_ms = rt.timed(gg.replay, args.steps) / len(g3.glob)
    for _ in range(args.warmup):
        gs.replay()
    swa_ms = rt.timed(gs.replay, args.steps) / len(g3.swa)
    g3.cache.check()
    del g, gg, gs
    g3.close()
    peak, _ = hbm_peak()
    total = step_bytes(cfg, args.kv)
    gbytes = 2 * cfg["nkv"] * (cfg["ctx"] + 1) * kv_row_bytes(args.kv, cfg["d"])
    sbytes = 2 * cfg["nkv"] * cfg["swa_window"] * kv_row_bytes(args.kv, cfg["d"])
    value = total / (ms * 1e-3) / 1e9
    return {"workload": f"cfg3: {cfg['desc']}", "ms_per_token": round(ms, 4),
            "tok_per_s": round(1000.0 / ms, 1), "value": round(value, 1), "unit": "GB/s",
            "frac": round(value / peak, 4), "bytes_per_token": total,
            "global_launch_ms": round(glob_ms, 5),
            "global_frac": round(gbytes / (glob_ms * 1e-3) / 1e9 / peak, 4),
            "swa_launch_ms": round(swa_ms, 5),
            "swa_frac": round(sbytes / (swa_ms * 1e-3) / 1e9 / peak, 4),
            "repeats_ms": [round(x, 4) for x in reps],
            "path": "molot_attn_step per layer (CUDA graph)"}


def run_gemma(args, cfg):
    """cfg3: one molot_attn_step launch per layer; SWA layers read 1024 slots."""
    rt = Rt()
    torch = rt.torch
    g3 = GemmaSeq(rt, args, cfg)
    L, nq, nkv, d, n = g3.L, g3.nq, g3.nkv, g3.d, g3.n
    for _ in range(args.warmup):
        g3.step()
    g3.cache.check()
    graph = capture(torch, g3.step)
    ggraph = capture(torch, lambda: g3.step(only=g3.glob))
    for _ in range(args.warmup):
        graph.replay()
    clocks = ClockSampler(rt.local)
    clocks.start()
    time.sleep(0.3)
    ms, reps = timed_repeats(rt, graph.replay, args.steps, args.repeats)
    clk = clocks.stop()
    for _ in range(args.warmup):
        ggraph.replay()
    glob_ms = rt.timed(ggraph.replay, args.steps) / len(g3.glob)
    g3.cache.check()

    h = [pinned_like(torch, t, 5 + i) for i, t in enumerate((g3.q_raw, g3.k_raw, g3.v_raw))]
    h_o = torch.empty((L, nq * d)).pin_memory()
    dq, dk, dv = (torch.empty_like(t) for t in (g3.q_raw, g3.k_raw, g3.v_raw))
    d_o = torch.empty_like(g3.out)

    def e2e_step():
        dq.copy_(h[0], non_blocking=True)
        dk.copy_(h[1], non_blocking=True)
        dv.copy_(h[2], non_blocking=True)
        g3.step(dq, dk, dv, d_o)
        h_o.copy_(d_o, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    e2e_ms = rt.max(rt.timed(e2e_step, args.steps))
    g3.cache.check()
    del graph, ggraph
    gbytes = 2 * nkv * n * kv_row_bytes(args.kv, d)
    if rt.rank == 0:
        emit(rt, args, cfg, ms, e2e_ms, clk,
             h2d=4 * L * (nq + 2 * nkv) * d, d2h=4 * L * nq * d, launches=L * args.steps,
             roof={"bound": "hbm", "achieved": round(gbytes / (glob_ms * 1e-3) / 1e9, 1),
                   "traffic": read_traffic("gqa_decode_kernel", args.config),
                   "kernel": "gqa_decode_kernel<256,2,1> (fused step, global layer)",
                   "timed": "the 5 global-layer launches alone",
                   "bytes_per_launch": gbytes, "avg_launch_ms": round(glob_ms, 5)},
             config=gemma_config(args, cfg, rt.world),
             scaling="weak",
             extra={"path": "molot_attn_step per layer (QK-norm, V-norm, RoPE, append, "
                            "decode in one launch)",
                    "repeats": {"windows": len(reps), "steps_each": args.steps,
                                "ms_per_step": [round(x, 4) for x in reps],
                                "reported": "median window (each window: max over ranks)"}})
    g3.close()
    rt.close()
    return 0


def run_prefill(args, cfg):
    """Prefill config: per layer molot_attn_append_rope_tokens (QK-norm/RoPE of
    the prompt's M tokens, rows appended) then molot_attn_prefill."""
    rt = Rt()
    torch = rt.torch
    import molot_b200 as mb

    L, nq, nkv, d, M = cfg["layers"], cfg["nq"], cfg["nkv"], cfg["d"], cfg["prompt"]
    window, scale = cfg["window"], 1.0 / math.sqrt(d)
    cache = mb.KVCache(L, nkv, d, M, dtype=args.kv)
    gen = torch.Generator(device=rt.dev)
    gen.manual_seed(1234 + rt.rank)
    q_raw = torch.randn((L, M, nq, d), device=rt.dev, generator=gen)
    k_raw = torch.randn((L, M, nkv, d), device=rt.dev, generator=gen)
    v_raw = torch.randn((L, M, nkv, d), device=rt.dev, generator=gen)
    q_rot = torch.empty_like(q_raw)
    out = torch.empty_like(q_raw)
    freq = rope_freq(torch, cfg["theta"], d, rt.dev)

    def step(qr, kr, vr, o, attn_only=False):
        st = torch.cuda.current_stream()
        for l in range(L):
            if not attn_only:
                cache.set_length(l, 0)
                cache.append_rope_tokens(l, qr[l], kr[l], vr[l], q_rot[l], None, None, False,
                                         1e-6, freq, 0, M, nq, st)
            cache.prefill(l, q_rot[l], o[l], scale, 0, window, M, nq, st)

    for _ in range(args.warmup):
        step(q_raw, k_raw, v_raw, out)
    cache.check()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step(q_raw, k_raw, v_raw, out)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph, agraph = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(q_raw, k_raw, v_raw, out)
    with torch.cuda.graph(agraph):
        step(q_raw, k_raw, v_raw, out, attn_only=True)
    graph.replay()
    clocks = ClockSampler(rt.local)
    clocks.start()
    time.sleep(0.3)
    ms = rt.max(rt.timed(graph.replay, args.steps))
    clk = clocks.stop()
    agraph.replay()
    attn_ms = rt.timed(agraph.replay, args.steps) / L
    cache.check()

    h = [pinned_like(torch, t, 5 + i) for i, t in enumerate((q_raw, k_raw, v_raw))]
    h_o = torch.empty(out.shape).pin_memory()
    dq, dk, dv = (torch.empty_like(t) for t in (q_raw, k_raw, v_raw))
    d_o = torch.empty_like(out)

    def e2e_step():
        dq.copy_(h[0], non_blocking=True)
        dk.copy_(h[1], non_blocking=True)
        dv.copy_(h[2], non_blocking=True)
        step(dq, dk, dv, d_o)
        h_o.copy_(d_o, non_blocking=True)

    e2e_step()
    e2e_ms = rt.max(rt.timed(e2e_step, max(1, args.steps // 4)))
    cache.check()
    del graph, agraph
    metric, unit, amount, div = step_work(cfg)
    flops_layer = prefill_flops(cfg)
    # FP32 caches at head_dim 64/128 run the tensor-core kernel: half the
    # useful FLOPs (S = QK^T) as three FP16 products at the measured bf16
    # GEMM rate R, half (O = PV) as three TF32 products at R / 2, so a
    # useful FLOP costs 0.5*3/R + 0.5*3/(R/2) = 4.5/R and the ceiling is
    # R / 4.5.  Other caches run the FP32 CUDA-core kernel: nominal FP32
    # peak (no measured figure).
    tc_path = args.kv == "f32" and cfg["d"] in (64, 128)
    sm_count = torch.cuda.get_device_properties(rt.dev).multi_processor_count
    if tc_path:
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
                bf16 = float(json.load(fh)["bf16_tflops"])
            peak_src = (f"measured bf16_tflops {bf16:.1f} / 4.5 (S: 3 FP16 products at the bf16 "
                        "rate; PV: 3 TF32 products at half of it; half the FLOPs each)")
        except Exception:
            bf16 = 1590.0
            peak_src = "fallback bf16 1590 TFLOP/s / 4.5 (3 FP16 S products, 3 TF32 PV products)"
        peak = bf16 / 4.5
    else:
        peak = sm_count * 128 * 2 * 1.965e9 / 1e12
        peak_src = "nominal FP32 CUDA-core peak (SMs x 128 lanes x 2 x 1965 MHz); no measured FP32 figure"
    if rt.rank == 0:
        value = amount * rt.world / (ms * 1e-3) / div
        line = {
            "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": rt.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) q/k/v generated on device)",
            "config": {"workload": f"prefill: {cfg['desc']}", "kv_dtype": args.kv,
                       "layers": L, "nq": nq, "nkv": nkv,
                       "head_dim": d, "prompt": M, "window": window,
                       "parallelism": f"replicas x{rt.world}",
                       "l2": "K/V of a layer (33.5 MB) stays in L2 across query blocks"},
            "tok_per_s": round(M * rt.world * 1000.0 / ms, 1),
            "e2e": {"value": round(amount * rt.world / (e2e_ms * 1e-3) / div, 2), "unit": unit,
                    "h2d_bytes_per_step": int(4 * (q_raw.numel() + k_raw.numel() + v_raw.numel())),
                    "d2h_bytes_per_step": int(4 * out.numel()), "ms_per_step": round(e2e_ms, 3)},
            "gpu_launches": 2 * L * args.steps,
            "roofline": {"bound": "tensor" if tc_path else "fp32",
                         "achieved": round(flops_layer / (attn_ms * 1e-3) / 1e12, 2),
                         "peak": round(peak, 1), "unit": "TFLOP/s",
                         "frac": round(flops_layer / (attn_ms * 1e-3) / 1e12 / peak, 4),
                         "traffic": None,
                         "kernel": ("gqa_prefill_tc_kernel<%d> (split FP16 S, split TF32 PV, tcgen05)" % cfg["d"]
                                    if tc_path else "gqa_prefill_kernel<%d>" % cfg["d"]),
                         "peak_source": peak_src,
                         "flops_per_launch": flops_layer, "avg_launch_ms": round(attn_ms, 4)},
            "clocks": clk,
            "path": "molot_attn_append_rope_tokens + molot_attn_prefill per layer",
        }
        if rt.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample(cfg)
        print(json.dumps(line), flush=True)
    cache.close()
    rt.close()
    return 0


def run_gemv(args, cfg):
    """Q4 projection GEMVs of one decode token (molot_gemv_q4_dev), distinct
    synthetic weights per layer (seeded random nibbles, scales, zeros)."""
    rt = Rt()
    torch = rt.torch
    import molot_b200 as mb

    L = cfg["layers"]
    gen = torch.Generator(device=rt.dev)
    gen.manual_seed(99 + rt.rank)
    mats = []
    for _ in range(L):
        layer = []
        for r, c in gemv_shapes(cfg):
            sc = (torch.rand((r, c // 32), device=rt.dev, generator=gen) * 9e-3 + 1e-3).contiguous()
            z = torch.randint(0, 16, (r, c // 32), device=rt.dev, generator=gen, dtype=torch.int8)
            data = torch.randint(0, 256, (r, c // 2), device=rt.dev, generator=gen,
                                 dtype=torch.uint8)
            layer.append((sc, z, data))
        mats.append(layer)
    (r0, c0), (r1, c1) = gemv_shapes(cfg)
    x = torch.randn((L, c0), device=rt.dev, generator=gen)
    qkv = torch.empty((L, r0), device=rt.dev)
    ao = torch.randn((L, c1), device=rt.dev, generator=gen)
    out = torch.empty((L, r1), device=rt.dev)

    def step(xx, a_in):
        st = torch.cuda.current_stream()
        for l in range(L):
            (s0, z0, d0), (s1, z1, d1) = mats[l]
            mb.gemv_q4_dev(s0, z0, d0, xx[l], qkv[l], st)
            mb.gemv_q4_dev(s1, z1, d1, a_in[l], out[l], st)

    for _ in range(args.warmup):
        step(x, ao)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step(x, ao)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(x, ao)
    graph.replay()
    clocks = ClockSampler(rt.local)
    clocks.start()
    time.sleep(0.3)
    ms = rt.max(rt.timed(graph.replay, args.steps))
    clk = clocks.stop()
    # the largest GEMV alone: L back-to-back QKV launches
    qgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(qgraph):
        for l in range(L):
            mb.gemv_q4_dev(mats[l][0][0], mats[l][0][1], mats[l][0][2], x[l], qkv[l])
    qgraph.replay()
    q_ms = rt.timed(qgraph.replay, args.steps) / L

    hx = pinned_like(torch, x, 5)
    ha = pinned_like(torch, ao, 6)
    ho = torch.empty(out.shape).pin_memory()
    hq = torch.empty(qkv.shape).pin_memory()
    dx, da = torch.empty_like(x), torch.empty_like(ao)

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        da.copy_(ha, non_blocking=True)
        step(dx, da)
        hq.copy_(qkv, non_blocking=True)
        ho.copy_(out, non_blocking=True)

    e2e_step()
    e2e_ms = rt.max(rt.timed(e2e_step, args.steps))
    del graph, qgraph
    metric, unit, amount, div = step_work(cfg)
    peak, peak_kind = hbm_peak()
    qbytes = gemv_bytes(r0, c0)
    if rt.rank == 0:
        value = amount * rt.world / (ms * 1e-3) / div
        line = {
            "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": rt.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/f32",
            "data": "synthetic (seeded random Q4 nibbles, scales, zeros; N(0,1) activations)",
            "config": {"workload": f"gemv: {cfg['desc']}", "layers": L,
                       "shapes": [list(s_) for s_ in gemv_shapes(cfg)],
                       "parallelism": f"replicas x{rt.world}",
                       "l2": f"{amount / 1e6:.0f} MB of weights per step > L2"},
            "tok_per_s": round(rt.world * 1000.0 / ms, 1),
            "pct_hbm_peak": round(100.0 * value / rt.world / peak, 2),
            "e2e": {"value": round(amount * rt.world / (e2e_ms * 1e-3) / div, 2), "unit": unit,
                    "h2d_bytes_per_step": int(4 * (x.numel() + ao.numel())),
                    "d2h_bytes_per_step": int(4 * (qkv.numel() + out.numel())),
                    "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": 2 * L * args.steps,  # one gemv_q4_kernel per GEMV
            "roofline": {"bound": "hbm", "achieved": round(qbytes / (q_ms * 1e-3) / 1e9, 1),
                         "peak": peak, "unit": "GB/s",
                         "frac": round(qbytes / (q_ms * 1e-3) / 1e9 / peak, 4), "traffic": None,
                         "kernel": "gemv_q4_kernel (activations quantized in each CTA; fused QKV, 6144x4096)",
                         "peak_source": f"{peak_kind} hbm_gbs", "bytes_per_launch": qbytes,
                         "avg_launch_ms": round(q_ms, 5)},
            "clocks": clk,
            "path": "molot_gemv_q4_dev x2 per layer",
        }
        if rt.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample(cfg)
        print(json.dumps(line), flush=True)
    rt.close()
    return 0


def fill_normal(torch, dst, template):
    """Fill a device tensor with N(0,1) values by tiling a seeded template
    (generating tens of GB of normals directly takes too long)."""
    flat = dst.view(-1)
    T = template.numel()
    for off in range(0, flat.numel(), T):
        k = min(T, flat.numel() - off)
        flat[off:off + k].copy_(template[:k])


class PagedBatch:
    """cfg4 (sequences split over the ranks by LPT, no collective) / cfg5 (kv
    heads split over the ranks, each layer's outputs gathered into every
    rank's [B][nq][d] by the decode itself over NVLink, molot_comm): the
    pools, block table, plan and per-layer inputs of this rank, and the step
    (batched append + paged decode per layer)."""

    def __init__(self, rt, args, cfg):
        import molot_b200 as mb
        from molot_b200 import shard
        torch = rt.torch
        self.rt, self.args, self.cfg, self.torch, self.mb = rt, args, cfg, torch, mb
        L, nq, nkv, d, ps = cfg["layers"], cfg["nq"], cfg["nkv"], cfg["d"], cfg["page"]
        self.L, self.nq, self.nkv, self.d, self.ps = L, nq, nkv, d, ps
        lens = self.lens = paged_lengths(cfg)
        B, G = len(lens), nq // nkv
        self.B = B
        self.head_sharded = cfg["kind"] == "paged_head"
        if not self.head_sharded:
            parts = shard.lpt_partition(lens, rt.world)
            mine = parts[rt.rank]
            g0, g1 = 0, nkv
            loads = [sum(lens[i] + 1 for i in p) for p in parts]
            self.imbalance = max(loads) / (sum(loads) / len(loads))
        else:
            mine = list(range(B))
            g0, g1 = shard.head_shard(nkv, rt.world, rt.rank)
            self.imbalance = 1.0
        self.mine, self.g0 = mine, g0
        nkv_l, Bl = g1 - g0, len(mine)
        nq_l = nkv_l * G
        self.nkv_l, self.nq_l, self.Bl = nkv_l, nq_l, Bl
        seq = self.seq = [lens[i] + 1 for i in mine]  # slots including the new token's
        pages = self.pages = [math.ceil(x / ps) for x in seq]
        P = sum(pages)
        rng = np.random.default_rng(cfg["seed"] + 1000 + rt.rank)
        perm = rng.permutation(P).astype(np.int32)
        bt = np.zeros((Bl, max(pages)), np.int32)
        k = 0
        for b, m in enumerate(pages):
            bt[b, :m] = perm[k:k + m]
            k += m
        self.bt_host = bt
        self.bt = torch.from_numpy(bt).to(rt.dev)
        rb = self.rb = kv_row_bytes(args.kv, d)
        self.pool_bytes = 2 * P * nkv_l * ps * rb
        self.L_res = max(1, min(L, int(args.resident_gb * 1e9 // self.pool_bytes)))
        gen = torch.Generator(device=rt.dev)
        gen.manual_seed(1234 + rt.rank)
        template = torch.randn(1 << 26, device=rt.dev, generator=gen)
        self.pools = []
        for _ in range(self.L_res):
            if args.kv == "q8":  # random codes, block scales 0.02
                K = torch.randint(0, 256, (P, nkv_l, ps, rb), dtype=torch.uint8, device=rt.dev,
                                  generator=gen)
                V = torch.randint(0, 256, (P, nkv_l, ps, rb), dtype=torch.uint8, device=rt.dev,
                                  generator=gen)
                for t in (K, V):
                    t[..., d:d + d // 8].view(torch.float32).fill_(0.02)
            else:
                dt = torch.bfloat16 if args.kv == "bf16" else torch.float32
                K = torch.empty((P, nkv_l, ps, d), device=rt.dev, dtype=dt)
                V = torch.empty((P, nkv_l, ps, d), device=rt.dev, dtype=dt)
                fill_normal(torch, K, template)
                fill_normal(torch, V, template[7:])
            self.pools.append((K, V))
        del template
        self.q_raw = torch.randn((L, Bl, nq_l, d), device=rt.dev, generator=gen)
        self.k_raw = torch.randn((L, Bl, nkv_l, d), device=rt.dev, generator=gen)
        self.v_raw = torch.randn((L, Bl, nkv_l, d), device=rt.dev, generator=gen)
        self.q_rot = torch.empty_like(self.q_raw)
        self.out = torch.empty_like(self.q_raw)
        self.freq = rope_freq(torch, cfg["theta"], d, rt.dev)
        self.scale = 1.0 / math.sqrt(d)
        self.plan = mb.PagedPlan(args.kv)
        self.plan.build(nq_l, nkv_l, d, seq, None, 0)
        self.local_layer_bytes = sum(2 * nkv_l * x * rb for x in seq)
        # cfg5: the peer gather (every rank's decode writes into every rank's
        # buffer); NCCL all-gather only if peer mappings cannot be made here
        self.mode, self.comm, self.note = None, None, None
        self.per_layer = B * nq * d
        if self.head_sharded:
            self.side = torch.cuda.Stream()
            self.events = [torch.cuda.Event() for _ in range(L)]
            try:
                self.comm = mb.Comm(rt.world, rt.rank, 4 * L * self.per_layer)
                if rt.world > 1:
                    hs = [None] * rt.world
                    rt.dist.all_gather_object(hs, self.comm.ipc_handle())
                    self.comm.open(hs)
                self.mode = "peer"
            except Exception as e:  # report, then gather with NCCL instead
                self.note = f"peer gather unavailable ({e}); NCCL all-gather used"
                if self.comm is not None:
                    self.comm.close()
                    self.comm = None
                self.mode = "nccl" if rt.world > 1 else None
                self.o_full = torch.empty((L, B, nq, d), device=rt.dev)
        torch.cuda.synchronize()

    def gathered(self):
        """[L][B][nq][d] view of this rank's gathered outputs (cfg5)."""
        if self.mode == "peer":
            return self.comm.buffer((self.L, self.B, self.nq, self.d))
        return self.o_full if self.mode == "nccl" else self.out

    def step(self, qr=None, kr=None, vr=None, decode_only=False, gather=True):
        from molot_b200 import shard
        torch = self.torch
        qr = self.q_raw if qr is None else qr
        kr = self.k_raw if kr is None else kr
        vr = self.v_raw if vr is None else vr
        st = torch.cuda.current_stream()
        peer = gather and not decode_only and self.mode == "peer"
        nccl = gather and not decode_only and self.mode == "nccl"
        plan, bt, ps = self.plan, self.bt, self.ps
        for l in range(self.L):
            K, V = self.pools[l % self.L_res]
            if not decode_only:
                plan.append(qr[l], kr[l], vr[l], self.q_rot[l], K, V, bt, ps, None, None, False,
                            1e-6, self.freq, st)
            if peer:
                plan.decode_gather(self.comm, self.q_rot[l], l * self.per_layer, K, V, bt, ps,
                                   self.scale, st)
                ev = self.events[l]
                ev.record(st)
                self.side.wait_event(ev)
                self.comm.wait(self.side)
            else:
                plan.decode(self.q_rot[l], self.out[l], K, V, bt, ps, self.scale, st)
                if nccl:
                    ev = self.events[l]
                    ev.record(st)
                    with torch.cuda.stream(self.side):
                        self.side.wait_event(ev)
                        shard.gather_heads(self.out[l], out=self.o_full[l])
        if peer or nccl:
            st.wait_stream(self.side)

    def check(self):
        self.plan.check()
        if self.comm is not None:
            self.comm.check()

    def parity(self):
        """Layer 0 after the timed steps (its pools hold the appended rows,
        q_rot[0] the rotated queries): this rank's decode against the oracle
        for the sequences `picked`, and for cfg5 the gathered [B][nq][d]
        against every rank's own decode output, bit for bit."""
        import oracle  # the checker, outside every timed region
        from concurrent.futures import ThreadPoolExecutor
        torch, rt = self.torch, self.rt
        K, V = self.pools[0]
        chk = torch.empty_like(self.out[0])
        self.plan.decode(self.q_rot[0], chk, K, V, self.bt, self.ps, self.scale)
        self.plan.check()
        order = sorted(range(self.Bl), key=lambda b: self.seq[b])
        if self.head_sharded:  # shortest, longest and two between
            picked = sorted({order[0], order[len(order) // 3], order[2 * len(order) // 3],
                             order[-1]})
        else:  # the longest sequence this rank holds
            picked = [order[-1]]
        q = self.q_rot[0].cpu().numpy()
        o = chk.cpu().numpy()
        res = {"kind": "oracle (attn.h:125-177 restated) on layer 0, after the timed steps",
               "seqs_checked_per_rank": len(picked), "tol": 1e-5}
        if self.args.kv != "f32":
            res.update(ok=None, skipped="oracle check only on FP32 pools")
            return res
        nkv_l, d, ps = self.nkv_l, self.d, self.ps

        def rows(pool, b):
            n = self.seq[b]
            idx = torch.from_numpy(self.bt_host[b, :self.pages[b]].astype(np.int64)).to(rt.dev)
            x = pool.index_select(0, idx).permute(0, 2, 1, 3).reshape(-1, nkv_l * d)[:n]
            return x.cpu().numpy()

        data = [(b, rows(K, b), rows(V, b)) for b in picked]

        def one(item):
            # the parity bar: within 1e-5 of the reference's algorithm, or --
            # at long contexts, where the reference's own FP32 sums drift
            # that far from the exact value -- no farther from a float64
            # evaluation than the reference itself (+1e-6)
            b, kb, vb = item
            n = self.seq[b]
            args_ = (q[b].reshape(-1), kb, vb, self.nq_l, nkv_l, n, d, self.scale, n - 1, 0)
            want = oracle.attn_decode_gqa_cache(*args_)
            e_ref = oracle.rel_err(o[b], want)
            if e_ref <= 1e-5:
                return e_ref, None, None, True
            f64 = oracle.attn_decode_gqa_cache_f64(*args_)
            e_gpu64, e_ref64 = oracle.rel_err(o[b], f64), oracle.rel_err(want, f64)
            return e_ref, e_gpu64, e_ref64, e_gpu64 <= e_ref64 + 1e-6

        with ThreadPoolExecutor(max_workers=min(len(data), os.cpu_count() or 1)) as ex:
            out = list(ex.map(one, data))
        del data
        err = rt.max(max(x[0] for x in out))
        ok = all(x[3] for x in out)
        res.update(max_rel_err=err,
                   bar="rel err <= 1e-5 vs the reference's algorithm, or vs float64 no more "
                       "than the reference's own + 1e-6")
        f64 = [x for x in out if x[1] is not None]
        if f64:
            res.update(vs_f64={"gpu": max(x[1] for x in f64), "reference": max(x[2] for x in f64),
                               "seqs": len(f64)})
        if self.head_sharded and self.mode == "peer":
            full = self.comm.buffer((self.B, self.nq, self.d))
            full.fill_(float("nan"))
            rt.barrier()
            self.plan.decode_gather(self.comm, self.q_rot[0], 0, K, V, self.bt, self.ps,
                                    self.scale)
            self.comm.wait()
            self.check()
            rt.barrier()
            if rt.world > 1:
                parts = torch.empty((rt.world,) + tuple(chk.shape), device=rt.dev)
                rt.dist.all_gather_into_tensor(parts, chk.contiguous())
                want = parts.permute(1, 0, 2, 3).reshape(self.B, self.nq, self.d)
            else:
                want = chk
            same = bool(torch.equal(full, want))
            bad = rt.max(0.0 if same else 1.0)
            res["gather_bit_exact"] = bad == 0.0
            ok = ok and bad == 0.0
            rt.barrier()
        res["ok"] = bool(rt.max(0.0 if ok else 1.0) == 0.0)
        return res

    def close(self):
        self.plan.close()
        if self.comm is not None:
            self.comm.close()
        self.pools = []


def paged_config(args, cfg, pb, world):
    lens = pb.lens
    par = (f"sequence-sharded (LPT on lengths) over {world} rank(s), no collective"
           if not pb.head_sharded else
           f"kv-head sharded over {world} rank(s) ({pb.nkv_l} kv heads each); outputs written "
           "into every rank's [B][nq][d] by the decode itself over NVLink (molot_comm)"
           if pb.mode == "peer" else
           f"kv-head sharded over {world} rank(s); per-layer NCCL all-gather on a second stream")
    return {"workload": f"{cfg['name']}: {cfg['desc']}",
            "layers": pb.L, "nq": pb.nq, "nkv": pb.nkv, "head_dim": pb.d, "batch": pb.B,
            "batch_rank0": pb.Bl, "len_min": min(lens), "len_mean": round(sum(lens) / pb.B, 1),
            "len_max": max(lens), "page_size": pb.ps, "resident_layer_pools": pb.L_res,
            "parallelism": par, "kv_dtype": args.kv,
            "l2": f"each layer pool ({pb.pool_bytes / 1e9:.2f} GB on rank 0) > L2"}


def paged_measure(rt, args, cfg, brief=False):
    """Device-time measurements of a paged config at this world size: the
    step (CUDA graph, max over ranks), rank 0's decode launches alone (the
    roofline), the limiter, and the in-run parity check."""
    torch = rt.torch
    pb = PagedBatch(rt, args, cfg)
    for _ in range(args.warmup):
        pb.step()
    pb.check()
    graph = capture(torch, pb.step)
    dgraph = capture(torch, lambda: pb.step(decode_only=True))
    for _ in range(args.warmup):
        graph.replay()
    ms, reps = timed_repeats(rt, graph.replay, args.steps, 3 if brief else args.repeats)
    mine_ms = rt.timed(graph.replay, args.steps)  # this rank alone, for the imbalance
    mean_ms = rt.sum(mine_ms) / rt.world
    for _ in range(args.warmup):
        dgraph.replay()
    dec_ms = rt.timed(dgraph.replay, args.steps) / pb.L
    pb.check()
    limiter = {"lpt_bytes_max_over_mean": round(pb.imbalance, 4),
               "rank_step_ms_max_over_mean": round(rt.max(mine_ms) / mean_ms, 4)}
    if pb.head_sharded and pb.mode is not None:
        ngraph = capture(torch, lambda: pb.step(gather=False))
        for _ in range(args.warmup):
            ngraph.replay()
        plain_ms = rt.max(rt.timed(ngraph.replay, args.steps))
        del ngraph
        limiter.update(gather=pb.mode, step_without_gather_ms=round(plain_ms, 4),
                       gather_cost_ms_per_step=round(ms - plain_ms, 4),
                       gather_cost_pct=round(100.0 * (ms - plain_ms) / ms, 2))
        if pb.note:
            limiter["note"] = pb.note
    pb.check()
    del graph, dgraph
    parity = pb.parity()
    peak, peak_kind = hbm_peak()
    total = step_bytes(cfg, args.kv)
    achieved = pb.local_layer_bytes / (dec_ms * 1e-3) / 1e9
    res = {"value": round(total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
           "ms_per_step": round(ms, 4), "tok_per_s": round(pb.B * 1000.0 / ms, 2),
           "scaling": "strong", "n_gpus": rt.world,
           "pct_hbm_peak": round(100.0 * total / (ms * 1e-3) / 1e9 / rt.world / peak, 2),
           "repeats_ms": [round(x, 4) for x in reps],
           "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                        "unit": "GB/s", "frac": round(achieved / peak, 4),
                        "kernel": "gqa_decode_kernel<128,%s> (paged plan)" %
                                  ("4,2" if pb.nq // pb.nkv == 8 else "4,1"),
                        "timed": "rank 0's paged decode launches alone",
                        "bytes_per_launch": pb.local_layer_bytes,
                        "avg_launch_ms": round(dec_ms, 5),
                        "peak_source": f"{peak_kind} hbm_gbs"},
           "limiter": limiter, "parity": parity,
           "config": paged_config(args, cfg, pb, rt.world),
           "path": "molot_paged_append + " + ("molot_paged_decode_gather + molot_comm_wait"
                                              if pb.mode == "peer" else "molot_paged_decode")
                   + " per layer (CUDA graph)"}
    if brief:
        pb.close()
        return res
    return res, pb


def run_paged(args, cfg):
    """cfg4 / cfg5 as the line's own workload (with e2e)."""
    rt = Rt()
    torch = rt.torch
    clocks = ClockSampler(rt.local)
    clocks.start()
    res, pb = paged_measure(rt, args, cfg)
    clk = clocks.stop()
    h = [pinned_like(torch, t, 5 + i) for i, t in enumerate((pb.q_raw, pb.k_raw, pb.v_raw))]
    res_dev = pb.gathered() if pb.head_sharded else pb.out
    h_o = torch.empty(tuple(res_dev.shape)).pin_memory()
    dq, dk, dv = (torch.empty_like(t) for t in (pb.q_raw, pb.k_raw, pb.v_raw))

    def e2e_step():
        dq.copy_(h[0], non_blocking=True)
        dk.copy_(h[1], non_blocking=True)
        dv.copy_(h[2], non_blocking=True)
        pb.step(dq, dk, dv)
        h_o.copy_(res_dev, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    e2e_ms = rt.max(rt.timed(e2e_step, args.steps))
    pb.check()
    h2d = rt.sum(4 * pb.L * pb.Bl * (pb.nq_l + 2 * pb.nkv_l) * pb.d)
    d2h = rt.sum(h_o.numel() * 4)
    if rt.rank == 0:
        emit(rt, args, cfg, res["ms_per_step"], e2e_ms, clk, h2d=h2d, d2h=d2h,
             launches=(2 if pb.mode != "peer" else 3) * pb.L * args.steps,
             roof={k: v for k, v in res["roofline"].items()
                   if k not in ("peak", "unit", "frac", "peak_source")} |
             {"traffic": read_traffic("gqa_decode_kernel", args.config)},
             config=res["config"], scaling="strong",
             extra={"path": res["path"], "limiter": res["limiter"], "parity": res["parity"],
                    "repeats_ms": res["repeats_ms"]})
    pb.close()
    rt.close()
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
    ap.add_argument("--kv", choices=["f32", "bf16", "q8"], default="f32",
                    help="KV-cache storage of cfg1/cfg2 (bf16: half the bytes; q8: int8 "
                         "codes + per-32 scales, 0.28x the bytes; FP32 math throughout)")
    ap.add_argument("--resident-gb", type=float, default=40.0,
                    help="cfg4/cfg5: device memory for distinct layer pools per rank")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (small cases for profiler captures)")
    ap.add_argument("--repeats", type=int, default=5,
                    help="timed windows of exactly --steps steps each; the line reports the "
                         "median window")
    ap.add_argument("--no-extras", dest="extras", action="store_false",
                    help="default run only: skip the cfg1/cfg3 objects (N=1) and the batched "
                         "cfg4/cfg5 objects (every N)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.layers > 0:
        cfg["layers"] = args.layers
    if args.impl == "reference":
        return run_reference(args, cfg)
    if cfg["kind"] == "single":
        return run_single(args, cfg)
    if cfg["kind"] == "gemma":
        return run_gemma(args, cfg)
    if cfg["kind"] == "prefill":
        return run_prefill(args, cfg)
    if cfg["kind"] == "gemv":
        return run_gemv(args, cfg)
    return run_paged(args, cfg)


if __name__ == "__main__":
    sys.exit(main())
