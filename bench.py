#!/usr/bin/env python
"""Decode-attention benchmark: Qwen3-4B-shaped paged decode, batch 128, 36 layers.

One step = one decode step of the model's attention: for each of 36 layers
(each with its own paged KV cache, so no layer is served from L2) the
split-KV paged decode over B=128 sequences with Hq=32, Hk=8, D=128, bf16,
page size 16 and context lengths prompt U[128,1024] + generated U[1,256].

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  ``value`` is the whole-job KV HBM throughput
(algorithmic K+V bytes of all ranks / max-over-ranks device time, GB/s) with
inputs resident; ``e2e`` is the same metric through the public
``flash_attn_with_kvcache`` with q copied from pinned host memory and every
layer's output read back inside the timed region.  Multi-GPU runs are weak
scaling for the headline: every rank decodes its own batch of 128 sequences,
no collective on the data path.

Extra keys of the same line (each its own measurement, same timing rules):
  ``fp8``      the headline workload with e4m3 KV caches (half the bytes);
  ``prefill``  config 5: causal varlen forward over {15000, 1024, 512, 37},
               Hq=32, Hk=8, D=128, TFLOP/s against the bf16 tensor peak;
               ``prefill_heads`` (N>1) the same batch split by KV-head groups;
  ``longctx``  config 5 decode: 16384-token contexts at B=8 and B=1; with N>1
               every rank holds a page-aligned range of every sequence and the
               (O, LSE) records are exchanged once per layer, by the fused
               NVLink peer-store kernels and by one NCCL all-gather, both
               checked against a one-GPU decode over the whole context;
  ``strong``   (N>1) the one config-2 batch of 128 split 128/N per rank.

``--impl reference`` times the reference's own CPU path
(``mxflashattn.flash_attn_with_kvcache`` with MXFLASHATTN_ALLOW_FALLBACK=1,
installed from the reference checkout into baseline/_ref) on all host cores;
when that package is absent it times the numpy oracle port instead and says
so (``kind: "port"``).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

HQ, HKV, D, PS, BATCH, LAYERS = 32, 8, 128, 16, 128, 36
LONG_CTX = 16384
LONG_BATCHES = (8, 1)
PREFILL_LENS = "15000,1024,512,37"
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one decode
# launch of the default workload (batch 128, seed 2026), taken once by ncu
# on one launch of this exact command; reported as a profile value
# (`traffic_source`), not measured by the run that prints it.
NCU_TRAFFIC_BYTES = {(128, 2026): 381.349120e6}
METRIC = "decode-attn KV HBM GB/s & tok/s (Qwen3-4B shape, b128) at 1/2/4/8 B200"
WORKLOAD = "qwen3-4b paged decode attention, b128, 36 layers (config 2)"
REF_PACKAGE_DIR = os.path.join(REPO, "baseline", "_ref")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--seed", type=int, default=2026)
    ap.add_argument("--workload", choices=("decode", "prefill"), default="decode",
                    help="decode: config 2 (headline); prefill: config 5 varlen causal forward")
    ap.add_argument("--prefill-lens", default=PREFILL_LENS)
    ap.add_argument("--kv-dtype", choices=("bf16", "fp8"), default="bf16",
                    help="decode KV cache type (fp8 = float8_e4m3fn at scale 1; bytes counted at 1 B/element)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="headline decode line only (no fp8 / prefill / longctx / strong keys)")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return None


def measured_peaks():
    data = _peaks()
    if data is not None:
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    data = _peaks()
    if data is not None:
        return float(data["bf16_tflops"]), "measured bf16_tflops (burst)"
    return 1590.0, "fallback bf16 burst"


def measured_tensor_peak_sustained():
    """cuBLAS bf16 back to back for seconds under the power cap (fallback: ~1.4 PFLOP/s)."""
    data = _peaks()
    if data is not None and data.get("bf16_tflops_sustained"):
        return float(data["bf16_tflops_sustained"]), "measured bf16_tflops_sustained"
    return 1400.0, "fallback bf16 sustained"


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons; ``summary`` keeps the
    samples whose timestamps fall inside the marked timed window."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, interval_ms: int = 50):
        self.device_index = device_index
        self.interval_ms = interval_ms
        self.proc = None
        self.window = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms",
                 str(self.interval_ms), "-i", str(self.device_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.5)  # let nvidia-smi attach before the timed region
        return self

    def mark(self, t0: float, t1: float):
        self.window = (t0, t1)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        import datetime

        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        parsed = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                parsed.append((ts, float(parts[2]), float(parts[3]), parts[6:10]))
            except ValueError:
                continue
        inside = parsed
        if self.window is not None and parsed:
            t0, t1 = self.window
            inside = [x for x in parsed if t0 - 0.06 <= x[0] <= t1 + 0.06]
            if not inside:  # window shorter than one interval: nearest sample
                inside = [min(parsed, key=lambda x: abs(x[0] - (t0 + t1) / 2))]
        reasons = sorted({n for x in inside for n, v in zip(names, x[3]) if v.lower() == "active"})
        sm = [x[1] for x in inside]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max((x[2] for x in inside), default=None),
                "reasons": reasons, "samples": len(sm)}


# ------------------------------------------------------- reference CPU path

def import_reference():
    """The reference package installed into baseline/_ref, or None when absent."""
    if not os.path.isdir(os.path.join(REF_PACKAGE_DIR, "mxflashattn")):
        return None
    sys.path.insert(0, REF_PACKAGE_DIR)
    try:
        import mxflashattn
    except Exception:  # noqa: BLE001 -- any import failure means: time the port instead
        return None
    finally:
        sys.path.remove(REF_PACKAGE_DIR)
    return mxflashattn


def reference_inputs(lengths, seed):
    """One layer of the config-2 workload as CPU torch tensors (bf16 q / caches, int32 table)."""
    import torch

    gen = torch.Generator().manual_seed(seed)
    lengths = [int(x) for x in lengths]
    need = [(L + PS - 1) // PS for L in lengths]
    pages = sum(need)
    k = torch.randn((pages, PS, HKV, D), generator=gen, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn((pages, PS, HKV, D), generator=gen, dtype=torch.float32).to(torch.bfloat16)
    q = torch.randn((len(lengths), 1, HQ, D), generator=gen, dtype=torch.float32).to(torch.bfloat16)
    perm = torch.randperm(pages, generator=gen).to(torch.int32)
    table = torch.zeros((len(lengths), max(need)), dtype=torch.int32)
    off = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[off:off + n]
        off += n
    seqlens = torch.tensor(lengths, dtype=torch.int32)
    return {"q": q, "k_cache": k, "v_cache": v, "block_table": table, "cache_seqlens": seqlens}


class CpuBaseline:
    """Times the reference's CPU implementation of the decode path on this host.

    The reference's own ``flash_attn_with_kvcache`` with its PyTorch fallback
    (kind "reference", torch threads = every core this process may use); when
    the reference package is not installed, the numpy oracle port of the same
    algorithm (kind "port").  One call = one layer of the config-2 batch.
    """

    def __init__(self, lengths, seed):
        import torch

        self.lengths = [int(x) for x in lengths]
        self.cores = host_cores()
        self.ref = import_reference()
        self.inputs = reference_inputs(self.lengths, seed)
        self.nbytes = sum(self.lengths) * HKV * D * 2 * 2
        torch.set_num_threads(self.cores)
        if self.ref is not None:
            self.kind = "reference"
            self.what = ("reference mxflashattn.flash_attn_with_kvcache (MXFLASHATTN_ALLOW_FALLBACK=1, torch "
                         f"{torch.__version__} CPU, {self.cores} threads)")
        else:
            self.kind = "port"
            self.what = "numpy fp32 oracle port of the reference's CPU path (reference package not installed)"
            self.np_inputs = {k: (v.float().numpy() if v.dtype == torch.bfloat16 else v.numpy())
                              for k, v in self.inputs.items() if v is not None}

    def call(self) -> float:
        import warnings

        t = self.inputs
        t0 = time.perf_counter()
        if self.ref is not None:
            # the reference reads its fallback switch at call time
            prev = os.environ.get("MXFLASHATTN_ALLOW_FALLBACK")
            os.environ["MXFLASHATTN_ALLOW_FALLBACK"] = "1"
            try:
                with warnings.catch_warnings():
                    warnings.simplefilter("ignore", RuntimeWarning)
                    self.ref.flash_attn_with_kvcache(t["q"], t["k_cache"], t["v_cache"],
                                                     cache_seqlens=t["cache_seqlens"], block_table=t["block_table"],
                                                     softmax_scale=D ** -0.5)
            finally:
                if prev is None:
                    del os.environ["MXFLASHATTN_ALLOW_FALLBACK"]
                else:
                    os.environ["MXFLASHATTN_ALLOW_FALLBACK"] = prev
        else:
            import oracle

            n = self.np_inputs
            oracle.attention_kvcache(n["q"], n["k_cache"], n["v_cache"], cache_seqlens=n["cache_seqlens"].copy(),
                                     block_table=n["block_table"], softmax_scale=D ** -0.5)
        return time.perf_counter() - t0

    def sample(self) -> str:
        return (f"all {len(self.lengths)} sequences of one layer per call (mean ctx "
                f"{sum(self.lengths) / len(self.lengths):.1f}), {self.what}, on {cpu_model()}")


def run_reference(args):
    """--impl reference: the reference's CPU path on this host's cores (rank 0 only)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from mxflashattn_b200 import synthetic as syn

    lengths = syn.qwen3_4b_lengths(args.seed, args.batch)
    base = CpuBaseline(lengths, args.seed)
    for _ in range(max(1, min(args.warmup, 3))):
        base.call()
    times = [base.call() for _ in range(args.steps)]
    sec = sum(times) / len(times)
    gbs = base.nbytes / sec / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 math)", "data": "synthetic",
        "config": headline_config(args, lengths, world, False),
        "sample": f"one step = one layer of the {args.batch}-sequence batch (all sequences); GB/s and tok/s "
                  "scale by the algorithmic bytes of that layer",
        "tok_per_s": args.batch / sec / args.layers,
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": base.cores, "kind": base.kind,
                         "sample": base.sample()},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def headline_config(args, lengths, world, fp8):
    """The ``config`` object of the headline line; both arms print the same one."""
    import numpy as np

    bytes_step = int(np.sum(lengths)) * HKV * D * 2 * (1 if fp8 else 2) * args.layers
    return {"workload": WORKLOAD + (", e4m3 KV cache" if fp8 else ""), "batch": args.batch,
            "layers": args.layers, "hq": HQ, "hkv": HKV, "head_dim": D, "page_size": PS,
            "mean_ctx": float(np.mean(lengths)),
            "l2": f"inputs larger than L2: {args.layers} distinct layer caches, "
                  f"{bytes_step / 1e9:.1f} GB read per step",
            "parallelism": f"dp{world} (independent batches, no collective)"}


# ------------------------------------------------------------ device helpers

class Ranks:
    """Process group plumbing: barrier, max-over-ranks reductions (no-ops at N=1)."""

    def __init__(self, world, rank, device):
        self.world, self.rank, self.device = world, rank, device
        self.dist = None
        if world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=device)
            self.dist = dist

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def max(self, values):
        """Elementwise max over ranks of a list of floats (one collective)."""
        if self.dist is None:
            return list(values)
        import torch

        t = torch.tensor(list(values), device=self.device, dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(x) for x in t.tolist()]

    def close(self):
        if self.dist is not None:
            self.dist.barrier()
            self.dist.destroy_process_group()


def capture(step, device):
    """A CUDA graph of ``step()`` (warmed up twice on a side stream first)."""
    import torch

    stream = torch.cuda.current_stream(device)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
    stream.wait_stream(side)
    torch.cuda.synchronize(device)
    with torch.cuda.graph(graph, stream=side):
        step()
    torch.cuda.synchronize(device)
    return graph


def time_graph(graph, steps, warmup, device, ranks, clocks=None):
    """Device ms of ``steps`` back-to-back replays (after ``warmup``), CUDA events on the launching stream."""
    import torch

    stream = torch.cuda.current_stream(device)
    for _ in range(max(warmup, 3)):
        graph.replay()
    torch.cuda.synchronize(device)
    ranks.barrier()
    torch.cuda.synchronize(device)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    w0 = time.time()
    t0.record(stream)
    for _ in range(steps):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize(device)
    if clocks is not None:
        clocks.mark(w0, time.time())
    ranks.barrier()
    return t0.elapsed_time(t1)


def build_layers(lengths, seed_base, layers, device, fp8=False):
    import torch

    from mxflashattn_b200 import synthetic as syn

    out = []
    for layer in range(layers):
        t = syn.device_paged_decode(seed=seed_base + layer, lengths=lengths, q_heads=HQ, kv_heads=HKV, head_dim=D,
                                    dtype="bf16", page_size=PS, device=device)
        if fp8:  # e4m3 caches at scale 1 (N(0,1) values fit the e4m3 range)
            t["k_cache"] = t["k_cache"].to(torch.float8_e4m3fn)
            t["v_cache"] = t["v_cache"].to(torch.float8_e4m3fn)
        out.append(t)
    torch.cuda.synchronize(device)
    return out


def decode_graph(layers, device):
    """(graph, step, plan) for one decode step over ``layers``.

    The step first computes the batch's longest-first order once
    (``kvcache_length_order``, one small kernel; None for a batch of one) and
    every layer's launch takes it, as a model's decode step would."""
    import torch

    from mxflashattn_b200 import backend

    B = layers[0]["q"].shape[0]
    max_len = layers[0]["block_table"].shape[1] * PS
    num_splits, chunk_len = backend.kvcache_plan(B, 1, HQ, HKV, D, max_len)
    outs = [torch.empty_like(t["q"]) for t in layers]
    scale = D ** -0.5

    def step(ev=None):
        stream = torch.cuda.current_stream(device)
        order = backend.kvcache_length_order(layers[0]["cache_seqlens"])  # every layer has the same lengths
        for i, t in enumerate(layers):
            if ev is not None:
                ev[2 * i].record(stream)
            backend.kvcache_attention(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"],
                                      scale, False, num_splits=num_splits, chunk_len=chunk_len, out=outs[i],
                                      length_order=order)
            if ev is not None:
                ev[2 * i + 1].record(stream)

    return capture(step, device), step, (num_splits, chunk_len)


# -------------------------------------------------------------------- ours

def run_ours(args):
    import torch

    world, rank, local = dist_env()
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)
    ranks = Ranks(world, rank, device)

    from mxflashattn_b200 import flash_attn_with_kvcache, kvcache_length_order, synthetic as syn

    lengths = syn.qwen3_4b_lengths(args.seed + rank, args.batch)
    fp8 = args.kv_dtype == "fp8"
    layers = build_layers(lengths, 1000 * (rank + 1), args.layers, device, fp8=fp8)
    bytes_layer = syn.kv_bytes(lengths, HKV, D, elem_bytes=1 if fp8 else 2)
    bytes_step = bytes_layer * args.layers
    stream = torch.cuda.current_stream(device)
    scale = D ** -0.5

    graph, step, (num_splits, chunk_len) = decode_graph(layers, device)
    launches_per_layer = 1  # split plans merge in the same launch (counted single launch)
    launches_per_step = 1 if 1 < args.batch <= 512 else 0  # the length order, once per step
    clocks = ClockSampler(device.index).start()
    elapsed_ms = time_graph(graph, args.steps, args.warmup, device, ranks, clocks)
    clocks.stop()
    per_launch_ms = elapsed_ms / args.steps / args.layers
    if num_splits > 1:  # one event pair per layer: the single launch per layer timed alone
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.layers)]
        step(evs)
        torch.cuda.synchronize(device)
        per_launch_ms = sum(evs[2 * i].elapsed_time(evs[2 * i + 1]) for i in range(args.layers)) / args.layers
    elapsed_ms = ranks.max([elapsed_ms])[0]
    ms_step = elapsed_ms / args.steps
    value = world * bytes_step / (ms_step * 1e-3) / 1e9
    tok_s = world * args.batch / (ms_step * 1e-3)
    del graph

    # --------------------------------------------------------------- e2e
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, layers, lengths, bytes_step, device, ranks, flash_attn_with_kvcache, scale,
                      order_fn=kvcache_length_order)

    # ------------------------------------------------------- CPU baseline
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = CpuBaseline(syn.qwen3_4b_lengths(args.seed, args.batch), args.seed)
        base.call()
        times = [base.call() for _ in range(5)]
        sec = sum(times) / len(times)
        cpu = {"value": base.nbytes / sec / 1e9, "unit": "GB/s", "cores": base.cores, "kind": base.kind,
               "sample": base.sample() + ", mean of 5 timed calls after 1 untimed"}

    peak, peak_kind = measured_peaks()
    achieved = bytes_layer / (per_launch_ms * 1e-3) / 1e9
    traffic = None if fp8 else NCU_TRAFFIC_BYTES.get((args.batch, args.seed))
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (e4m3 KV cache)" if fp8 else "bf16", "data": "synthetic",
        "config": headline_config(args, lengths, world, fp8),
        "plan": {"num_splits": num_splits, "chunk_len": chunk_len},
        "tok_per_s": tok_s,
        "e2e": e2e,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of this "
                                        "workload (profile value, not measured by this run)") if traffic else None,
                     "peak_source": f"{peak_kind} hbm_gbs",
                     "kernel": "paged_decode_kernel", "bytes_per_launch": bytes_layer,
                     "avg_launch_ms": per_launch_ms},
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "gpu_launches": args.steps * (args.layers * launches_per_layer + launches_per_step),
        "timing": "CUDA graph replay of the 36-layer step; e2e is eager through the public API",
    }
    del layers
    torch.cuda.empty_cache()

    if not args.no_extras:
        if not fp8:
            line["fp8"] = extra_fp8(args, lengths, device, ranks)
        line["prefill"] = prefill_measure(args, device, ranks, sharded=False, with_cpu=False)
        if world > 1:
            line["prefill_heads"] = prefill_measure(args, device, ranks, sharded=True, with_cpu=False)
            line["strong"] = extra_strong(args, device, ranks)
        line["longctx"] = extra_longctx(args, device, ranks)
    if rank == 0:
        print(json.dumps(line), flush=True)
    ranks.close()


def run_e2e(args, layers, lengths, bytes_step, device, ranks, api, scale, order_fn=None):
    """The headline metric through the public API with host buffers, copies inside the timed region.

    Every step uploads that step's inputs (the 36 layers' q and the lengths)
    from pinned host memory in one copy and reads the 36 layers' outputs back
    in one copy.  Device buffers alternate by step parity, so the upload of
    step s+1 and the read-back of step s-1 run on the copy engines while step
    s computes; every copy of every timed step lies inside the timed region.
    """
    import torch

    world = ranks.world
    stream = torch.cuda.current_stream(device)
    q_host = torch.stack([t["q"] for t in layers]).cpu().pin_memory()  # [layers, B, 1, HQ, D]
    out_host = torch.empty_like(q_host, pin_memory=True)
    sl_host = layers[0]["cache_seqlens"].cpu().pin_memory()
    q_dev = [torch.empty_like(q_host, device=device) for _ in range(2)]
    out_dev = [torch.empty_like(q_host, device=device) for _ in range(2)]
    sl_dev = [torch.empty_like(layers[0]["cache_seqlens"]) for _ in range(2)]
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    ev_up = [torch.cuda.Event() for _ in range(2)]    # inputs of buffer p uploaded
    ev_used = [torch.cuda.Event() for _ in range(2)]  # the step on buffer p finished its kernels
    ev_down = [torch.cuda.Event() for _ in range(2)]  # outputs of buffer p read back
    count = [0]

    def e2e_step():
        p = count[0] & 1
        count[0] += 1
        with torch.cuda.stream(h2d):
            h2d.wait_event(ev_used[p])  # the step two back has finished reading these inputs
            q_dev[p].copy_(q_host, non_blocking=True)
            sl_dev[p].copy_(sl_host, non_blocking=True)
            ev_up[p].record(h2d)
        stream.wait_event(ev_up[p])
        stream.wait_event(ev_down[p])  # ... and its outputs have left this buffer
        kw = {} if order_fn is None else {"length_order": order_fn(sl_dev[p])}  # once per step
        for i, t in enumerate(layers):
            api(q_dev[p][i], t["k_cache"], t["v_cache"], cache_seqlens=sl_dev[p], block_table=t["block_table"],
                softmax_scale=scale, out=out_dev[p][i], **kw)
        ev_used[p].record(stream)
        with torch.cuda.stream(d2h):
            d2h.wait_event(ev_used[p])
            out_host.copy_(out_dev[p], non_blocking=True)
            ev_down[p].record(d2h)

    for _ in range(4):
        e2e_step()
    torch.cuda.synchronize(device)
    ranks.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    h0 = time.perf_counter()
    e0.record(stream)
    h2d.wait_stream(stream)  # the first upload starts inside the timed region
    for _ in range(args.steps):
        e2e_step()
    stream.wait_stream(d2h)  # the last read-back ends inside the timed region
    e1.record(stream)
    host_s = time.perf_counter() - h0  # host time to enqueue every step (no synchronisation inside)
    torch.cuda.synchronize(device)
    ranks.barrier()
    e_ms = e0.elapsed_time(e1)

    # the copy engines alone: one step's upload, then its read-back
    c = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    torch.cuda.synchronize(device)
    c[0].record(h2d)
    with torch.cuda.stream(h2d):
        q_dev[0].copy_(q_host, non_blocking=True)
    c[1].record(h2d)
    c[2].record(d2h)
    with torch.cuda.stream(d2h):
        d2h.wait_event(c[1])
        out_host.copy_(out_dev[0], non_blocking=True)
    c[3].record(d2h)
    torch.cuda.synchronize(device)
    h2d_ms, d2h_ms = c[0].elapsed_time(c[1]), c[1].elapsed_time(c[3])
    e_ms, host_ms = ranks.max([e_ms, host_s * 1e3])
    e_step = e_ms / args.steps
    q_bytes = q_host.numel() * q_host.element_size()
    o_bytes = out_host.numel() * out_host.element_size()
    return {"value": world * bytes_step / (e_step * 1e-3) / 1e9, "unit": "GB/s",
            "h2d_bytes_per_step": q_bytes + sl_host.numel() * sl_host.element_size(),
            "d2h_bytes_per_step": o_bytes, "ms_per_step": e_step,
            "tok_per_s": world * args.batch / (e_step * 1e-3),
            "host_ms_per_step": host_ms / args.steps,
            "host_us_per_call": host_ms * 1e3 / (args.steps * len(layers)),
            "h2d_gbs_alone": q_bytes / (h2d_ms * 1e-3) / 1e9 if h2d_ms > 0 else None,
            "d2h_gbs_alone": o_bytes / (d2h_ms * 1e-3) / 1e9 if d2h_ms > 0 else None,
            "method": "public flash_attn_with_kvcache per layer (out= a slot of the step's output buffer, "
                      "length_order= from kvcache_length_order once per step), eager; "
                      "per step one upload of every layer's q and the lengths and one read-back of every layer's "
                      "output, on copy streams overlapping the neighbouring steps' kernels; *_gbs_alone = one "
                      "step's copies timed alone"}


def extra_fp8(args, lengths, device, ranks):
    """The headline workload over e4m3 caches (k_scale = v_scale = 1)."""
    import torch

    from mxflashattn_b200 import synthetic as syn

    layers = build_layers(lengths, 1000 * (ranks.rank + 1), args.layers, device, fp8=True)
    graph, _, (num_splits, _) = decode_graph(layers, device)
    ms = time_graph(graph, args.steps, args.warmup, device, ranks)
    per_launch = ms / args.steps / args.layers
    ms = ranks.max([ms])[0]
    del graph, layers
    torch.cuda.empty_cache()
    bytes_layer = syn.kv_bytes(lengths, HKV, D, elem_bytes=1)
    ms_step = ms / args.steps
    peak, kind = measured_peaks()
    achieved = bytes_layer / (per_launch * 1e-3) / 1e9
    return {"metric": "decode-attn KV HBM GB/s, e4m3 KV cache (config 2 shape)",
            "value": ranks.world * bytes_layer * args.layers / (ms_step * 1e-3) / 1e9, "unit": "GB/s",
            "ms_per_step": ms_step, "tok_per_s": ranks.world * args.batch / (ms_step * 1e-3),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": f"{kind} hbm_gbs",
                         "bytes_per_launch": bytes_layer, "bytes_rule": "1 B per cached e4m3 element"},
            "num_splits": num_splits, "gpu_launches": args.steps * (args.layers + (1 < len(lengths) <= 512))}


def extra_strong(args, device, ranks):
    """The one config-2 batch of 128 sequences split 128/N per rank (no collective)."""
    import torch

    from mxflashattn_b200 import context_split as cs, synthetic as syn

    all_lengths = syn.qwen3_4b_lengths(args.seed, args.batch)
    mine = cs.shard_batch(args.batch, ranks.world, ranks.rank)
    lengths = all_lengths[mine.start:mine.stop]
    layers = build_layers(lengths, 5000 + 100 * ranks.rank, args.layers, device)
    graph, _, (num_splits, _) = decode_graph(layers, device)
    ms = ranks.max([time_graph(graph, args.steps, args.warmup, device, ranks)])[0]
    del graph, layers
    torch.cuda.empty_cache()
    total = syn.kv_bytes(all_lengths, HKV, D) * args.layers
    ms_step = ms / args.steps
    return {"metric": "decode-attn KV HBM GB/s, config-2 batch of 128 split over the ranks",
            "value": total / (ms_step * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms_step,
            "tok_per_s": args.batch / (ms_step * 1e-3), "scaling": "strong",
            "sequences_per_rank": len(lengths), "num_splits": num_splits}


# ------------------------------------------------------------------ prefill

def prefill_measure(args, device, ranks, *, sharded: bool, with_cpu: bool):
    """Config 5 prefill: causal flash_attn_varlen_func over packed sequences.

    ``sharded``: each rank runs the KV heads ``shard_kv_heads(HKV, N, rank)``
    of the one batch (strong scaling); otherwise every rank runs the whole
    batch (weak scaling).
    """
    import numpy as np
    import torch

    from mxflashattn_b200 import backend, context_split as cs, flash_attn_varlen_func

    world, rank = ranks.world, ranks.rank
    lens = [int(x) for x in args.prefill_lens.split(",")]
    total = sum(lens)
    heads = cs.shard_kv_heads(HKV, world, rank) if sharded else range(HKV)
    hkv = len(heads)
    hq = hkv * (HQ // HKV)
    gen = torch.Generator(device=device)
    gen.manual_seed(args.seed + (0 if sharded else rank))
    q = torch.randn((total, HQ, D), generator=gen, device=device, dtype=torch.bfloat16)
    k = torch.randn((total, HKV, D), generator=gen, device=device, dtype=torch.bfloat16)
    v = torch.randn((total, HKV, D), generator=gen, device=device, dtype=torch.bfloat16)
    if sharded:
        g = HQ // HKV
        q = q[:, heads.start * g:heads.stop * g].contiguous()
        k = k[:, heads.start:heads.stop].contiguous()
        v = v[:, heads.start:heads.stop].contiguous()
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=device)
    flops_rank = 4 * hq * D * sum(L * (L + 1) // 2 for L in lens)
    flops_job = flops_rank * world if not sharded else 4 * HQ * D * sum(L * (L + 1) // 2 for L in lens)
    scale = D ** -0.5
    stream = torch.cuda.current_stream(device)

    def step():
        backend.flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), True, scale)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(device)
    ranks.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(device.index).start()
    w0 = time.time()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    clocks.mark(w0, time.time())
    clocks.stop()
    ms_local = e0.elapsed_time(e1) / args.steps

    e2e_ms = None
    hq_b = hk_b = None
    if not args.no_e2e:  # public API with host inputs: q/k/v and cu_seqlens uploaded, output read back
        hq_b, hk_b, hv_b = (t.cpu().pin_memory() for t in (q, k, v))
        hcu = cu.cpu()
        hout = torch.empty_like(hq_b, pin_memory=True)

        def e2e_step():
            dq, dk, dv = (t.to(device, non_blocking=True) for t in (hq_b, hk_b, hv_b))
            dcu = hcu.to(device, non_blocking=True)
            out = flash_attn_varlen_func(dq, dk, dv, dcu, dcu, max(lens), max(lens), causal=True)
            hout.copy_(out, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize(device)
        ranks.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        f1.record(stream)
        torch.cuda.synchronize(device)
        e2e_ms = f0.elapsed_time(f1) / args.steps
        h2d = sum(t.numel() * t.element_size() for t in (hq_b, hk_b, hv_b, hcu))
        d2h = hout.numel() * hout.element_size()
    ms, e2e_ms_max = ranks.max([ms_local, e2e_ms if e2e_ms is not None else 0.0])
    e2e = None
    if e2e_ms is not None:
        e2e = {"value": flops_job / (e2e_ms_max * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms_max}

    cpu = None
    if with_cpu and rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle
        from mxflashattn_b200 import synthetic as syn

        sample = [L for L in lens if L <= 1024] or [min(lens)]
        c = syn.varlen_case(args.seed, q_lens=sample, q_heads=HQ, kv_heads=HKV, head_dim=D, dtype="bf16")
        t0 = time.perf_counter()
        oracle.attention_varlen(c.q, c.k, c.v, c.cu_q, c.cu_k, causal=True)
        sec = time.perf_counter() - t0
        sflops = 4 * HQ * D * sum(L * (L + 1) // 2 for L in sample)
        cpu = {"value": sflops / sec / 1e12, "unit": "TFLOP/s", "cores": host_cores(), "kind": "port",
               "sample": f"sequences {sample} of the batch, numpy fp32 oracle on {cpu_model()}"}

    peak, kind = measured_tensor_peak()
    peak_s, kind_s = measured_tensor_peak_sustained()
    per_gpu = flops_rank / (ms_local * 1e-3) / 1e12
    return {
        "metric": "causal varlen prefill forward TFLOP/s (config 5)"
                  + (", KV-head groups split over the ranks" if sharded else ""),
        "value": flops_job / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong" if sharded else "weak",
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "prefill varlen causal (config 5)", "lengths": lens, "hq": hq, "hkv": hkv,
                   "head_dim": D, "flops_per_step": flops_job,
                   "l2": "q/k/v 0.08 GB reused from L2 by design (compute-bound kernel)",
                   "parallelism": (f"KV heads {heads.start}..{heads.stop - 1} on this rank" if sharded
                                   else f"dp{world}")},
        "e2e": e2e,
        "roofline": {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s",
                     "frac": per_gpu / peak, "traffic": None, "peak_source": kind, "kernel": "prefill_tc_kernel",
                     # the launches run back to back for steps x ms_per_step: long loops settle at the power cap,
                     # as the sustained cuBLAS figure does
                     "timed_ms": ms_local * args.steps, "peak_sustained": peak_s,
                     "frac_of_sustained": per_gpu / peak_s, "peak_sustained_source": kind_s},
        "cpu_baseline": cpu, "clocks": clocks.summary(), "gpu_launches": args.steps,
    }


def run_prefill(args):
    """--workload prefill: config 5 as the line's own metric (weak scaling over ranks)."""
    import torch

    world, rank, local = dist_env()
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)
    ranks = Ranks(world, rank, device)
    line = prefill_measure(args, device, ranks, sharded=False, with_cpu=True)
    line["warmup"] = args.warmup
    line["vs_baseline"] = None
    if rank == 0:
        print(json.dumps(line), flush=True)
    ranks.close()


# ------------------------------------------------------- long-context decode

def extra_longctx(args, device, ranks):
    """Config 5 decode: 16384-token contexts, B=8 and B=1, 36 layers.

    N=1: the one-GPU split decode (the baseline the context split is compared
    with).  N>1: each rank holds a page-aligned range of every sequence
    (``context_split.local_view``) and the per-rank (O, LSE) records are
    exchanged once per layer: (a) fused into the kernels over NVLink peer
    memory (``FusedContextParallelDecode``), (b) by one NCCL all-gather plus
    the local merge kernel (``context_parallel_decode``).  Both run as CUDA
    graph replays of the 36-layer step.  Layer 0's merged output and LSE of
    both forms are checked on every rank against a one-GPU decode over the
    whole context; device error flags are read on every rank.
    """
    import torch

    from mxflashattn_b200 import _lib, backend, context_split as cs, synthetic as syn

    world = ranks.world
    scale = D ** -0.5
    peak, kind = measured_peaks()
    res = {"metric": "long-context decode, KV HBM GB/s (config 5: ctx 16384, Hq32/Hk8/D128 bf16)",
           "unit": "GB/s", "layers": args.layers}
    for B in LONG_BATCHES:
        lengths = [LONG_CTX] * B
        full = build_layers(lengths, 90000 + 1000 * B, args.layers, device)  # identical on every rank
        bytes_layer = syn.kv_bytes(lengths, HKV, D)
        entry = {"batch": B, "bytes_per_layer": bytes_layer}
        if world == 1:
            graph, _, (ns, _) = decode_graph(full, device)
            ms = time_graph(graph, args.steps, args.warmup, device, ranks)
            del graph
            us = ms * 1e3 / args.steps / args.layers
            entry.update({"us_per_layer": us, "value": bytes_layer / (us * 1e-6) / 1e9,
                          "frac": bytes_layer / (us * 1e-6) / 1e9 / peak, "num_splits": ns,
                          "form": "one-GPU split decode (single launch per layer)"})
        else:
            locs = []
            for t in full:
                ll, table = cs.local_view(t["cache_seqlens"].cpu().numpy(), t["block_table"].cpu().numpy(), world,
                                          ranks.rank, PS)
                locs.append((torch.from_numpy(ll).to(device), torch.from_numpy(table).to(device)))
            fused = cs.FusedContextParallelDecode(B, HQ, HKV, D, device=device)
            outs_f = [None] * len(full)
            outs_n = [None] * len(full)

            def step_fused():
                for i, t in enumerate(full):
                    outs_f[i] = fused(t["q"], t["k_cache"], t["v_cache"], locs[i][0], locs[i][1], scale)

            def step_nccl():
                for i, t in enumerate(full):
                    outs_n[i] = cs.context_parallel_decode(t["q"], t["k_cache"], t["v_cache"], locs[i][0],
                                                           locs[i][1], scale)

            g_f = capture(step_fused, device)
            launches_fused = fused.launches_per_call  # 1: exchange and merge inside the decode kernel
            ms_f = time_graph(g_f, args.steps, args.warmup, device, ranks)
            g_n = capture(step_nccl, device)
            ms_n = time_graph(g_n, args.steps, args.warmup, device, ranks)
            torch.cuda.synchronize(device)
            # parity of layer 0 against the one-GPU decode over the whole context (eager calls)
            t0 = full[0]
            ref, ref_lse = backend.kvcache_attention(t0["q"], t0["k_cache"], t0["v_cache"], t0["cache_seqlens"],
                                                     t0["block_table"], scale, False, return_lse=True)
            of, lf = fused(t0["q"], t0["k_cache"], t0["v_cache"], locs[0][0], locs[0][1], scale, return_lse=True)
            on, ln = cs.context_parallel_decode(t0["q"], t0["k_cache"], t0["v_cache"], locs[0][0], locs[0][1],
                                                scale, return_lse=True)
            torch.cuda.synchronize(device)
            err_f = float((of.float() - ref.float()).abs().max())
            err_n = float((on.float() - ref.float()).abs().max())
            lerr_f = float((lf.reshape(-1) - ref_lse.reshape(-1)).abs().max())
            lerr_n = float((ln.reshape(-1) - ref_lse.reshape(-1)).abs().max())
            flags = float(_lib.read_error_flags())
            del g_f, g_n
            fused.close()
            ms_f, ms_n, err_f, err_n, lerr_f, lerr_n, flags = ranks.max([ms_f, ms_n, err_f, err_n, lerr_f, lerr_n,
                                                                          flags])
            us_f = ms_f * 1e3 / args.steps / args.layers
            us_n = ms_n * 1e3 / args.steps / args.layers
            entry.update({
                "us_per_layer_fused": us_f, "us_per_layer_nccl": us_n,
                "value": bytes_layer / (us_f * 1e-6) / 1e9,
                "value_nccl": bytes_layer / (us_n * 1e-6) / 1e9,
                "frac_of_n_gpu_peak": bytes_layer / (us_f * 1e-6) / 1e9 / (peak * world),
                "max_abs_err_fused": err_f, "max_abs_err_nccl": err_n,
                "lse_err_fused": lerr_f, "lse_err_nccl": lerr_n,
                "tolerance": {"out": 1e-2, "lse": 1e-3, "against": "one-GPU decode over the whole context"},
                "parity_ok": bool(max(err_f, err_n) <= 1e-2 and max(lerr_f, lerr_n) <= 1e-3 and flags == 0),
                "device_flags": int(flags),
                "form": ("decode with the (O, LSE) exchange over NVLink peer stores and the merge in one kernel"
                         if launches_fused == 1 else "decode with the exchange over NVLink peer stores + merge kernel")
                        + " vs NCCL all-gather + merge kernel, CUDA graph replay",
                "gpu_launches_fused": args.steps * args.layers * launches_fused,
            })
        res[f"b{B}"] = entry
        del full
        torch.cuda.empty_cache()
    return res


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill":
        run_prefill(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
