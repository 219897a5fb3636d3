#!/usr/bin/env python
"""Throughput of the bge-large-shaped encoder forward on B200: sentences/s.

One step = one forward pass (embed+LN, 24 post-LN layers, CLS pooling + L2) over
the rank's slice of a batch of 256 sentences with lognormal lengths (median 96,
sigma 0.6, truncated to [8, 512]), packed without padding.  With N GPUs
(torchrun, one process per GPU) the global batch is 256*N sentences (the 256 lengths
N times, fresh ids), sorted by length and cut into N contiguous slices of equal
estimated time (fe_plan_shards: projection FLOPs plus a per-tile attention cost):
replica data parallelism with no collective on the data path (weak scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload bge-large|bge-small|bge-base|qwen3-0.6b|gemma-300m]

Prints one JSON line on rank 0.  `value` is device-timed with inputs resident in
HBM; `e2e` goes through the C ABI's host-buffer entry point (H2D of the ids and
D2H of the embeddings inside the timed region).  `--impl reference` times the
reference's own CPU ops (oracle/_ref, compiled from the reference sources) with all
host threads on a stratified sample of the same workload: every 16th sentence of the
length-sorted batch, the longest included, each timed on its own thread.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from fastembed_b200 import workload as W  # noqa: E402

METRIC = "sentences/s bge-large b=256 L=512 @1/2/4/8 B200; attn+GEMM % TC peak"
UNIT = "sentences/s"
WORKLOAD = "bge-large"
# --workload: the headline bge-large shape (default), the bge-small / bge-base shapes, or
# the Qwen3 / Gemma3 shapes, which the reference has no path for (no CPU baseline)
DESCRIPTIONS = {
    "bge-small": "bge-small shape (4L, D512, 8x64 heads, F2048 GELU, post-LN, CLS+L2), 8 sentences per GPU, "
                 "lengths U[16,128], packed without padding, seeded N(0,0.02) weights",
    "bge-base": "bge-base shape (12L, D768, 12x64 heads, F3072 GELU, post-LN, CLS+L2), 64 sentences per GPU, "
                "lengths U[32,512], packed without padding, seeded N(0,0.02) weights",
    "bge-large": "bge-large shape (24L, D1024, 16x64 heads, F4096 GELU, post-LN, CLS+L2), 256 sentences per GPU, "
                 "lognormal lengths median 96 sigma 0.6 in [8,512], packed without padding, seeded N(0,0.02) weights",
    "qwen3-0.6b": "Qwen3-0.6B shape (28L, D1024, 16q/8kv x 128 heads, vocab 151669, causal, RoPE 1e6, F3072 SwiGLU, "
                  "pre-RMSNorm, last-token+L2), 128 sentences per GPU, lengths U[64,1024], packed, seeded N(0,0.02) "
                  "weights rounded to bf16",
    "gemma-300m": "Gemma-300M shape (24L, D768, 3q/1kv x 256 heads, bidirectional, RoPE 1e4/1e6, F1152 GeGLU, "
                  "sandwich RMSNorm, mean+L2), 512 sentences per GPU, lengths U[8,256], packed, seeded N(0,0.02) "
                  "weights",
}


def metric_name(workload):
    return METRIC if workload == WORKLOAD else f"sentences/s {workload} @1/2/4/8 B200"


def workload_shape(name):
    return W.SHAPES[name] if name in W.SHAPES else W.RMS_SHAPES[name]


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ------------------------------------------------------------------ workload
def global_batch(shape, world, per_gpu=None):
    """The batch of `world` GPUs: the per-GPU length sample taken `world` times (so every N
    runs the same length mix and the same work per GPU), with fresh token ids throughout;
    sorted by length, longest first."""
    if hasattr(shape, "family"):
        lengths = np.tile(W.sample_rms_lengths(shape, batch=per_gpu or shape.batch, seed=1), world)
        ids = W.sample_rms_ids(shape, lengths, seed=1)
    else:
        lengths = np.tile(W.sample_lengths(shape, batch=per_gpu or shape.batch, seed=1), world)
        ids, _ = W.sample_ids(shape, lengths, seed=1, pad_to=int(lengths.max()))
    order = np.argsort(-lengths, kind="stable")
    return lengths[order], ids[order]


def rank_slice(shape, lengths_sorted, world, rank):
    from fastembed_b200 import ops
    cuts = ops.plan_shards(shape, lengths_sorted, world) if world > 1 else []
    bounds = [0] + cuts + [lengths_sorted.size]
    return bounds[rank], bounds[rank + 1]


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(str(g) for g in self.gpus), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        if self.path and os.path.exists(self.path):
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        smax = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ CPU side
def cpu_plan(shape, lengths_sorted, cores):
    """The stratified sample the CPU legs time: every `stride`-th sentence of the
    length-sorted batch, longest first (so the longest sentence is always in it), with
    at least one sentence per host thread (16 at the least, 64 at most).  `depth` is
    how many encoder layers each sampled sentence runs: all of them when the longest
    sampled sentence takes under ~8 s at the reference's ~2 GFLOP/s per core, else one
    (every layer has the same shapes, so the per-layer time scales by the depth)."""
    n = lengths_sorted.size
    want = min(64, max(16, cores))
    stride = max(1, n // want)
    pick = np.arange(0, n, stride)
    longest = shape.flops_per_sentence(int(lengths_sorted[pick].max())) if pick.size else 0.0
    depth = shape.layers if longest <= 8 * 2e9 else 1
    return pick, stride, depth


def _time_sentences(model, ids, lens, kind, threads):
    """Per-sentence wall times of the reference's single-sentence forward, `threads`
    sentences in flight at once (one per host thread, longest first)."""
    from concurrent.futures import ThreadPoolExecutor

    def one(i):
        t0 = time.perf_counter()
        model.forward(ids[i, :int(lens[i])], kind=kind)  # ctypes releases the GIL
        return time.perf_counter() - t0

    with ThreadPoolExecutor(max_workers=threads) as ex:
        return np.array(list(ex.map(one, range(lens.size))), dtype=np.float64)


def run_cpu_reference(shape, lengths_sorted, ids_sorted, weights, steps, warmup, single_thread=False):
    """Times the reference's own CPU forward (oracle/_ref: its src/ops/cpu ops driven by
    the restated bge_forward) on the stratified sample of cpu_plan, all host threads busy.

    Each sampled sentence stands for `stride` sentences of the batch, and a sample run
    at depth d < layers stands for layers / d times its time.  The whole batch's CPU
    time is therefore estimated as stride * (layers / d) * sum(per-sentence times), and
    sentences/s on T threads as batch * T / that (sentences are independent, so T
    threads share a batch of hundreds of sentences evenly).  With `single_thread` the
    sample also runs once on one thread, for the reference's own serial encode_batch
    (src/sentence_transformers_impl.cpp:359-365)."""
    import dataclasses
    from oracle import oracle as O
    kind = "ref" if O.available("ref") else "port"
    cores = os.cpu_count() or 1
    pick, stride, depth = cpu_plan(shape, lengths_sorted, cores)
    model = O.Model(dataclasses.replace(shape, layers=depth), weights)
    ids = np.ascontiguousarray(ids_sorted[pick])
    lens = np.ascontiguousarray(lengths_sorted[pick])
    threads = int(min(cores, lens.size))
    scale = stride * shape.layers / depth
    for _ in range(warmup):
        _time_sentences(model, ids, lens, kind, threads)
    t0 = time.perf_counter()
    per_step = []
    for _ in range(max(1, steps)):
        per_step.append(_time_sentences(model, ids, lens, kind, threads).sum() * scale)
    wall = (time.perf_counter() - t0) / max(1, steps)
    batch = lengths_sorted.size
    cpu_s = float(np.mean(per_step))  # estimated CPU seconds of the whole batch
    sent_s = batch * threads / cpu_s
    depth_txt = f"all {depth}" if depth == shape.layers else f"{depth} of {shape.layers}"
    info = {
        "kind": "reference" if kind == "ref" else "port",
        "cores": threads,
        "sample": (f"{lens.size} sentences, every {stride}th of the {batch}-sentence batch sorted by length "
                   f"(lengths {int(lens.min())}-{int(lens.max())}, the longest included), {depth_txt} layers "
                   f"each, one sentence per thread on {threads} threads, {wall:.1f} s per step; sentences/s = "
                   f"{batch} x {threads} threads / ({stride} x {shape.layers // depth} x the summed "
                   f"per-sentence times)"),
        "batch_cpu_seconds": cpu_s,
        "tokens_per_s": float(lengths_sorted.sum()) * threads / cpu_s,
    }
    if single_thread:
        t1 = _time_sentences(model, ids, lens, kind, 1).sum() * scale
        info["single_thread"] = {"value": batch / t1, "unit": UNIT, "cores": 1,
                                 "tokens_per_s": float(lengths_sorted.sum()) / t1,
                                 "sample": "the same sample run once on one thread"}
    return sent_s, info


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    shape = W.SHAPES[args.workload]
    lengths, ids = global_batch(shape, 1, args.batch)
    weights = W.make_weights(shape)
    steps, warmup = args.steps, args.warmup
    value, info = run_cpu_reference(shape, lengths, ids, weights, steps, warmup, single_thread=True)
    line = {
        "impl": "reference", "metric": metric_name(args.workload), "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": steps, "warmup": warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": DESCRIPTIONS[args.workload], "global_batch": int(lengths.size),
                   "valid_tokens_per_step": int(lengths.sum()), "tokens_per_s": info["tokens_per_s"],
                   "parallelism": f"{info['cores']} host threads, one sentence per thread"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": info["cores"], "kind": info["kind"],
                         "sample": info["sample"], "single_thread": info["single_thread"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU arm
def ours(args):
    import torch
    import torch.distributed as dist
    from fastembed_b200 import ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    shape = workload_shape(args.workload)
    rms = hasattr(shape, "family")
    lengths_all, ids_all = global_batch(shape, world, args.batch)
    lo, hi = rank_slice(shape, lengths_all, world, rank)
    lengths = np.ascontiguousarray(lengths_all[lo:hi])
    ids = np.ascontiguousarray(ids_all[lo:hi])
    weights = W.make_rms_weights(shape) if rms else W.make_weights(shape)
    eng = ops.Engine(shape, local)
    eng.load_weights(weights)

    packed, cu = ops.pack(ids, lengths)
    ids_dev = torch.tensor(packed, device=dev)
    cu_dev = torch.tensor(cu, device=dev)
    out = torch.empty(lengths.size, shape.hidden, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    tokens_local = int(lengths.sum())

    def step():
        eng.encode_packed(ids_dev, cu_dev, cu, out=out, stream=stream)

    # ---- device-timed region, inputs resident in HBM
    for _ in range(args.warmup):
        step()
    barrier()
    clocks = ClockSampler([local] if world == 1 else list(range(world)))
    clocks.__enter__()  # sampled through the timed and end-to-end regions (both under load)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    e1.synchronize()
    barrier()
    elapsed_ms = max_over_ranks(e0.elapsed_time(e1))
    launches = sum_over_ranks(float(eng.stats()["launches"] * args.steps))

    sentences = sum_over_ranks(float(lengths.size))
    tokens = sum_over_ranks(float(tokens_local))
    ms_per_step = elapsed_ms / args.steps
    value = sentences / (ms_per_step / 1e3)

    # ---- end to end through the host-buffer C ABI entry point
    for _ in range(max(1, args.warmup // 2)):
        eng.encode_host(ids, lengths)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.encode_host(ids, lengths)
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    clocks.__exit__(None, None, None)
    clock_info = clocks.summary() if rank == 0 else None
    e2e_value = sentences * args.steps / e2e_s
    h2d = sum_over_ranks(float(tokens_local * 4 + (lengths.size + 1) * 4))
    d2h = sum_over_ranks(float(lengths.size * shape.hidden * 4))

    # ---- per-kernel device time (CUDA events around every launch, same stream), same K steps
    eng.set_profiling(True)
    gemm_ms = attn_ms = other_ms = 0.0
    for _ in range(args.steps):
        step()
        st = eng.stats()
        gemm_ms += st["gemm_ms"]
        attn_ms += st["attention_ms"]
        other_ms += st["other_ms"]
    eng.set_profiling(False)
    st = eng.stats()
    gemm_flops = st["gemm_flops"]
    attn_flops = st["attention_flops"]
    gemm_ms = max_over_ranks(gemm_ms)
    attn_ms = max_over_ranks(attn_ms)
    other_ms = max_over_ranks(other_ms)
    hbm_gbs, burst_tf, sustained_tf, peak_kind = peaks()
    gemm_tflops = gemm_flops * args.steps / (gemm_ms / 1e3) / 1e12 if gemm_ms else 0.0
    attn_tflops = attn_flops * args.steps / (attn_ms / 1e3) / 1e12 if attn_ms else 0.0
    # attention is HBM-bound at these lengths: its algorithmic bytes are one read of Q, K, V
    # and one write of O per layer, all bf16
    if rms:  # Q, K, V and O of every head, bf16
        attn_bytes = shape.layers * tokens_local * (2 * shape.q_heads + 2 * shape.kv_heads) * shape.head_dim * 2
    else:
        attn_bytes = shape.layers * tokens_local * 4 * shape.hidden * 2
    attn_gbs = attn_bytes * args.steps / (attn_ms / 1e3) / 1e9 if attn_ms else 0.0

    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not rms:
        v, info = run_cpu_reference(shape, lengths_all, ids_all, weights, steps=1, warmup=0)
        cpu_base = {"value": v, "unit": UNIT, "cores": info["cores"], "kind": info["kind"], "sample": info["sample"]}

    if rank == 0:
        traffic = None
        tpath = os.path.join(ROOT, "profiles", "projections_bge-large.md")
        if os.path.exists(tpath) and args.workload == "bge-large":
            with open(tpath) as f:
                for ln in f:
                    if ln.startswith("traffic_bytes_per_launch:"):
                        traffic = int(ln.split(":")[1])
        line = {
            "metric": metric_name(args.workload),
            "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": DESCRIPTIONS[args.workload],
                       "global_batch": int(sentences), "valid_tokens_per_step": int(tokens),
                       "tokens_per_s": tokens / (ms_per_step / 1e3),
                       "parallelism": f"replica dp{world}, cost-balanced contiguous slices of the length-sorted batch, "
                                      "no collective",
                       "l2": "inputs larger than L2: the bf16 weights and the activations of a step are each "
                             "several times the 126 MB L2"},
            "roofline": {"bound": "tensor",
                         "kernel": "tcgen05 projection GEMMs: linear_tcgen05_pair (QKV, FFN1), linear_ln_cluster "
                                   "(out-proj + LN), linear_ln_tcgen05_pair (FFN2 + LN)",
                         "achieved": gemm_tflops, "peak": burst_tf, "unit": "TFLOP/s",
                         "frac": gemm_tflops / burst_tf, "peak_kind": f"bf16 burst, {peak_kind}",
                         "frac_of_sustained": gemm_tflops / sustained_tf,
                         "traffic": traffic,
                         "traffic_note": "DRAM bytes per launch, mean of one layer's four projection launches "
                                         "(ncu, profiles/projections_bge-large.md)",
                         "gemm_flops_per_step": gemm_flops, "gemm_ms_per_step": gemm_ms / args.steps,
                         "attention": {"bound": "hbm", "achieved": attn_gbs, "peak": hbm_gbs, "unit": "GB/s",
                                       "frac": attn_gbs / hbm_gbs, "tflops": attn_tflops,
                                       "tensor_frac": attn_tflops / burst_tf,
                                       "ms_per_step": attn_ms / args.steps, "flops_per_step": attn_flops,
                                       "bytes_per_step": attn_bytes},
                         "other_ms_per_step": other_ms / args.steps,
                         "profiled_ms_per_step": (gemm_ms + attn_ms + other_ms) / args.steps},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": int(launches),
            "clocks": clock_info,
            "cpu_baseline": cpu_base,
            **({"cpu_baseline_note": "the reference has no Qwen3 / Gemma3 forward"} if rms else {}),
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None, help="sentences per GPU (default: the workload's)")
    ap.add_argument("--workload", choices=sorted(DESCRIPTIONS), default=WORKLOAD,
                    help="bge-large (the headline), bge-small / bge-base, or the Qwen3 / Gemma3 shapes")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        if args.workload not in W.SHAPES:
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference has no Qwen3 / Gemma3 forward"}))
            return 0
        return reference_arm(args)
    return ours(args)


if __name__ == "__main__":
    sys.exit(main())
