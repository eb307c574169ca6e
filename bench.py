#!/usr/bin/env python3
"""Benchmark of the quantized-expert hot path (BASELINE config 1 workload).

A step = one decode token through a ring of L (default 30, the model depth)
distinct, HBM-resident config-1 MoE FFN layers: int8 router (128 experts x
2816) -> softmax top-8 -> 8 routed int4 g64 experts (gate/up 704x2816, GELU,
down 2816x704) + int4 shared expert (2112) -> weighted sum.  The layers'
weights (~13 GB) never fit in L2 (126 MB), so every step streams its bytes
from HBM; the step's tokens come from a ring of 8 input sets so routing
varies from step to step.

value  : algorithmic HBM bytes of the step / device time (GB/s), inputs resident.
e2e    : same metric through the public C ABI call with host buffers: the
         step's inputs are copied H2D from pinned memory and its outputs D2H
         inside the timed region.
tok_s  : decode tokens per second through the L MoE layers (whole job).

`--impl reference` times the reference's CPU math (the C oracle port of its
validation references; the Swift/Metal original cannot run on Linux) on the
host cores for the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "int4 expert GEMV HBM GB/s vs peak; MoE decode tok/s at 1/2/4/8 B200"
D, F, FS, E, TOPK = 2816, 704, 2112, 128, 8


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0,
                    help="timed steps (default per workload: a timed region of about half a second)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=30)
    ap.add_argument("--ring", type=int, default=8)
    ap.add_argument("--scale-dtype", choices=["bf16", "f16"], default=None,
                    help="scale/bias storage; default fp16 for config 0 (as BASELINE states it), else bf16")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemv", action="store_true", help="decode: skip the config-0 GEMV sub-record")
    ap.add_argument("--no-stack", action="store_true", help="moe: skip the full decoder-stack sub-record")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="expert-parallel exchange at N > 1: peer-memory stores (default) or NCCL all-to-alls")
    ap.add_argument("--overlap-shared", type=int, default=1,
                    help="moe: run each layer's shared expert on a forked stream beside the routed path (1) or after it (0)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--workload", choices=["moe", "decode", "gemv", "batched", "prefill", "ep", "attention"],
                    default="moe",
                    help="moe (default) = config-4 MoE decode step at batch 256/32/1 through 30 layers, experts "
                         "sharded over the GPUs (plus, on one GPU, the batch-1 roofline and the config-0 GEMV); "
                         "decode = config 1 (batch 1, GB/s); gemv = config 0 (int4 GEMV 1408x2816 streamed from "
                         "HBM); batched = config 2 (64 tokens); prefill = config 3 (4096 tokens); ep = one layer "
                         "of the expert-parallel batch; attention = config-4 decode attention of one layer "
                         "(--tokens sequences, default 32, over a 4096-token fp16 KV cache)")
    ap.add_argument("--matrices", type=int, default=256, help="gemv: distinct weight matrices per step")
    ap.add_argument("--tokens", type=int, default=0, help="override the chunk's token count (batched/prefill)")
    return ap.parse_args()


# ---------------------------------------------------------------- clocks ----
class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi takes a few hundred ms to start: wait (up to 3 s) for its first
            # sample, so even a short timed region is covered
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0 and self.proc.poll() is None:
                time.sleep(0.01)
            self.lines.clear()  # that sample predates the timed region; later ones arrive every 20 ms
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- CPU arm ---
def host_threads() -> int:
    """All host threads this process may use (torchrun sets OMP_NUM_THREADS=1
    per rank; the CPU baseline passes its thread count explicitly instead)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1

def cpu_model() -> str:
    """The host CPU's model name (the `lscpu` "Model name" line)."""
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_sample(seconds: float, label: str = "cpu", threads: int | None = None):
    """Oracle port of the reference CPU math on the host cores: router + top-8
    + 8 routed experts + shared expert for one token of one config-1 layer,
    repeated for ~`seconds`.  Returns (layer-tokens/s, threads, sample text)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np

    import oracle as O
    threads = threads or host_threads()
    rng = O.seed_tree(0, f"bench-{label}")
    W8, S8, B8 = rng.synthetic_affine(E, D, 8, 0)
    es = O.bf16_bits(np.full(D, D ** -0.5, np.float32))
    pes = O.bf16_bits(np.ones(E, np.float32))
    experts = [[rng.synthetic_affine(F, D, 4, 0), rng.synthetic_affine(F, D, 4, 0), rng.synthetic_affine(D, F, 4, 0)]
               for _ in range(TOPK)]
    blobs, offs = [], None
    for g, u, dn in experts:
        parts = [*g, *u, *dn]
        chunks, cur, o = [], 0, []
        for p in parts:
            b = np.ascontiguousarray(p).view(np.uint8).reshape(-1)
            o.append(cur)
            chunks.append(b)
            cur += (b.size + 15) // 16 * 16
            chunks.append(np.zeros((b.size + 15) // 16 * 16 - b.size, np.uint8))
        blobs.append(np.concatenate(chunks))
        offs = O.Offsets(*o)
    sg, su, sd = rng.synthetic_affine(FS, D, 4, 0), rng.synthetic_affine(FS, D, 4, 0), rng.synthetic_affine(D, FS, 4, 0)
    xs = [rng.normal_f16(D) for _ in range(4)]
    n = 0
    t0 = time.perf_counter()
    while True:
        x = xs[n % len(xs)]
        l32, _ = O.router_logits(W8, S8, B8, x, es)
        idx, w16, _ = O.router_topk(l32, pes, TOPK)
        acts = O.moe_phase1(blobs, offs, x, D, F, 0, threads)   # the 8 selected experts
        O.moe_phase2(blobs, offs, acts, w16, None, D, F, 0, threads)
        O.shared_expert(sg, su, sd, x, D, FS, 4, 0, threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return n / el, threads, f"{n} config-1 layer-tokens (router 128x2816 int8 + 8 routed + shared int4) in {el:.1f} s"


def layer_bytes():
    from edgeexpert_b200.format import moe_layer_bytes
    return moe_layer_bytes(D, F, FS, E, TOPK, 4)


def run_reference(a, rank):
    if rank != 0:
        return
    if a.workload == "gemv":
        gps, threads, sample = gemv_cpu_sample(max(5.0, a.cpu_seconds))
        v = gps * G_BYTES / 1e9
        print(json.dumps({"metric": "int4 g64 GEMV HBM GB/s (config 0)", "value": v, "unit": "GB/s",
                          "impl": "reference", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
                          "ms_per_step": 1e3 * a.matrices / gps, "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "f32-acc/int4", "data": "synthetic (BASELINE config 0)",
                          "config": {"workload": "config0 int4 GEMV 1408x2816", "matrices": a.matrices},
                          "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                                           "sample": sample},
                          "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return
    if a.workload == "moe":
        rec = cpu_baseline_record(lambda sec, th: cpu_sample(sec, "reference", th), 1e9 / a.layers,
                                  max(10.0, a.cpu_seconds), unit="tok/s")
        v = rec["value"]
        B = a.tokens or MOE_BATCHES[0]
        rec["sample"] += f"; tok/s = layer-tokens/s / {a.layers} layers"
        print(json.dumps({
            "metric": METRIC, "value": v, "unit": "tok/s", "impl": "reference", "n_gpus": a.gpus, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": B / v * 1e3, "tok_s": v, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32-acc/int4",
            "data": "synthetic (BASELINE config-1 distributions, SplitMix64 seed 0)",
            "config": {"workload": f"config-4 MoE decode step: batch {B} through {a.layers} config-1 MoE layers "
                                   "(the reference's per-token CPU math, oracle port)", "global_batch": B,
                       "layers": a.layers},
            "cpu_baseline": rec,
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)
        return
    lps, threads, sample = cpu_sample(max(5.0, a.cpu_seconds), "reference")
    if a.workload != "decode":
        T = a.tokens or CHUNK_TOKENS[a.workload]
        step_s = T / lps
        if a.workload == "prefill":
            metric, unit, v = "MoE prefill TFLOP/s (config 3)", "TFLOP/s", chunk_flops(T) / step_s / 1e12
        else:
            # a CPU reads the weights of every routed expert the chunk hits; count all 128 (64 tokens x top-8
            # over 128 experts hits nearly every expert)
            metric, unit, v = "MoE batched-decode weight GB/s (config 2)", "GB/s", chunk_bytes(E) / step_s / 1e9
        line = {"metric": metric, "value": v, "unit": unit, "impl": "reference", "n_gpus": a.gpus, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": step_s * 1e3, "tok_s": lps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32-acc/int4",
                "data": "synthetic (BASELINE distributions, SplitMix64 seed 0)",
                "config": {"workload": f"{T}-token chunk through the config-1 MoE layer", "tokens": T},
                "cpu_baseline": {"value": v, "unit": unit, "cores": threads, "kind": "port",
                                 "sample": sample + f"; scaled to a {T}-token chunk"},
                "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    per_layer_b = layer_bytes()
    gbs = lps * per_layer_b / 1e9
    line = {
        "metric": METRIC, "value": gbs, "unit": "GB/s", "impl": "reference", "n_gpus": a.gpus, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": 1e3 * a.layers / lps, "tok_s": lps / a.layers,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32-acc/int4",
        "data": "synthetic (BASELINE config-1 distributions, SplitMix64 seed 0)",
        "config": {"workload": f"config1 MoE decode layer x{a.layers} layers, batch 1", "d": D, "f": F, "fs": FS,
                   "experts": E, "top_k": TOPK, "layers": a.layers},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm ---
def run_ours(a, rank, world, local_rank, emit: bool = True, layers=None):
    """Config 1: batch-1 decode through `--layers` distinct MoE layers (GB/s).
    `layers` reuses already-built layer weights."""
    import torch
    import torch.distributed as dist

    from edgeexpert_b200._lib import Context
    from edgeexpert_b200.format import synthetic_moe_layer
    from edgeexpert_b200.moe import MoE, moe_decode_layer

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    ctx = Context.get(local_rank)
    sdt = torch.bfloat16 if a.scale_dtype == "bf16" else torch.float16
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    if layers is None:
        layers = [synthetic_moe_layer(D, F, FS, E, TOPK, 4, sdt, dev, gen) for _ in range(a.layers)]
    c_layers = [L.as_c() for L in layers]
    L, R = len(layers), a.ring
    x_ring = torch.randn(R, L, D, device=dev, generator=gen).to(torch.float16)
    y = torch.empty(L, D, dtype=torch.float16, device=dev)
    ids = torch.empty(L, TOPK, dtype=torch.int32, device=dev)
    wts = torch.empty(L, TOPK, dtype=torch.float16, device=dev)
    x_in = torch.empty(L, D, dtype=torch.float16, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(xs, s):
        for l in range(L):
            moe_decode_layer(layers[l], xs[l], xs[l], y[l], out_indices=ids[l], out_weights=wts[l], stream=s,
                             context=ctx, c_layer=c_layers[l])

    # eager warm-up (sets kernel attributes), then one graph per ring slot + one for x_in
    with torch.cuda.stream(stream):
        step(x_ring[0], stream)
    torch.cuda.synchronize()
    graphs = []
    for r in range(R + 1):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(x_ring[r] if r < R else x_in, stream)
        graphs.append(g)
    torch.cuda.synchronize()
    launches_per_step = 3 * L

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing
    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            graphs[i % R].replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for i in range(a.steps):
            graphs[i % R].replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / a.steps)
    clk = clocks.stop()

    # ---- end to end through the C ABI with host buffers
    h_in = torch.empty(R, L, D, dtype=torch.float16, pin_memory=True)
    h_in.copy_(x_ring.cpu())
    h_out = torch.empty(L, D, dtype=torch.float16, pin_memory=True)
    h_ids = torch.empty(L, TOPK, dtype=torch.int32, pin_memory=True)
    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            x_in.copy_(h_in[i % R], non_blocking=True)
            graphs[R].replay()
            h_out.copy_(y, non_blocking=True)
            h_ids.copy_(ids, non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(a.steps):
            x_in.copy_(h_in[i % R], non_blocking=True)
            graphs[R].replay()
            h_out.copy_(y, non_blocking=True)
            h_ids.copy_(ids, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    h2d = L * D * 2
    d2h = L * D * 2 + L * TOPK * 4

    # ---- roofline of the dominant kernel: phase 1 (routed gate/up of 8
    # experts + shared gate/up), timed alone over the L layers' saved routing
    moe = MoE(ctx)
    acts = torch.empty(L, TOPK * F, dtype=torch.float16, device=dev)
    from edgeexpert_b200.format import affine_bytes
    p1_bytes = TOPK * 2 * affine_bytes(F, D) + D * 2  # routed gate+up of 8 experts + x
    with torch.cuda.stream(stream):
        graphs[0].replay()
        for l in range(L):
            moe.encode_routed_phase1(layers[l].experts, x_ring[0][l], acts[l], D, F, TOPK, expert_ids=ids[l],
                                     stream=stream)
        pg = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.graph(pg, stream=stream):
        for l in range(L):
            moe.encode_routed_phase1(layers[l].experts, x_ring[0][l], acts[l], D, F, TOPK, expert_ids=ids[l],
                                     stream=stream)
    with torch.cuda.stream(stream):
        for _ in range(3):
            pg.replay()
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    with torch.cuda.stream(stream):
        p0.record(stream)
        for _ in range(reps):
            pg.replay()
        p1.record(stream)
    torch.cuda.synchronize()
    p1_us = p0.elapsed_time(p1) * 1e3 / (reps * L)
    ctx.check_device(stream)

    peaks = {}
    pk_path = ROOT / "MEASURED_PEAKS.json"
    if pk_path.exists():
        peaks = json.loads(pk_path.read_text())
    peak, peak_src = (peaks["hbm_gbs"], "measured") if "hbm_gbs" in peaks else (6650.0, "fallback")
    achieved = p1_bytes / (p1_us * 1e-6) / 1e9
    traffic = None
    tr_path = ROOT / "profiles" / "moe_phase1_traffic.json"
    if tr_path.exists():
        traffic = json.loads(tr_path.read_text()).get("bytes_per_launch")

    per_step_bytes = L * layer_bytes()
    value = world * per_step_bytes / (ms * 1e-3) / 1e9
    e2e_value = world * per_step_bytes / (ms_e2e * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline_record(lambda sec, th: cpu_sample(sec, "cpu", th), layer_bytes(),
                                  a.cpu_seconds if emit else min(a.cpu_seconds, 8.0))

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16-act/int4-w/fp32-acc",
            "data": "synthetic (BASELINE config-1 distributions, random-init weights, device RNG)",
            "config": {"workload": f"config1 MoE decode layer x{L} distinct layers (one token), batch 1",
                       "d": D, "f": F, "fs": FS, "experts": E, "top_k": TOPK, "layers": L,
                       "scale_dtype": a.scale_dtype, "parallelism": f"replicas{world}" if world > 1 else "1gpu",
                       "l2": "weights per step (%.2f GB) exceed L2 (126 MB); no flush needed" %
                             (per_step_bytes / 1e9)},
            "tok_s": world * 1e3 / ms, "tok_s_e2e": world * 1e3 / ms_e2e,
            "bytes_per_step_per_gpu": per_step_bytes,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "hbm", "kernel": "engine_kernel<Phase1Policy> (routed gate/up, 8 experts)",
                         "achieved": achieved, "peak": peak, "peak_source": f"{peak_src} hbm_gbs", "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "bytes_per_launch": p1_bytes,
                         "us_per_launch": p1_us},
            "cpu_baseline": cpu,
            "clocks": clk,
            "gpu_launches": launches_per_step * a.steps,
        }
        if emit:
            print(json.dumps(line), flush=True)
        return line


# --------------------------------------------------------- config 0 GEMV ----
G_M, G_N = 1408, 2816
G_BYTES = G_M * G_N // 2 + 2 * G_M * (G_N // 64) * 2 + G_N * 2 + G_M * 2  # 2,238,720 B (W + s/b + x + y)


def gemv_cpu_sample(seconds: float, threads: int | None = None):
    """Oracle port of the reference's int4 GEMV (kernel order) on the host cores."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    threads = threads or host_threads()
    rng = O.seed_tree(0, "bench-gemv")
    W, S, B = rng.synthetic_affine(G_M, G_N, 4, 1)
    x = rng.normal_f16(G_N)
    n, t0 = 0, time.perf_counter()
    while True:
        O.int4_gemv_kernel_order(W, S, B, x, 1, threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return n / el, threads, f"{n} config-0 GEMVs (1408x2816 int4 g64, fp16 scales) in {el:.1f} s"


def cpu_baseline_record(sampler, unit_bytes: float, seconds: float, unit: str = "GB/s") -> dict:
    """The oracle port timed twice on the host: one thread, then every host
    thread; `value` is the all-thread figure.  sampler(seconds, threads)
    returns (units/s, threads, sample text); unit_bytes scales units to bytes."""
    half = max(2.0, seconds / 2)
    u1, _, s1 = sampler(half, 1)
    un, thr, sn = sampler(half, host_threads())
    return {"value": un * unit_bytes / 1e9, "unit": unit, "cores": thr, "kind": "port",
            "sample": f"all threads: {sn}; 1 thread: {s1}",
            "single_thread": {"value": u1 * unit_bytes / 1e9, "unit": unit, "cores": 1},
            "cpu_model": cpu_model()}


def run_gemv(a, rank, world, local_rank, emit: bool = True):
    """Config 0: the int4 g64 GEMV 1408x2816 over `--matrices` distinct,
    HBM-resident weight matrices (> L2 in total), one batched launch per step."""
    import torch
    import torch.distributed as dist

    from edgeexpert_b200._lib import Context
    from edgeexpert_b200.format import synthetic_affine
    from edgeexpert_b200.quant import DequantInt4GEMV, affine_gemv_batched

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    ctx = Context.get(local_rank)
    sdt = torch.bfloat16 if a.scale_dtype == "bf16" else torch.float16
    gen = torch.Generator(device=dev)
    gen.manual_seed(77 + rank)
    R = a.matrices
    W, S, B = synthetic_affine(R * G_M, G_N, 4, sdt, dev, gen)
    x = torch.randn(G_N, device=dev, generator=gen).to(torch.float16)
    y = torch.empty(R, G_M, dtype=torch.float16, device=dev)
    stream = torch.cuda.Stream(device=dev)
    wstride, sbstride = G_M * G_N // 2, G_M * (G_N // 64)

    def step(s, xx):
        affine_gemv_batched(W, S, B, xx, y, bits=4, m=G_M, n=G_N, batch=R, w_stride_bytes=wstride,
                            sb_stride=sbstride, y_batch_stride=G_M, stream=s, context=ctx)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    x_in = torch.empty_like(x)
    with torch.cuda.stream(stream):
        step(stream, x)
    torch.cuda.synchronize()
    g, g_in = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step(stream, x)
    with torch.cuda.graph(g_in, stream=stream):
        step(stream, x_in)
    with torch.cuda.stream(stream):
        for _ in range(a.warmup):
            g.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(a.steps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    clk = clocks.stop()

    # end to end: x H2D (pinned) and every y D2H each step
    h_x = torch.empty(G_N, dtype=torch.float16, pin_memory=True)
    h_x.copy_(x.cpu())
    h_y = torch.empty(R, G_M, dtype=torch.float16, pin_memory=True)
    with torch.cuda.stream(stream):
        for _ in range(a.warmup):
            x_in.copy_(h_x, non_blocking=True)
            g_in.replay()
            h_y.copy_(y, non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        for _ in range(a.steps):
            x_in.copy_(h_x, non_blocking=True)
            g_in.replay()
            h_y.copy_(y, non_blocking=True)
        f1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = max_over_ranks(f0.elapsed_time(f1) / a.steps)

    # single-GEMV latency through DequantInt4GEMV.encode (one launch per matrix)
    q = DequantInt4GEMV(ctx)
    gs = torch.cuda.CUDAGraph()
    nl = min(R, 64)
    with torch.cuda.stream(stream):
        q.encode(W[:G_M], S[:G_M], B[:G_M], x, y[0], G_M, G_N, stream=stream)
    torch.cuda.synchronize()
    with torch.cuda.graph(gs, stream=stream):
        for i in range(nl):
            q.encode(W[i * G_M:(i + 1) * G_M], S[i * G_M:(i + 1) * G_M], B[i * G_M:(i + 1) * G_M], x, y[i], G_M, G_N,
                     stream=stream)
    with torch.cuda.stream(stream):
        gs.replay()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        s0.record(stream)
        gs.replay()
        s1.record(stream)
    torch.cuda.synchronize()
    single_us = s0.elapsed_time(s1) * 1e3 / nl
    ctx.check_device(stream)

    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak, src = (peaks["hbm_gbs"], "measured hbm_gbs") if "hbm_gbs" in peaks else (6650.0, "fallback")
    per_step = R * G_BYTES
    value = world * per_step / (ms * 1e-3) / 1e9
    achieved = per_step / (ms * 1e-3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline_record(gemv_cpu_sample, G_BYTES, a.cpu_seconds if emit else min(a.cpu_seconds, 6.0))
    traffic = None
    tr = ROOT / "profiles" / "gemv_traffic.json"
    if tr.exists():
        traffic = json.loads(tr.read_text()).get("bytes_per_launch")
    if rank == 0:
        line = {
            "metric": "int4 g64 GEMV HBM GB/s (config 0)", "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16-act/int4-w/fp32-acc",
            "data": "synthetic (BASELINE config-0 distributions, random-init weights)",
            "config": {"workload": f"config0: int4 g64 GEMV 1408x2816 over {R} distinct HBM-resident matrices "
                                   "(one batched launch per step)", "matrices": R, "m": G_M, "n": G_N,
                       "scale_dtype": a.scale_dtype,
                       "l2": "%.0f MB of weights per step exceed L2 (126 MB); no flush needed" % (per_step / 1e6)},
            "single_gemv_us": single_us, "single_gemv_gbs": G_BYTES / (single_us * 1e-6) / 1e9,
            "e2e": {"value": world * per_step / (ms_e2e * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": G_N * 2,
                    "d2h_bytes_per_step": R * G_M * 2},
            "roofline": {"bound": "hbm", "kernel": "gemv_stream_kernel (ring-streamed integer GEMV, 16 mma.sync consumer warps)", "achieved": achieved,
                         "peak": peak, "peak_source": src, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": traffic, "bytes_per_launch": per_step, "us_per_launch": ms * 1e3},
            "cpu_baseline": cpu, "clocks": clk, "gpu_launches": a.steps,
        }
        if emit:
            print(json.dumps(line), flush=True)
        return line


# ------------------------------------------------- expert parallel (EP) ----
def run_ep(a, rank, world, local_rank):
    """A decode batch of B tokens (default 256, config 4's largest) through
    one config-1 MoE layer per step, experts sharded E/N per GPU, tokens split
    B/N per GPU (strong scaling: the job is fixed).  Per rank: batched router
    on its tokens, expert-parallel routed experts (NCCL all-to-all dispatch
    and combine), shared expert on its tokens."""
    import torch
    import torch.distributed as dist

    from edgeexpert_b200._lib import Context
    from edgeexpert_b200.ep import ExpertParallelMoE
    from edgeexpert_b200.format import synthetic_moe_layer
    from edgeexpert_b200.moe import ExpertPool
    from edgeexpert_b200.prefill import PrefillRouter, PrefillSharedExpert

    B = a.tokens or 256
    if B % world:
        raise SystemExit(f"--tokens {B} must split over {world} GPUs")
    T = B // world
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    ctx = Context.get(local_rank)
    sdt = torch.bfloat16 if a.scale_dtype == "bf16" else torch.float16
    gen = torch.Generator(device=dev)
    gen.manual_seed(2024)  # identical layer on every rank; each keeps its experts
    nl = 4
    layers, pools = [], []
    per = E // world
    for _ in range(nl):
        L = synthetic_moe_layer(D, F, FS, E, TOPK, 4, sdt, dev, gen)
        L.per_expert_scale.copy_((1.0 + 0.3 * torch.randn(E, device=dev, generator=gen)).abs().to(torch.bfloat16))
        full = L.experts
        blob = full.blob.view(E, -1)[rank * per:(rank + 1) * per].reshape(-1).clone()
        pools.append(ExpertPool(blob, full.stride, per, full.offsets, D, F, full.scale_dtype))
        L.experts = None
        del full
        layers.append(L)
    torch.cuda.empty_cache()
    g2 = torch.Generator(device=dev)
    g2.manual_seed(99 + rank)
    xs = torch.randn(nl, T, D, device=dev, generator=g2).to(torch.float16)
    idx = torch.empty(T, TOPK, dtype=torch.int32, device=dev)
    wts = torch.empty(T, TOPK, dtype=torch.float16, device=dev)
    h2 = torch.empty(T, D, dtype=torch.float16, device=dev)
    acts = torch.empty(T, FS, dtype=torch.float16, device=dev)
    ys = torch.empty(T, D, dtype=torch.float16, device=dev)
    router, shared = PrefillRouter(ctx), PrefillSharedExpert(ctx)
    eps = [ExpertParallelMoE(pools[i], E, TOPK, context=ctx) for i in range(nl)]

    def step(i):
        L, x = layers[i % nl], xs[i % nl]
        router.encode_gemma4_block(L.router_w, L.router_s, L.router_b, x, L.eff_scale, L.per_expert_scale, idx,
                                   wts, T, E, D, TOPK)
        eps[i % nl].forward(x, idx, wts, h2)
        shared.encode(x, L.shared_gate, L.shared_up, L.shared_down, acts, ys, T)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(a.warmup):
        step(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(a.steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    clk = clocks.stop()
    ctx.check_device(None)
    sent = eps[(a.steps - 1) % nl].last.sent
    flops = chunk_flops(B)
    if rank == 0:
        print(json.dumps({
            "metric": "MoE decode tok/s, experts sharded over GPUs (config 4 batch)", "value": B * 1e3 / ms,
            "unit": "tok/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16-act/int4-w/fp32-acc",
            "data": "synthetic (BASELINE distributions, random-init weights)",
            "config": {"workload": f"config-4 decode batch of {B} tokens through one config-1 MoE layer, "
                                   f"{per} routed experts per GPU, {T} tokens per GPU, NCCL all-to-all",
                       "tokens": B, "experts_per_gpu": per, "parallelism": f"ep{world}", "layer_ring": nl,
                       "rank0_sent_pairs_per_rank": sent},
            "tflops": flops / (ms * 1e-3) / 1e12,
            "e2e": None, "roofline": None, "cpu_baseline": None, "clocks": clk,
            "gpu_launches": None,
        }), flush=True)


# ------------------------------------------- MoE decode stack (default) ----
MOE_BATCHES = (256, 32, 1)


def tokens_of(B: int, world: int, rank: int) -> int:
    """Tokens rank `rank` owns of a global decode batch B (DP split)."""
    return B // world + (1 if rank < B % world else 0)


def moe_step_bytes(B: int, world: int, distinct_local: float, L: int) -> float:
    """Algorithmic HBM bytes one GPU reads in one step of a batch-B decode
    through L MoE layers: router + shared expert (replicated) + every local
    routed expert the batch hits, once."""
    from edgeexpert_b200.format import affine_bytes
    expert = 2 * affine_bytes(F, D) + affine_bytes(D, F)
    shared = 2 * affine_bytes(FS, D) + affine_bytes(D, FS)
    router = affine_bytes(E, D, 8)
    return L * (router + shared + distinct_local * expert)


def run_moe(a, rank, world, local_rank):
    """Config-4-shaped decode through `--layers` (30) config-1 MoE layers at
    global batches 256, 32 and 1, experts sharded E/N per GPU and tokens split
    B/N per GPU (strong scaling: the batch is fixed as N grows).  Per layer and
    rank: batched router over its tokens, the routed experts (N=1: device sort
    + grouped int4 GEMMs + token-major reduce; N>1: fixed-capacity NCCL
    all-to-all dispatch / combine), the shared expert over its tokens.  Batch
    1 on one GPU runs the fused decode layer (tf_moe_decode_layer).  Each
    batch's L-layer step is one CUDA graph; layer inputs come from a ring of 4
    sets.  value = whole-job tok/s at batch 256."""
    import copy

    import torch
    import torch.distributed as dist

    from edgeexpert_b200._lib import Context
    from edgeexpert_b200.ep import ExpertParallelMoE
    from edgeexpert_b200.format import synthetic_moe_layer
    from edgeexpert_b200.moe import ExpertPool, moe_decode_layer
    from edgeexpert_b200.prefill import (PrefillGroupedRoutedMoE, PrefillMoE, PrefillRouter, PrefillSharedExpert,
                                         route_sort)

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    ctx = Context.get(local_rank)
    sdt = torch.bfloat16 if a.scale_dtype == "bf16" else torch.float16
    L, per = a.layers, E // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(2024)  # the same model on every rank; each keeps its experts
    layers = []
    for _ in range(L):
        Lw = synthetic_moe_layer(D, F, FS, E, TOPK, 4, sdt, dev, gen)
        if world > 1:
            full = Lw.experts
            blob = full.blob.view(E, -1)[rank * per:(rank + 1) * per].reshape(-1).clone()
            Lw.experts = ExpertPool(blob, full.stride, per, full.offsets, D, F, full.scale_dtype)
            del full, blob
        layers.append(Lw)
    torch.cuda.empty_cache()
    c_layers = [Lw.as_c() for Lw in layers]
    router, shared = PrefillRouter(ctx), PrefillSharedExpert(ctx)
    grouped = PrefillGroupedRoutedMoE(ctx)
    stream = torch.cuda.Stream(device=dev)
    R = 4

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    batches = [a.tokens] if a.tokens else list(MOE_BATCHES)
    results = {}
    clk_all = None
    for B in batches:
        T = tokens_of(B, world, rank)
        cap = -(-B // world)
        Tm = max(T, 1)
        g2 = torch.Generator(device=dev)
        g2.manual_seed(99 + 7 * rank + B)
        xs = torch.randn(R, L, Tm, D, device=dev, generator=g2).to(torch.float16)
        x_in = torch.empty(L, Tm, D, dtype=torch.float16, device=dev)
        def io_set():  # one step's routing and outputs: (idx, wts, h2, ys)
            return (torch.empty(L, Tm, TOPK, dtype=torch.int32, device=dev),
                    torch.empty(L, Tm, TOPK, dtype=torch.float16, device=dev),
                    torch.empty(L, Tm, D, dtype=torch.float16, device=dev),
                    torch.empty(L, Tm, D, dtype=torch.float16, device=dev))

        idx, wts, h2, ys = idx0, wts0, h20, ys0 = io_set()
        # end-to-end steps alternate two input/output sets, so one step's copies
        # overlap the neighbouring steps' kernels
        x_e2e = [x_in, torch.empty(L, Tm, D, dtype=torch.float16, device=dev)]
        io_e2e = [io_set(), io_set()]
        sact = torch.empty(Tm, FS, dtype=torch.float16, device=dev)
        fused_b1 = world == 1 and B == 1
        xch = None
        if world > 1:
            from edgeexpert_b200.ep import P2PExchange
            xch = P2PExchange(world, rank, cap, D, context=ctx, device=dev) if a.exchange == "p2p" else None
            eps = [ExpertParallelMoE(layers[l].experts, E, TOPK, cap, D, F, context=ctx, device=dev, p2p=xch)
                   for l in range(L)]
        elif not fused_b1:
            act = torch.empty(T * TOPK, F, dtype=torch.float16, device=dev)
            part = torch.empty(T * TOPK, D, dtype=torch.float16, device=dev)
            from edgeexpert_b200.prefill import DeviceRoutes
            i32 = dict(dtype=torch.int32, device=dev)
            routes = DeviceRoutes(torch.empty(T * TOPK, 4, **i32), torch.empty(E, **i32), torch.empty(E, **i32),
                                  torch.empty(E, 3, **i32), torch.empty(1, **i32), torch.empty(E, 4, **i32),
                                  torch.empty(1, **i32))
        launches = 0
        side = torch.cuda.Stream(device=dev) if a.overlap_shared else None

        def step(xx, io=None):
            nonlocal launches
            launches = 0
            idx, wts, h2, ys = io if io is not None else (idx0, wts0, h20, ys0)
            for l in range(L):
                Lw, x = layers[l], xx[l]
                if T and side is not None and not fused_b1:
                    # the shared expert depends only on the layer input: it runs on a
                    # forked stream while the router, the grouping and the exchange
                    # (latency-bound, few SMs) run on the main one; joined at the
                    # layer's end
                    side.wait_stream(stream)
                    shared.encode(x, Lw.shared_gate, Lw.shared_up, Lw.shared_down, sact, ys[l], T, stream=side)
                    launches += 3
                if fused_b1:
                    moe_decode_layer(Lw, x[0], x[0], h2[l][0], out_indices=idx[l][0], out_weights=wts[l][0],
                                     stream=stream, context=ctx, c_layer=c_layers[l])
                    launches += 3
                    continue
                if T:
                    router.encode_gemma4_block(Lw.router_w, Lw.router_s, Lw.router_b, x, Lw.eff_scale,
                                               Lw.per_expert_scale, idx[l], wts[l], T, E, D, TOPK, stream=stream)
                    launches += 1
                if world > 1:
                    eps[l].forward(x[:T], idx[l][:T], wts[l][:T], h2[l][:T], stream=stream)
                    launches += 9
                else:
                    route_sort(idx[l], wts[l], T, TOPK, E, 16, stream=stream, context=ctx, out=routes)
                    grouped.encode(Lw.experts, routes, x, act, part, T, TOPK, stream=stream)
                    PrefillMoE.encode_reduce_token_major(part, wts[l], h2[l], T, TOPK, D, stream=stream, context=ctx)
                    launches += 7
                if T and side is not None:
                    stream.wait_stream(side)
                elif T:
                    shared.encode(x, Lw.shared_gate, Lw.shared_up, Lw.shared_down, sact, ys[l], T, stream=stream)
                    launches += 3

        def slot_args(r):  # ring slots 0..R-1, then the two end-to-end sets
            return (xs[r],) if r < R else (x_e2e[r - R], io_e2e[r - R])

        # eager warm-up (kernel attributes, NCCL communicators), then one graph per ring slot + x_in
        torch.cuda.synchronize()
        barrier()
        with torch.cuda.stream(stream):
            step(xs[0])
        torch.cuda.synchronize()
        barrier()
        graphs = []
        use_graph = True
        try:
            for r in range(R + 2):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    step(*slot_args(r))
                graphs.append(g)
        except Exception as exc:  # noqa: BLE001 -- fall back to eager launches, reported in the line
            use_graph = False
            graphs = []
            torch.cuda.synchronize()
            print(f"[bench] CUDA graph capture failed ({exc}); timing eager launches", file=sys.stderr)
        torch.cuda.synchronize()
        barrier()

        def run(r):
            if use_graph:
                graphs[r].replay()
            else:
                step(*slot_args(r))

        with torch.cuda.stream(stream):
            for i in range(a.warmup):
                run(i % R)
        torch.cuda.synchronize()
        clocks = ClockSampler(local_rank)
        clocks.start()
        barrier()
        torch.cuda.synchronize()
        steps = max(3, a.steps if B > 1 else a.steps)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for i in range(steps):
                run(i % R)
            e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1) / steps)
        clk = clocks.stop()
        if clk_all is None:
            clk_all = clk

        # end to end: each step's inputs H2D from pinned memory, outputs (h2, ys, routing) D2H.
        # The copies run on two copy streams (in, out) and the steps alternate two
        # device sets, so step i's input copy and step i-1's output copy overlap the
        # neighbouring steps' kernels; every copy is inside the timed region (the
        # copy streams start after the start event, the end event waits for both).
        h_in = torch.empty(L, Tm, D, dtype=torch.float16, pin_memory=True)
        h_in.copy_(xs[0].cpu())
        h_out = [(torch.empty(L, Tm, D, dtype=torch.float16, pin_memory=True),
                  torch.empty(L, Tm, D, dtype=torch.float16, pin_memory=True),
                  torch.empty(L, Tm, TOPK, dtype=torch.int32, pin_memory=True)) for _ in range(2)]
        cin, cout = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

        def e2e_steps(n):
            done = [None, None]  # per set: its last step's kernels finished
            freed = [None, None]  # per set: its last output copy finished
            cin.wait_stream(stream)
            cout.wait_stream(stream)
            for i in range(n):
                k = i & 1
                xin, (ei, _, eh2, eys) = x_e2e[k], io_e2e[k]
                if done[k] is not None:
                    cin.wait_event(done[k])  # step i-2 no longer reads this input set
                with torch.cuda.stream(cin):
                    xin.copy_(h_in, non_blocking=True)
                stream.wait_stream(cin)
                if freed[k] is not None:
                    stream.wait_event(freed[k])  # step i-2's outputs are on the host
                run(R + k)
                done[k] = torch.cuda.Event()
                done[k].record(stream)
                cout.wait_event(done[k])
                with torch.cuda.stream(cout):
                    hh2, hys, hidx = h_out[k]
                    hh2.copy_(eh2, non_blocking=True)
                    hys.copy_(eys, non_blocking=True)
                    hidx.copy_(ei, non_blocking=True)
                    freed[k] = torch.cuda.Event()
                    freed[k].record(cout)
            stream.wait_stream(cout)
            stream.wait_stream(cin)

        with torch.cuda.stream(stream):
            e2e_steps(max(2, a.warmup))
        torch.cuda.synchronize()
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            f0.record(stream)
            e2e_steps(steps)
            f1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms_e2e = max_over_ranks(f0.elapsed_time(f1) / steps)
        ctx.check_device(stream)

        # distinct local experts the step hit (routing of ring slot 0), for the HBM roofline
        with torch.cuda.stream(stream):
            run(0)
        torch.cuda.synchronize()
        ids_all = idx[:, :T].reshape(L, -1).cpu() if T else torch.empty(L, 0, dtype=torch.int32)
        if world > 1:  # what this rank's experts saw: every rank's routing
            ids_g = [torch.empty(L, cap * TOPK, dtype=torch.int32, device=dev) for _ in range(world)]
            mine = torch.full((L, cap * TOPK), -1, dtype=torch.int32, device=dev)
            if T:
                mine[:, :T * TOPK] = idx[:, :T].reshape(L, -1)
            dist.all_gather(ids_g, mine)
            ids_all = torch.cat([t.cpu() for t in ids_g], dim=1)
        distinct = 0.0
        for l in range(L):
            v = ids_all[l]
            v = v[(v >= rank * per) & (v < (rank + 1) * per)]
            distinct += float(torch.unique(v).numel())
        distinct /= L
        bytes_gpu = moe_step_bytes(B, world, distinct, L)
        # the dominant kernel alone: the grouped routed experts (gate/up + GELU, down)
        # of the last layer's routing, replayed over every layer's expert pool
        kern = None
        if not fused_b1:
            from edgeexpert_b200.format import affine_bytes
            if world > 1:
                eb = eps[-1].buf
                g_routes, g_x, g_rows = eb.routes, (xch.recv if xch is not None else eb.recv), world * cap
                g_act, g_part, g_stride = eb.act, eb.part, (2 * D + 64) // 2
                last = ids_all[L - 1]
                g_distinct = float(torch.unique(last[(last >= rank * per) & (last < (rank + 1) * per)]).numel())
            else:
                g_routes, g_x, g_rows, g_act, g_part, g_stride = routes, xs[0][L - 1], T, act, part, 0
                g_distinct = float(torch.unique(ids_all[L - 1]).numel())

            def grouped_all():
                for l in range(L):
                    grouped.encode(layers[l].experts, g_routes, g_x, g_act, g_part, g_rows, TOPK,
                                   hidden_stride=g_stride, stream=stream)

            with torch.cuda.stream(stream):
                grouped_all()
            torch.cuda.synchronize()
            gg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gg, stream=stream):
                grouped_all()
            with torch.cuda.stream(stream):
                for _ in range(3):
                    gg.replay()
            torch.cuda.synchronize()
            k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                k0.record(stream)
                for _ in range(5):
                    gg.replay()
                k1.record(stream)
            torch.cuda.synchronize()
            k_us = k0.elapsed_time(k1) * 1e3 / (5 * L)
            k_bytes = g_distinct * (2 * affine_bytes(F, D) + affine_bytes(D, F))
            kern = {"kernel": "grouped routed experts (grouped_stream_kernel gate/up + down, or the tcgen05 "
                              "qmm_kernel pair above 24 pairs per expert)",
                    "us_per_layer": k_us, "bytes_per_layer": k_bytes,
                    "achieved_gbs": k_bytes / (k_us * 1e-6) / 1e9, "distinct_experts": g_distinct}
            del gg
        results[B] = {
            "tokens": B, "tokens_per_gpu": cap, "ms_per_step": ms, "tok_s": B * 1e3 / ms,
            "tok_s_e2e": B * 1e3 / ms_e2e, "ms_e2e": ms_e2e, "graph": use_graph,
            "distinct_local_experts_per_layer": distinct,
            "hbm_bytes_per_gpu": bytes_gpu, "hbm_gbs_per_gpu": bytes_gpu / (ms * 1e-3) / 1e9,
            "gpu_launches_per_step": launches,
            "h2d_bytes_per_step": L * T * D * 2, "d2h_bytes_per_step": L * T * (2 * D * 2 + TOPK * 4),
            "nvlink_bytes_per_gpu_per_step": (L * (world - 1) * cap * (2 * D + 64 + 4 * D)) if world > 1 else 0,
            "exchange": (a.exchange if world > 1 else "none"),
            "dominant_kernel": kern,
            "clocks": clk,
        }
        del graphs
        if world > 1:
            del eps
            if xch is not None:
                barrier()
                xch.close()
        torch.cuda.empty_cache()

    # the full config-4 decode step (attention over a 4096-token fp16 KV cache,
    # norms, the MoE layers above, the int4 LM head and greedy selection)
    stack = None
    if not a.no_stack:
        stack = run_decoder_stack(a, rank, world, local_rank, layers, dev, ctx, stream, max_over_ranks, barrier)

    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak, peak_src = (peaks["hbm_gbs"], "measured hbm_gbs") if "hbm_gbs" in peaks else (6650.0, "fallback")
    Bh = batches[0]
    head = results[Bh]

    # single-GPU extras: the batch-1 decode roofline and the config-0 GEMV, in the same run
    dec = None
    gemv = None
    cpu = None
    if world == 1 and rank == 0:
        if not a.no_gemv:
            da = copy.copy(a)
            da.steps = max(20, a.steps)
            dec = run_ours(da, rank, world, local_rank, emit=False, layers=layers)
            ga = copy.copy(a)
            ga.steps, ga.scale_dtype = max(10 * a.steps, DEFAULT_STEPS["gemv"] // 3), "f16"
            gemv = run_gemv(ga, rank, world, local_rank, emit=False)
        if not a.no_cpu_baseline:
            # the oracle's per-token layer math, scaled to tokens through L layers
            cpu = cpu_baseline_record(lambda sec, th: cpu_sample(sec, "cpu", th), 1.0 / L * 1e9, a.cpu_seconds,
                                      unit="tok/s")
            cpu["sample"] += f"; tok/s = layer-tokens/s / {L} layers"
    if rank != 0:
        return
    # ncu DRAM bytes of the grouped gate/up + down pair per layer (one GPU, batch 256, all 128 experts hit)
    gs_traffic = None
    gs_tr = ROOT / "profiles" / "grouped_stream_traffic.json"
    if world == 1 and head.get("tokens") == 256 and gs_tr.exists():
        gs_traffic = json.loads(gs_tr.read_text()).get("bytes_per_launch")
    line = {
        "metric": METRIC, "value": head["tok_s"], "unit": "tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16-act/int4-w/fp32-acc",
        "data": "synthetic (BASELINE config-1 layer distributions, random-init weights, device RNG)",
        "config": {"workload": f"config-4 MoE decode step: batch {Bh} through {L} config-1 MoE layers "
                               f"(router + {TOPK} routed of {E} + shared), experts sharded {per} per GPU",
                   "d": D, "f": F, "fs": FS, "experts": E, "top_k": TOPK, "layers": L, "global_batch": Bh,
                   "parallelism": f"ep{world}" if world > 1 else "1gpu", "scale_dtype": a.scale_dtype,
                   "exchange": (f"{a.exchange} (fixed capacity, no host readback)" if world > 1 else "none"),
                   "l2": "weights per step (%.1f GB per GPU) exceed L2 (126 MB); no flush needed" %
                         (head["hbm_bytes_per_gpu"] / 1e9),
                   "outputs": "routed h2 and shared y per layer, kept separate",
                   "shared_expert": "forked stream beside the routed path" if a.overlap_shared else "after the routed path"},
        "batches": {str(b): results[b] for b in batches},
        "tok_s": head["tok_s"],
        "e2e": {"value": head["tok_s_e2e"], "unit": "tok/s", "h2d_bytes_per_step": head["h2d_bytes_per_step"],
                "d2h_bytes_per_step": head["d2h_bytes_per_step"],
                "copies": "pinned host buffers; in/out copy streams, two device sets alternating"},
        "roofline": ({"bound": "hbm", "kernel": head["dominant_kernel"]["kernel"],
                      "achieved": head["dominant_kernel"]["achieved_gbs"], "peak": peak, "peak_source": peak_src,
                      "unit": "GB/s", "frac": head["dominant_kernel"]["achieved_gbs"] / peak,
                      "traffic": gs_traffic, "bytes_per_launch": head["dominant_kernel"]["bytes_per_layer"],
                      "us_per_launch": head["dominant_kernel"]["us_per_layer"]}
                     if head.get("dominant_kernel") else None),
        "roofline_step": {"bound": "hbm", "kernel": "whole step per GPU (all kernels)",
                          "achieved": head["hbm_gbs_per_gpu"], "peak": peak,
                          "peak_source": peak_src, "unit": "GB/s", "frac": head["hbm_gbs_per_gpu"] / peak,
                          "bytes_per_step_per_gpu": head["hbm_bytes_per_gpu"]},
        "cpu_baseline": cpu,
        "clocks": head["clocks"],
        "gpu_launches": head["gpu_launches_per_step"] * a.steps,
    }
    if dec is not None:
        line["decode_b1"] = {k: dec[k] for k in ("metric", "value", "unit", "ms_per_step", "tok_s", "config", "e2e",
                                                 "roofline", "cpu_baseline", "clocks", "gpu_launches")}
        line["roofline_dominant_kernel"] = dec["roofline"]
    if gemv is not None:
        line["gemv"] = {k: gemv[k] for k in ("metric", "value", "unit", "steps", "ms_per_step", "config",
                                             "single_gemv_us", "single_gemv_gbs", "e2e", "roofline", "cpu_baseline",
                                             "clocks", "gpu_launches")}
    if stack is not None:
        line["decoder_stack"] = stack
    print(json.dumps(line), flush=True)


CONTEXT = 4096


def run_decoder_stack(a, rank, world, local_rank, moe_layers, dev, ctx, stream, max_over_ranks, barrier):
    """Config 4: one decode step of B sequences at position 4095 (attention over
    4096 cached tokens) through every layer (input norm, q/k/v int4 GEMVs, q/k/v
    norms + RoPE, split-KV attention, o_proj, post-attention norms, router,
    routed experts -- expert-parallel over the GPUs --, shared expert, layer
    tail) and the int4 LM head with greedy selection.  Tokens are split B/N
    per GPU with their KV caches.  A batch whose caches do not fit (1 GB per
    sequence) on every rank is reported as skipped."""
    import torch
    import torch.distributed as dist

    from edgeexpert_b200.decoder import Decoder, DecoderConfig, KVCache, synthetic_decoder
    from edgeexpert_b200.ep import ExpertParallelMoE
    cfg = DecoderConfig(layers=len(moe_layers), max_context=CONTEXT)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4040)
    w = synthetic_decoder(cfg, dev, gen, moe_layers=moe_layers)
    per = E // world
    out = {"context": CONTEXT, "layers": cfg.layers, "heads": f"{cfg.num_q_heads}q/{cfg.num_kv_heads}kv x {cfg.head_dim}",
           "vocab": cfg.vocab, "batches": {}}
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    for B in (1, 32, 256):
        T = tokens_of(B, world, rank)
        cap = -(-B // world)
        kv_bytes = 2 * cfg.layers * max(T, 1) * CONTEXT * cfg.num_kv_heads * cfg.head_dim * 2
        free, _ = torch.cuda.mem_get_info(dev)
        fits = kv_bytes + (6 << 30) < free
        if world > 1:
            f = torch.tensor([1 if fits else 0], device=dev)
            dist.all_reduce(f, op=dist.ReduceOp.MIN)
            fits = bool(f.item())
        if not fits:
            out["batches"][str(B)] = {"skipped": f"KV cache of {max(T, 1)} sequences x {CONTEXT} tokens "
                                                 f"({kv_bytes / 1e9:.0f} GB per GPU) does not fit"}
            continue
        cache = KVCache(cfg, max(T, 1), dev)
        cache.fill_random(gen, CONTEXT)
        eps, xch = None, None
        if world > 1:
            from edgeexpert_b200.ep import P2PExchange
            xch = P2PExchange(world, rank, cap, D, context=ctx, device=dev) if a.exchange == "p2p" else None
            eps = [ExpertParallelMoE(L.experts, E, TOPK, cap, D, F, context=ctx, device=dev, p2p=xch)
                   for L in moe_layers]
        dec = Decoder(w, T, cache, context=ctx, device=dev, ep_layers=eps)
        toks = torch.randint(0, cfg.vocab, (max(T, 1),), device=dev, dtype=torch.int32, generator=gen)
        torch.cuda.synchronize()
        barrier()
        with torch.cuda.stream(stream):
            dec.step(toks, CONTEXT - 1, stream=stream)
        torch.cuda.synchronize()
        barrier()
        g = torch.cuda.CUDAGraph()
        use_graph = True
        try:
            with torch.cuda.graph(g, stream=stream):
                dec.step(toks, CONTEXT - 1, stream=stream)
        except Exception as exc:  # noqa: BLE001 -- eager launches, reported
            use_graph = False
            torch.cuda.synchronize()
            print(f"[bench] decoder graph capture failed ({exc}); timing eager launches", file=sys.stderr)
        torch.cuda.synchronize()
        barrier()

        def run():
            if use_graph:
                g.replay()
            else:
                dec.step(toks, CONTEXT - 1, stream=stream)

        with torch.cuda.stream(stream):
            for _ in range(max(3, a.warmup)):
                run()
        torch.cuda.synchronize()
        barrier()
        steps = max(5, a.steps // 2)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(steps):
                run()
            e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1) / steps)
        # end to end: the step's token ids from pinned host memory, the next tokens back
        h_tok = torch.empty(max(T, 1), dtype=torch.int32, pin_memory=True)
        h_tok.copy_(toks.cpu())
        h_next = torch.empty(max(T, 1), dtype=torch.int32, pin_memory=True)
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            f0.record(stream)
            for _ in range(steps):
                toks.copy_(h_tok, non_blocking=True)
                run()
                h_next.copy_(dec.tokens, non_blocking=True)
            f1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms_e2e = max_over_ranks(f0.elapsed_time(f1) / steps)
        ctx.check_device(stream)
        # distinct local experts of the last layer's routing (every rank's tokens reach these experts)
        mine = torch.full((cap * TOPK,), -1, dtype=torch.int32, device=dev)
        if T:
            mine[:T * TOPK] = dec.idx[:T].reshape(-1)
        if world > 1:
            allr = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(allr, mine)
            idx_all = torch.cat(allr).cpu()
        else:
            idx_all = mine.cpu()
        distinct = float(torch.unique(idx_all[(idx_all >= rank * per) & (idx_all < (rank + 1) * per)]).numel())
        wbytes = dec.weight_bytes_per_step(distinct)
        kv_read = cache.nbytes_per_token(CONTEXT) * T
        out["batches"][str(B)] = {
            "tokens": B, "tokens_per_gpu": T, "ms_per_step": ms, "tok_s": B * 1e3 / ms, "tok_s_e2e": B * 1e3 / ms_e2e,
            "graph": use_graph, "gpu_launches_per_step": dec.launches,
            "hbm_bytes_per_gpu": wbytes + kv_read, "kv_bytes_per_gpu": kv_read,
            "hbm_gbs_per_gpu": (wbytes + kv_read) / (ms * 1e-3) / 1e9,
            "roofline_frac": (wbytes + kv_read) / (ms * 1e-3) / 1e9 / peak,
            "h2d_bytes_per_step": 4 * T, "d2h_bytes_per_step": 4 * T,
        }
        del g, dec, cache, eps
        if xch is not None:
            barrier()
            xch.close()
        torch.cuda.empty_cache()
    return out


# ------------------------------------------------------ decode attention ----
def attention_cpu_sample(seconds: float, threads: int | None = None):
    """The oracle's split-KV attention (double precision) over one sequence
    of the config-4 layer (16 query / 8 KV heads of 256, 4096 positions),
    repeated for ~`seconds`; one sequence at a time (the oracle is scalar).
    Returns (sequences/s, threads, sample text)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np

    import oracle as O
    rng = np.random.default_rng(5)
    K = rng.standard_normal((CONTEXT, 8, 256)).astype(np.float16).view(np.uint16)
    V = rng.standard_normal((CONTEXT, 8, 256)).astype(np.float16).view(np.uint16)
    q = (rng.standard_normal((16, 256)) * 0.08).astype(np.float16).view(np.uint16)
    n, t0 = 0, time.perf_counter()
    while True:
        O.attention_decode(q, K, V, 256, 16, 8, CONTEXT, 0, 1.0)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return n / el, 1, f"{n} sequences of 4096 positions x 8 KV heads x 256 through the oracle in {el:.1f} s"


def run_attention(a, rank, world, local_rank):
    """Config 4's decode attention alone: `--tokens` sequences (default 32)
    at position 4095 over a 4096-token fp16 KV cache, 16 query / 8 KV heads
    of dim 256 (tf_attention_decode: the split-KV partial kernel and the
    chunk merge).  value = KV-cache bytes read per second; one layer's cache
    (1.07 GB at 32 sequences) exceeds L2, so no flush is needed.  Replicas
    at N > 1 (attention does not shard across GPUs)."""
    import torch
    import torch.distributed as dist

    from edgeexpert_b200._lib import Context
    from edgeexpert_b200.decoder import Attention

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    ctx = Context.get(local_rank)
    B = a.tokens or 32
    nq, nkv, hd = 16, 8, 256
    gen = torch.Generator(device=dev)
    gen.manual_seed(91 + rank)
    K = torch.randn(B, CONTEXT, nkv, hd, device=dev, generator=gen, dtype=torch.float32).to(torch.float16)
    V = torch.randn(B, CONTEXT, nkv, hd, device=dev, generator=gen, dtype=torch.float32).to(torch.float16)
    q = (torch.randn(B, nq * hd, device=dev, generator=gen) * 0.08).to(torch.float16)
    out = torch.empty(B, nq * hd, dtype=torch.float16, device=dev)
    att = Attention(context=ctx)
    ws = torch.empty(att.workspace_bytes(B, hd, nq, nkv, CONTEXT) // 4 + 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(s, qq, oo):
        att.encode(qq, K, V, oo, hd, nq, nkv, B, CONTEXT, ws, scale=hd ** -0.5, seq_stride=CONTEXT * nkv * hd,
                   stream=s)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.cuda.stream(stream):
        for _ in range(max(3, a.warmup)):
            step(stream, q, out)
    torch.cuda.synchronize()
    barrier()
    clk = ClockSampler(local_rank)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(a.steps):
        step(stream, q, out)
    e1.record(stream)
    torch.cuda.synchronize()
    clocks = clk.stop()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    # end to end: q from pinned host memory, the attention output back, every step
    h_q = torch.empty_like(q, device="cpu").pin_memory()
    h_q.copy_(q.cpu())
    h_out = torch.empty_like(out, device="cpu").pin_memory()
    q_in, out_d = torch.empty_like(q), torch.empty_like(out)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        for _ in range(a.steps):
            q_in.copy_(h_q, non_blocking=True)
            step(stream, q_in, out_d)
            h_out.copy_(out_d, non_blocking=True)
        f1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = max_over_ranks(f0.elapsed_time(f1) / a.steps)
    ctx.check_device(stream)
    kv = 2 * B * CONTEXT * nkv * hd * 2
    per_gpu = (kv + 2 * q.numel() * 2) / (ms * 1e-3) / 1e9
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    src = "measured hbm_gbs" if "hbm_gbs" in peaks else "fallback 6.65 TB/s"
    if rank != 0:
        return
    line = {
        "metric": "decode attention KV-cache GB/s (config 4 layer)", "value": per_gpu * world, "unit": "GB/s",
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16-kv/fp32-acc", "data": "synthetic N(0,1) cache",
        "config": {"workload": f"config-4 decode attention, {B} sequences x {CONTEXT} positions, 16q/8kv x 256",
                   "parallelism": f"replicas{world}", "l2": "1.07 GB of cache per step at 32 sequences exceeds L2"},
        "e2e": {"value": (kv + 2 * q.numel() * 2) / (ms_e2e * 1e-3) / 1e9 * world, "unit": "GB/s",
                "h2d_bytes_per_step": q.numel() * 2, "d2h_bytes_per_step": out.numel() * 2},
        "roofline": {"bound": "hbm", "kernel": "attention_stream_kernel + attention_combine_kernel",
                     "achieved": per_gpu, "peak": peak, "peak_source": src, "unit": "GB/s", "frac": per_gpu / peak,
                     "traffic": (1074024000 + 5156864) * B // 32 if B == 32 else None,
                     "traffic_source": "profiles/attention_stream_kernel_ncu.md (32 sequences)",
                     "bytes_per_launch": kv, "us_per_launch": ms * 1e3},
        "gpu_launches": 2 * a.steps, "clocks": clocks,
    }
    if not a.no_cpu_baseline:
        u, thr, txt = attention_cpu_sample(min(a.cpu_seconds, 10.0))
        line["cpu_baseline"] = {"value": u * (kv / B) / 1e9, "unit": "GB/s", "cores": thr, "kind": "port",
                                "sample": txt, "cpu_model": cpu_model()}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------ chunk workloads ----
CHUNK_TOKENS = {"batched": 64, "prefill": 4096}


def chunk_flops(T: int) -> float:
    """Algorithmic FLOPs of one chunk through the config-1 layer: router,
    top-8 routed experts (gate, up, down) and the shared expert."""
    return 2.0 * T * (TOPK * 3 * F * D + 3 * FS * D + E * D)


def chunk_bytes(distinct: int) -> int:
    """Algorithmic weight bytes of one chunk: every distinct routed expert,
    the shared expert and the router, each read once."""
    from edgeexpert_b200.format import affine_bytes
    expert = 2 * affine_bytes(F, D) + affine_bytes(D, F)
    shared = 2 * affine_bytes(FS, D) + affine_bytes(D, FS)
    router = E * D + 2 * E * (D // 64) * 2
    return distinct * expert + shared + router


def run_chunk(a, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from edgeexpert_b200._lib import Context
    from edgeexpert_b200.format import synthetic_moe_layer
    from edgeexpert_b200.prefill import (PrefillGroupedRoutedMoE, PrefillMoE, PrefillRouter, PrefillSharedExpert,
                                         route_sort)

    T = a.tokens or CHUNK_TOKENS[a.workload]
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    ctx = Context.get(local_rank)
    sdt = torch.bfloat16 if a.scale_dtype == "bf16" else torch.float16
    gen = torch.Generator(device=dev)
    gen.manual_seed(4321 + rank)
    nl = 4  # ring of distinct layers (>= 1.7 GB of weights: no L2 reuse between steps)
    layers = [synthetic_moe_layer(D, F, FS, E, TOPK, 4, sdt, dev, gen) for _ in range(nl)]
    # random router weights give a skewed expert histogram
    for L in layers:
        L.per_expert_scale.copy_((1.0 + 0.3 * torch.randn(E, device=dev, generator=gen)).abs().to(torch.bfloat16))
    xs = torch.randn(nl, T, D, device=dev, generator=gen).to(torch.float16)
    idx = torch.empty(T, TOPK, dtype=torch.int32, device=dev)
    wts = torch.empty(T, TOPK, dtype=torch.float16, device=dev)
    act = torch.empty(T * TOPK, F, dtype=torch.float16, device=dev)
    part = torch.empty(T * TOPK, D, dtype=torch.float16, device=dev)
    h2 = torch.empty(T, D, dtype=torch.float16, device=dev)
    acts = torch.empty(T, FS, dtype=torch.float16, device=dev)
    ys = torch.empty(T, D, dtype=torch.float16, device=dev)
    x_in = torch.empty(T, D, dtype=torch.float16, device=dev)
    routes = route_sort(idx.zero_(), wts.zero_(), T, TOPK, E, 16, context=ctx)
    router, grouped, shared = PrefillRouter(ctx), PrefillGroupedRoutedMoE(ctx), PrefillSharedExpert(ctx)
    stream = torch.cuda.Stream(device=dev)

    def step(L, x, s):
        router.encode_gemma4_block(L.router_w, L.router_s, L.router_b, x, L.eff_scale, L.per_expert_scale, idx, wts,
                                   T, E, D, TOPK, stream=s)
        route_sort(idx, wts, T, TOPK, E, 16, stream=s, context=ctx, out=routes)
        grouped.encode(L.experts, routes, x, act, part, T, TOPK, stream=s)
        PrefillMoE.encode_reduce_token_major(part, wts, h2, T, TOPK, D, stream=s, context=ctx)
        shared.encode(x, L.shared_gate, L.shared_up, L.shared_down, acts, ys, T, stream=s)

    launches_per_step = 8  # router, sort, gather, 2 grouped QMM, reduce, 2 shared QMM
    with torch.cuda.stream(stream):
        step(layers[0], xs[0], stream)
    torch.cuda.synchronize()
    graphs = []
    for r in range(nl + 1):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(layers[r % nl], xs[r] if r < nl else x_in, stream)
        graphs.append(g)
    torch.cuda.synchronize()
    # distinct experts hit per layer (the weight bytes a step must read)
    distinct = []
    for r in range(nl):
        graphs[r].replay()
        torch.cuda.synchronize()
        distinct.append(int(routes.n_groups.item()))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            graphs[i % nl].replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for i in range(a.steps):
            graphs[i % nl].replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / a.steps)
    clk = clocks.stop()

    # end to end: the chunk's activations H2D from pinned memory, both outputs D2H
    h_in = torch.empty(nl, T, D, dtype=torch.float16, pin_memory=True)
    h_in.copy_(xs.cpu())
    h_h2 = torch.empty(T, D, dtype=torch.float16, pin_memory=True)
    h_ys = torch.empty(T, D, dtype=torch.float16, pin_memory=True)
    h_ids = torch.empty(T, TOPK, dtype=torch.int32, pin_memory=True)

    def e2e_step(i):
        x_in.copy_(h_in[i % nl], non_blocking=True)
        graphs[nl].replay()
        h_h2.copy_(h2, non_blocking=True)
        h_ys.copy_(ys, non_blocking=True)
        h_ids.copy_(idx, non_blocking=True)

    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(a.steps):
            e2e_step(i)
        e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    h2d = T * D * 2
    d2h = 2 * T * D * 2 + T * TOPK * 4

    # roofline of the dominant kernel: the grouped gate/up tcgen05 GEMM, timed alone
    from edgeexpert_b200._lib import lib, ptr, stream_ptr
    import ctypes as C
    L0 = layers[0]
    with torch.cuda.stream(stream):
        graphs[0].replay()
    torch.cuda.synchronize()
    gg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gg, stream=stream):
        for _ in range(5):
            grouped.encode(L0.experts, routes, xs[0], act, part, T, TOPK, stream=stream)
    with torch.cuda.stream(stream):
        gg.replay()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        g0.record(stream)
        gg.replay()
        g1.record(stream)
    torch.cuda.synchronize()
    grouped_us = g0.elapsed_time(g1) * 1e3 / 5
    grouped_flops = 2.0 * T * TOPK * 3 * F * D
    ctx.check_device(stream)

    peaks = {}
    pk_path = ROOT / "MEASURED_PEAKS.json"
    if pk_path.exists():
        peaks = json.loads(pk_path.read_text())
    if a.workload == "prefill":
        peak, peak_src, unit_r = (peaks.get("bf16_tflops", 1590.0), "measured" if "bf16_tflops" in peaks else
                                  "fallback", "TFLOP/s")
        achieved = grouped_flops / (grouped_us * 1e-6) / 1e12
        bound = "tensor"
    else:
        peak, peak_src, unit_r = (peaks.get("hbm_gbs", 6650.0), "measured" if "hbm_gbs" in peaks else "fallback",
                                  "GB/s")
        achieved = (chunk_bytes(distinct[0]) - chunk_bytes(0)) / (grouped_us * 1e-6) / 1e9
        bound = "hbm"

    flops = chunk_flops(T)
    bytes_step = sum(chunk_bytes(d) for d in distinct) / nl
    if a.workload == "prefill":
        metric, unit = "MoE prefill TFLOP/s (config 3)", "TFLOP/s"
        value = world * flops / (ms * 1e-3) / 1e12
        e2e_value = world * flops / (ms_e2e * 1e-3) / 1e12
    else:
        metric, unit = "MoE batched-decode weight GB/s (config 2)", "GB/s"
        value = world * bytes_step / (ms * 1e-3) / 1e9
        e2e_value = world * bytes_step / (ms_e2e * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        lps, threads, sample = cpu_sample(a.cpu_seconds)
        cpu_ms = T * 1e3 / lps
        cpu_v = flops / (cpu_ms * 1e-3) / 1e12 if a.workload == "prefill" else bytes_step / (cpu_ms * 1e-3) / 1e9
        cpu = {"value": cpu_v, "unit": unit, "cores": threads, "kind": "port",
               "sample": sample + f"; scaled to a {T}-token chunk"}

    if rank == 0:
        line = {
            "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16-act/int4-w/fp32-acc", "data": "synthetic (BASELINE distributions, random-init weights)",
            "config": {"workload": f"config{3 if a.workload == 'prefill' else 2}: {T}-token chunk through the "
                                   "config-1 MoE layer (router, device grouping, grouped routed experts, "
                                   "token-major reduce, shared expert)",
                       "tokens": T, "d": D, "f": F, "fs": FS, "experts": E, "top_k": TOPK, "layer_ring": nl,
                       "distinct_experts": distinct, "scale_dtype": a.scale_dtype,
                       "l2": "ring of 4 layers (%.1f GB) exceeds L2; no flush needed" %
                             (nl * chunk_bytes(E) / 1e9),
                       "outputs": "routed h2 and shared y kept separate (the reference combines them in its norm "
                                  "kernel, outside this path)"},
            "tok_s": world * T * 1e3 / ms, "tok_s_e2e": world * T * 1e3 / ms_e2e,
            "flops_per_step": flops, "weight_bytes_per_step": bytes_step,
            "e2e": {"value": e2e_value, "unit": unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": {"bound": bound, "kernel": "qmm_kernel (grouped gate/up + down, incl. row gather)",
                         "achieved": achieved, "peak": peak, "peak_source": f"{peak_src}", "unit": unit_r,
                         "frac": achieved / peak, "traffic": None, "us_per_launch": grouped_us,
                         "work_per_launch": grouped_flops if bound == "tensor" else
                         chunk_bytes(distinct[0]) - chunk_bytes(0)},
            "cpu_baseline": cpu,
            "clocks": clk,
            "gpu_launches": launches_per_step * a.steps,
        }
        print(json.dumps(line), flush=True)


DEFAULT_STEPS = {"moe": 50, "decode": 400, "gemv": 3000, "batched": 1000, "prefill": 300, "ep": 200, "attention": 2000}


def main():
    a = parse()
    if a.steps <= 0:
        a.steps = DEFAULT_STEPS[a.workload]
    if a.scale_dtype is None:
        a.scale_dtype = "f16" if a.workload == "gemv" else "bf16"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference(a, rank)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    if a.workload == "moe":
        run_moe(a, rank, world, local_rank)
    elif a.workload == "decode":
        run_ours(a, rank, world, local_rank)
    elif a.workload == "gemv":
        run_gemv(a, rank, world, local_rank)
    elif a.workload == "ep":
        run_ep(a, rank, world, local_rank)
    elif a.workload == "attention":
        run_attention(a, rank, world, local_rank)
    else:
        run_chunk(a, rank, world, local_rank)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
