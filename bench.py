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
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=30)
    ap.add_argument("--ring", type=int, default=8)
    ap.add_argument("--scale-dtype", choices=["bf16", "f16"], default="bf16")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
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
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
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
def cpu_sample(seconds: float, label: str = "cpu"):
    """Oracle port of the reference CPU math on the host cores: router + top-8
    + 8 routed experts + shared expert for one token of one config-1 layer,
    repeated for ~`seconds`.  Returns (layer-tokens/s, threads, sample text)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np

    import oracle as O
    threads = O.lib().orc_max_threads()
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
    lps, threads, sample = cpu_sample(max(5.0, a.cpu_seconds), "reference")
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
def run_ours(a, rank, world, local_rank):
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
    layers = [synthetic_moe_layer(D, F, FS, E, TOPK, 4, sdt, dev, gen) for _ in range(a.layers)]
    c_layers = [L.as_c() for L in layers]
    L, R = a.layers, a.ring
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
        lps, threads, sample = cpu_sample(a.cpu_seconds)
        cpu = {"value": lps * layer_bytes() / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": sample}

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
        print(json.dumps(line), flush=True)


def main():
    a = parse()
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
    run_ours(a, rank, world, local_rank)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
