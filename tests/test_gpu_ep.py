"""Expert parallelism on 2 GPUs (NCCL): each rank owns half of the routed
experts and its own tokens; the result for its tokens must equal the
single-GPU grouped path (route sort -> grouped GEMMs -> token-major reduce)
run on the same rank with all experts.  Skips with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

D, F, E, K = 512, 256, 16, 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from edgeexpert_b200.ep import ExpertParallelMoE
        from edgeexpert_b200.format import synthetic_expert_pool
        from edgeexpert_b200.moe import ExpertPool
        from edgeexpert_b200.prefill import PrefillGroupedRoutedMoE, PrefillMoE, route_sort
        gen = torch.Generator(device=dev)
        gen.manual_seed(5)  # identical experts on every rank
        full = synthetic_expert_pool(E, D, F, torch.bfloat16, dev, gen)
        per = E // world
        local = ExpertPool(full.blob.view(E, -1)[rank * per:(rank + 1) * per].reshape(-1).clone(), full.stride, per,
                           full.offsets, D, F, full.scale_dtype)
        T = [40, 24, 33, 7][rank]
        g2 = torch.Generator(device=dev)
        g2.manual_seed(100 + rank)
        X = torch.randn(T, D, device=dev, generator=g2).half()
        idx = torch.stack([torch.randperm(E, device=dev, generator=g2)[:K] for _ in range(T)]).int()
        w = (torch.rand(T, K, device=dev, generator=g2) * 0.5 + 0.1).half()
        h2 = torch.empty(T, D, dtype=torch.float16, device=dev)
        ExpertParallelMoE(local, E, K).forward(X, idx, w, h2)
        # single-GPU path with every expert
        routes = route_sort(idx, w, T, K, E, 16)
        act = torch.empty(T * K, F, dtype=torch.float16, device=dev)
        part = torch.empty(T * K, D, dtype=torch.float16, device=dev)
        PrefillGroupedRoutedMoE().encode(full, routes, X, act, part, T, K)
        ref = torch.empty_like(h2)
        PrefillMoE.encode_reduce_token_major(part, w, ref, T, K, D)
        torch.cuda.synchronize()
        err = float((h2.float() - ref.float()).abs().max() / ref.float().abs().max().clamp_min(1e-6))
        results[rank] = (err, bool(torch.equal(h2, ref)))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_two_gpus_matches_single_gpu(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
    for r in range(world):
        err, same = results[r]
        assert err < 2e-3, f"rank {r}: rel error {err}"
