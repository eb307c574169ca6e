"""Expert parallelism on the GPU against the oracle.

Each rank owns E/P of the routed experts and routes its own tokens; its
routed output h2 must match the oracle's layer (per-pair expert FFN of
prefill.metal:336-440,598-670, then the token-major reduce of
prefill.metal:575-596) within RelError 2e-3 (the fp32 sum is regrouped by
owner rank, so agreement is to fp32 rounding, not bitwise).

* world 1: the fixed-capacity dispatch kernels with an identity exchange (any box);
* world 2: two GPUs (skips with fewer than 2 GPUs), with the NCCL
  all-to-alls and with the peer-memory exchange (tf_ep_*_p2p), including a
  rank whose tokens all route to its own experts and uneven token counts.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O

pytestmark = pytest.mark.gpu

D, F, E, K = 512, 256, 16, 8
FP16_TOL = 2e-3


def host_experts():
    from edgeexpert_b200.format import expert_layout
    lay = expert_layout(D, F)
    rng = O.seed_tree(0xE9, "gpu-ep")
    o = lay.offsets
    host = np.zeros((E, lay.stride), np.uint8)
    for e in range(E):
        for proj, rows, cols in (("gate", F, D), ("up", F, D), ("down", D, F)):
            W, S, B = rng.synthetic_affine(rows, cols, 4, 0)
            for part, arr in (("w", W), ("s", S), ("b", B)):
                b = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
                off = getattr(o, f"{proj}_{part}")
                host[e, off:off + b.size] = b
    return host, lay


def tokens_for(rank, T, own_only=False, world=2):
    rng = np.random.default_rng(100 + rank)
    X = O.seed_tree(rank, "gpu-ep-x").normal_f16(T * D).reshape(T, D)
    per = E // world
    lo, hi = (rank * per, (rank + 1) * per) if own_only else (0, E)
    idx = np.stack([rng.choice(np.arange(lo, hi), K, replace=False) for _ in range(T)]).astype(np.int32)
    w = (rng.random((T, K)) * 0.5 + 0.1).astype(np.float16)
    return X, idx, w


def oracle_h2(host, lay, X, idx, w):
    from edgeexpert_b200.prefill import PrefillRouter
    T = X.shape[0]
    off = O.Offsets(*[getattr(lay.offsets, n) for n, _ in O.Offsets._fields_])
    pairs = PrefillRouter.make_token_expert_pairs(idx.astype(np.uint32), w, T, K)
    g = O.group_pairs(pairs, T, K, E, 16)
    part = O.grouped_routed(host.reshape(-1), lay.stride, off, g["sorted"], X, D, D, F, K, T, 0)
    return O.reduce_token_major(part, w.view(np.uint16), T, K, D)


def run_rank(rank, world, T, capacity, own_only, dev, p2p=False):
    from edgeexpert_b200.ep import ExpertParallelMoE, P2PExchange
    from edgeexpert_b200.moe import ExpertPool
    host, lay = host_experts()
    per = E // world
    local = ExpertPool(torch.from_numpy(host[rank * per:(rank + 1) * per].reshape(-1).copy()).to(dev), lay.stride, per,
                       lay.offsets, D, F, torch.bfloat16)
    X, idx, w = tokens_for(rank, T, own_only, world)
    x = P2PExchange(world, rank, capacity, D, device=dev) if p2p else None
    ep = ExpertParallelMoE(local, E, K, capacity, D, F, device=dev, p2p=x)
    h2 = torch.empty(T, D, dtype=torch.float16, device=dev)
    args = (torch.from_numpy(X.view(np.float16)).to(dev), torch.from_numpy(idx).to(dev), torch.from_numpy(w).to(dev))
    ep.forward(*args, h2)
    h2b = torch.empty_like(h2)
    ep.forward(*args, h2b)  # second call on the same buffers: deterministic
    torch.cuda.synchronize()
    got = O.f16_to_f32(h2.cpu().numpy().view(np.uint16))
    ref = O.f16_to_f32(oracle_h2(host, lay, X, idx, w).reshape(T, D))
    if x is not None:
        if world > 1:
            dist.barrier()  # no peer still writes into this rank's buffers
        x.close()
    return O.rel_error(got, ref), bool(torch.equal(h2, h2b))


def test_expert_parallel_world1_matches_oracle(cuda):
    """The dispatch/unpack/combine/reduce kernels with one rank (identity
    exchange), capacity larger than T (empty slots)."""
    before = device_flags()  # read and clear what earlier tests left
    err, det = run_rank(0, 1, 37, 48, False, torch.device("cuda", 0))
    assert err < FP16_TOL, err
    assert det
    assert device_flags() == 0, f"flags raised by the EP layer (before it: {before:#x})"


def device_flags(device: int = 0) -> int:
    """The context's device error flags, read and cleared without raising."""
    import ctypes as C

    from edgeexpert_b200._lib import Context, lib
    flags = C.c_uint32(0)
    lib().tf_context_check_device(Context.get(device).handle, C.c_void_p(0), C.byref(flags))
    return flags.value


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        T = [40, 23][rank]
        results[(rank, "nccl")] = run_rank(rank, world, T, 40, own_only=(rank == 1), dev=dev)
        results[(rank, "p2p")] = run_rank(rank, world, T, 40, own_only=(rank == 1), dev=dev, p2p=True)
        results[(rank, "flags")] = device_flags(rank)
    finally:
        dist.destroy_process_group()


def test_expert_parallel_two_gpus_matches_oracle(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
    for r in range(world):
        for mode in ("nccl", "p2p"):
            err, det = results[(r, mode)]
            assert err < FP16_TOL, f"rank {r} {mode}: rel error {err}"
            assert det, f"rank {r} {mode}: not deterministic"
        assert results[(r, "flags")] == 0
