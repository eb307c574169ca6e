"""Expert-parallel exchange logic on CPU: world_size 2 over gloo.

The device work is replaced by the C oracle (grouping, per-pair expert FFN of
prefill.metal:336-440,598-670, token-major reduce of prefill.metal:575-596),
so the test checks the host side of edgeexpert_b200.ep: per-destination
counts, the all-to-all-v of rows and local expert ids, the return trip in
sorted-pair order and the combine.  Each rank's output must equal a
single-process run of the same layer bit for bit.
"""
import os
import socket
from dataclasses import dataclass

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O

D, F, E, K = 128, 64, 8, 2


@dataclass
class HostRoutes:
    sorted_pairs: np.ndarray
    counts: np.ndarray


class OracleOps:
    """CPU stand-in for edgeexpert_b200.ep.CudaOps (same contract)."""

    def __init__(self, host_experts, lay_stride, off, per_rank, rank):
        self.host, self.stride, self.off = host_experts, lay_stride, off
        self.per_rank, self.rank = per_rank, rank

    def route(self, expert_ids, weights, T, K_, E_):
        from edgeexpert_b200.prefill import PrefillRouter
        idx = expert_ids.numpy().astype(np.uint32).reshape(T, K_)
        w = weights.numpy().reshape(T, K_)
        pairs = PrefillRouter.make_token_expert_pairs(idx, w, T, K_)
        g = O.group_pairs(pairs, T, K_, E_, 16)
        return HostRoutes(g["sorted"], g["counts"])

    def send_counts(self, routes, E_, per_rank, world):
        c = routes.counts.astype(np.int64)
        return [int(c[r * per_rank:(r + 1) * per_rank].sum()) for r in range(world)]

    def pack(self, hidden, routes, n, T, per_rank):
        sp = routes.sorted_pairs
        rows = hidden[torch.from_numpy(sp["token"].astype(np.int64))] if n else hidden[:0]
        local = torch.from_numpy((sp["expert"] % per_rank).astype(np.int32))
        return rows.contiguous(), local

    def experts(self, pool, rows, local):
        n = rows.shape[0]
        if n == 0:
            return torch.empty(0, D, dtype=torch.float16)
        lo = self.rank * self.per_rank
        local_host = self.host[lo:lo + self.per_rank].reshape(-1)
        pairs = np.zeros(n, O.PAIR_DTYPE)
        pairs["token"] = np.arange(n)
        pairs["expert"] = local.numpy().astype(np.uint32)
        pairs["weight_bits"] = 0x3C00
        order = np.lexsort((pairs["token"], pairs["expert"]))
        part = O.grouped_routed(local_host, self.stride, self.off, pairs[order], rows.numpy().view(np.uint16), D, D, F,
                                1, n, 0)
        return torch.from_numpy(part.view(np.float16).reshape(n, D).copy())

    def combine(self, routes, back, weights, h2, T, K_):
        sp = routes.sorted_pairs
        tok = np.zeros((T * K_, D), np.uint16)
        if T:
            tok[sp["token"].astype(np.int64) * K_ + sp["rank"].astype(np.int64)] = back.numpy().view(np.uint16)
        out = O.reduce_token_major(tok.reshape(-1), weights.numpy().view(np.uint16).reshape(-1), T, K_, D)
        h2.copy_(torch.from_numpy(out.view(np.float16).reshape(T, D).copy()))


def make_layer():
    from edgeexpert_b200.format import expert_layout
    lay = expert_layout(D, F)
    rng = O.seed_tree(0xEE, "ep-host")
    o = lay.offsets
    host = np.zeros((E, lay.stride), np.uint8)
    for e in range(E):
        for proj, rows, cols in (("gate", F, D), ("up", F, D), ("down", D, F)):
            W, S, B = rng.synthetic_affine(rows, cols, 4, 0)
            for part, arr in (("w", W), ("s", S), ("b", B)):
                b = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
                off = getattr(o, f"{proj}_{part}")
                host[e, off:off + b.size] = b
    off = O.Offsets(*[getattr(o, n) for n, _ in O.Offsets._fields_])
    return host, lay.stride, off


def tokens_for(rank, skew):
    T = [5, 3][rank]
    rng = np.random.default_rng(100 + rank)
    X = O.seed_tree(rank, "ep-x").normal_f16(T * D).reshape(T, D)
    if skew:  # every pair of rank 0 goes to rank 0's own experts, rank 1 sends everywhere
        lo, hi = (0, E // 2) if rank == 0 else (0, E)
    else:
        lo, hi = 0, E
    idx = np.stack([rng.choice(np.arange(lo, hi), K, replace=False) for _ in range(T)]).astype(np.int32)
    w = (rng.random((T, K)) * 0.5 + 0.1).astype(np.float16)
    return X, idx, w


def single_process_reference(host, stride, off, X, idx, w):
    from edgeexpert_b200.prefill import PrefillRouter
    T = X.shape[0]
    pairs = PrefillRouter.make_token_expert_pairs(idx.astype(np.uint32), w, T, K)
    g = O.group_pairs(pairs, T, K, E, 16)
    part = O.grouped_routed(host.reshape(-1), stride, off, g["sorted"], X, D, D, F, K, T, 0)
    return O.reduce_token_major(part, w.view(np.uint16), T, K, D)


def _worker(rank, world, port, skew, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from edgeexpert_b200.ep import ExpertParallelMoE
        host, stride, off = make_layer()
        X, idx, w = tokens_for(rank, skew)
        ops = OracleOps(host, stride, off, E // world, rank)
        ep = ExpertParallelMoE(None, E, K, ops=ops)
        h2 = torch.empty(X.shape[0], D, dtype=torch.float16)
        ep.forward(torch.from_numpy(X.view(np.float16)), torch.from_numpy(idx), torch.from_numpy(w), h2)
        ref = single_process_reference(host, stride, off, X, idx, w)
        results[rank] = (bool(np.array_equal(h2.numpy().view(np.uint16).reshape(-1), ref)), ep.last.sent,
                         ep.last.received)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("skew", [False, True])
def test_expert_parallel_world2_matches_single_process(skew):
    world = 2
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), skew, results), nprocs=world, join=True)
    assert set(results.keys()) == {0, 1}
    for r in range(world):
        ok, sent, recv = results[r]
        assert ok, f"rank {r} differs from the single-process layer"
        assert sum(sent) == [5, 3][r] * K
    # what rank a sent to rank b is what rank b received from rank a
    assert results[0][1][1] == results[1][2][0] and results[1][1][0] == results[0][2][1]
    if skew:
        assert results[0][1][1] == 0  # rank 0 routed only to its own experts


def test_single_rank_exchange_is_identity():
    """Without a process group (one GPU) nothing leaves the rank."""
    from edgeexpert_b200 import ep
    assert ep.exchange_counts([7]) == [7]
    t = torch.arange(6).reshape(3, 2)
    assert ep.exchange_rows(t, [3], [3]) is t
