"""Expert-parallel exchange logic on CPU: world_size 2 over gloo.

The device work is replaced by numpy and the C oracle (the tf_ep_row_header
row format, the per-pair expert FFN of prefill.metal:336-440,598-670), so the
test checks the host side of edgeexpert_b200.ep: the fixed-capacity slots,
the two equal-split all-to-alls and the combines.  Each rank's output must
equal a single-process run of the same layer (token-major reduce,
prefill.metal:575-596) within the fp16 bar.
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


def _pack_header(ids, wbits, n, token):
    h = np.zeros(64, np.uint8)
    h[0:32] = np.asarray(ids, np.uint32).view(np.uint8)
    h[32:48] = np.asarray(wbits, np.uint16).view(np.uint8)
    h[48:56] = np.array([n, token], np.uint32).view(np.uint8)
    return h


class OracleOps:
    """CPU stand-in for edgeexpert_b200.ep.CudaOps (same contract): the row
    format of tf_ep_row_header, the per-pair expert FFN of the C oracle
    (prefill.metal:336-440,598-670) and the fp32 combines."""

    def __init__(self, host_experts, lay_stride, off, per_rank, rank):
        self.host, self.stride, self.off = host_experts, lay_stride, off
        self.per_rank, self.rank = per_rank, rank

    def alloc(self, world, capacity, K_, d, f, num_local, device):
        from edgeexpert_b200.ep import EPBuffers, row_bytes
        rows = world * capacity
        return EPBuffers(torch.zeros(rows, row_bytes(d), dtype=torch.uint8),
                         torch.zeros(rows, row_bytes(d), dtype=torch.uint8),
                         torch.zeros(rows, K_, dtype=torch.int64), torch.zeros(rows, K_, dtype=torch.float16),
                         None, None, torch.zeros(rows, d, dtype=torch.float32),
                         torch.zeros(rows, d, dtype=torch.float32), None)

    def dispatch_pack(self, hidden, expert_ids, weights, T, K_, E_, per_rank, world, capacity, send, stream=None):
        d = hidden.shape[1]
        ids = expert_ids.numpy().astype(np.int64).reshape(T, K_)
        wb = weights.numpy().view(np.uint16).reshape(T, K_)
        x = hidden.numpy().view(np.uint8).reshape(T, 2 * d)
        out = send.numpy()
        for r in range(world):
            for t in range(capacity):
                loc = [0xFFFFFFFF] * 8
                wl = [0] * 8
                n = 0
                if t < T:
                    for k in range(K_):
                        if ids[t, k] // per_rank == r:
                            loc[k] = int(ids[t, k] - r * per_rank)
                            wl[k] = int(wb[t, k])
                            n += 1
                row = out[r * capacity + t]
                row[2 * d:] = _pack_header(loc, wl, n, t)
                if n:
                    row[:2 * d] = x[t]

    def unpack(self, recv, rows, d, K_, ids, w, stream=None):
        hdr = recv.numpy()[:rows, 2 * d:]
        ids.copy_(torch.from_numpy(hdr[:, :32].copy().view(np.uint32)[:, :K_].astype(np.int64)))
        w.copy_(torch.from_numpy(hdr[:, 32:48].copy().view(np.float16)[:, :K_]))

    def experts(self, pool, buf, recv, rows, K_, stream=None):
        d = D
        ids = buf.ids.numpy()
        X = recv.numpy()[:rows, :2 * d].copy().view(np.uint16)
        lo = self.rank * self.per_rank
        local_host = self.host[lo:lo + self.per_rank].reshape(-1)
        valid = [(i, k) for i in range(rows) for k in range(K_) if ids[i, k] != 0xFFFFFFFF]
        ret = np.zeros((rows, d), np.float32)
        if valid:
            pairs = np.zeros(len(valid), O.PAIR_DTYPE)
            pairs["token"] = [i for i, _ in valid]
            pairs["rank"] = [k for _, k in valid]
            pairs["expert"] = [ids[i, k] for i, k in valid]
            order = np.lexsort((pairs["rank"], pairs["token"], pairs["expert"]))
            part = O.grouped_routed(local_host, self.stride, self.off, pairs[order], X, d, d, F, K_, rows, 0)
            part = O.f16_to_f32(part.reshape(rows, K_, d))
            wv = buf.w.numpy().astype(np.float32)
            for i in range(rows):
                acc = np.zeros(d, np.float32)
                for k in range(K_):
                    if ids[i, k] != 0xFFFFFFFF:
                        acc = np.float32(wv[i, k]) * part[i, k] + acc  # fp32 (the kernel fuses this fma)
                ret[i] = acc
        buf.ret.copy_(torch.from_numpy(ret))

    def reduce(self, back, world, capacity, T, h2, stream=None):
        b = back.numpy().reshape(world, capacity, -1)
        acc = np.zeros((T, b.shape[2]), np.float32)
        for r in range(world):
            acc = acc + b[r, :T]
        h2.copy_(torch.from_numpy(acc.astype(np.float16)))


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
        ep = ExpertParallelMoE(None, E, K, 5, D, F, ops=ops, device="cpu")
        h2 = torch.empty(X.shape[0], D, dtype=torch.float16)
        ep.forward(torch.from_numpy(X.view(np.float16)), torch.from_numpy(idx), torch.from_numpy(w), h2)
        ref = single_process_reference(host, stride, off, X, idx, w)
        got = h2.numpy().view(np.uint16).reshape(-1)
        err = O.rel_error(O.f16_to_f32(got), O.f16_to_f32(ref))
        # what reached this rank: the number of (token, slot) pairs it owns
        hdr = ep.buf.recv.numpy()[:, 2 * D:]
        n_recv = int(hdr[:, 48:52].copy().view(np.uint32).sum())
        owned = 0
        for r in range(world):
            _, idx_r, _ = tokens_for(r, skew)
            owned += int(np.sum(idx_r // (E // world) == rank))
        results[rank] = (err, n_recv, owned)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("skew", [False, True])
def test_expert_parallel_world2_matches_single_process(skew):
    """Each rank's routed output equals the single-process layer within the
    fp16 bar (the fp32 sum is regrouped by owner rank), and every rank
    receives exactly the (token, slot) pairs whose experts it owns."""
    world = 2
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), skew, results), nprocs=world, join=True)
    assert set(results.keys()) == {0, 1}
    for r in range(world):
        err, n_recv, owned = results[r]
        assert err < 2e-3, f"rank {r}: rel error {err}"
        assert n_recv == owned, (r, n_recv, owned)
    if skew:  # rank 0 routes only to its own experts: rank 1 owns none of them
        assert results[1][2] == int(np.sum(tokens_for(1, True)[1] >= E // 2))


def test_single_rank_exchange_is_identity():
    """Without a process group (one GPU) nothing leaves the rank."""
    from edgeexpert_b200 import ep
    t = torch.arange(6).reshape(3, 2)
    assert ep.exchange_equal(t, torch.empty_like(t)) is t


def test_row_header_is_64_bytes():
    import ctypes as C

    class Hdr(C.Structure):  # tf_ep_row_header
        _fields_ = [("local_expert", C.c_uint32 * 8), ("weight_bits", C.c_uint16 * 8), ("n_valid", C.c_uint32),
                    ("src_token", C.c_uint32), ("reserved", C.c_uint32 * 2)]
    from edgeexpert_b200.ep import ROW_HEADER_BYTES, row_bytes
    assert C.sizeof(Hdr) == ROW_HEADER_BYTES == 64
    assert row_bytes(2816) % 16 == 0
