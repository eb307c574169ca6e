"""Expert-parallel routed MoE: routed experts sharded over the ranks of a
process group in contiguous id ranges (rank r owns experts
[r*E/P, (r+1)*E/P)), tokens owned by the rank that routed them.

The reference has no multi-GPU path (one Apple GPU, experts streamed from
SSD); this is the B200 layout for 2/4/8 GPUs.  One step on every rank:

1. sort its token->expert pairs by expert on the device (tf_moe_route_sort):
   the pairs for each destination rank are then one contiguous range;
2. exchange the per-destination pair counts (all-to-all of P integers);
3. pack the pairs' token rows and local expert ids (tf_ep_pack) and send them
   to the owners (all-to-all-v);
4. on the owner: group the received rows by local expert (tf_moe_route_sort
   with K = 1) and run the grouped gate/up/GELU and down GEMMs on them
   (tf_moe_grouped_routed with top_k = 1: one output row per received row);
5. send the output rows back (all-to-all-v with the splits swapped): they
   arrive in the sender's sorted-pair order;
6. h2[t] = half(sum_r w[t][r] * out[pair(t, r)]) in rank order
   (tf_moe_combine_sorted), the reference's token-major reduce.

The collectives go through torch.distributed (NCCL between GPUs, gloo in the
CPU tests); the device work goes through `ops`, by default the CUDA kernels of
libtfcuda.so.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ._lib import Context, lib, ptr, stream_ptr


def exchange_counts(send_counts, group=None, device=None) -> list[int]:
    """recv[r] = what rank r sends here, given send[r] = what this rank sends to r."""
    if not dist.is_initialized():  # one rank: everything stays here
        return [int(v) for v in send_counts]
    p = dist.get_world_size(group)
    dev = device if device is not None else torch.device("cpu")
    s = torch.as_tensor(list(send_counts), dtype=torch.int64, device=dev)
    if s.numel() != p:
        raise ValueError(f"send_counts has {s.numel()} entries for {p} ranks")
    r = torch.empty_like(s)
    dist.all_to_all_single(r, s, group=group)
    return [int(v) for v in r.cpu().tolist()]


def exchange_rows(send: torch.Tensor, send_counts, recv_counts, group=None) -> torch.Tensor:
    """All-to-all-v of the leading dimension: send[sum(send_counts[:r]) : ...] goes to rank r."""
    if not dist.is_initialized():
        return send
    out = torch.empty((int(sum(recv_counts)),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
    dist.all_to_all_single(out, send.contiguous(), [int(c) for c in recv_counts], [int(c) for c in send_counts],
                           group=group)
    return out


@dataclass
class EPStats:
    sent: list
    received: list


class CudaOps:
    """The device work of an expert-parallel step on one GPU (libtfcuda.so)."""

    def __init__(self, context: Context):
        self.ctx = context

    def route(self, expert_ids, weights, T, K, E):
        from .prefill import route_sort
        return route_sort(expert_ids, weights, T, K, E, 16, context=self.ctx)

    def send_counts(self, routes, E, per_rank, world):
        out = torch.empty(world, dtype=torch.int32, device=routes.counts.device)
        st = lib().tf_ep_send_counts(self.ctx.handle, ptr(routes.counts), E, per_rank, world, ptr(out),
                                     stream_ptr(None))
        self.ctx.check(st, "tf_ep_send_counts")
        return [int(v) for v in out.cpu().tolist()]

    def pack(self, hidden, routes, n, T, per_rank):
        d = hidden.shape[1]
        rows = torch.empty(n, d, dtype=torch.float16, device=hidden.device)
        local = torch.empty(n, dtype=torch.int32, device=hidden.device)
        st = lib().tf_ep_pack(self.ctx.handle, ptr(hidden), hidden.stride(0), ptr(routes.sorted_pairs), n, d, T,
                              per_rank, ptr(rows), ptr(local), stream_ptr(None))
        self.ctx.check(st, "tf_ep_pack")
        return rows, local

    def experts(self, pool, rows, local):
        """out[i] = down_e(gelu(gate_e . rows[i]) * up_e . rows[i]), e = local[i]."""
        from .prefill import PrefillGroupedRoutedMoE
        n = rows.shape[0]
        d = rows.shape[1]
        out = torch.empty(n, d, dtype=torch.float16, device=rows.device)
        if n == 0:
            return out
        ones = torch.ones(n, dtype=torch.float16, device=rows.device)
        routes = self.route(local, ones, n, 1, pool.num_experts)
        act = torch.empty(n, pool.f, dtype=torch.float16, device=rows.device)
        PrefillGroupedRoutedMoE(self.ctx).encode(pool, routes, rows, act, out, n, 1)
        return out

    def combine(self, routes, back, weights, h2, T, K):
        d = h2.shape[1]
        inv = torch.empty(max(T * K, 1), dtype=torch.int32, device=h2.device)
        src = back if back.numel() else torch.empty(1, d, dtype=torch.float16, device=h2.device)
        st = lib().tf_moe_combine_sorted(self.ctx.handle, ptr(routes.sorted_pairs), ptr(src), ptr(weights),
                                         ptr(inv), ptr(h2), T, K, d, stream_ptr(None))
        self.ctx.check(st, "tf_moe_combine_sorted")


class ExpertParallelMoE:
    """Routed experts of one MoE layer sharded over `group`.

    `experts_local` holds this rank's E/P experts (local ids 0..E/P-1 are
    global ids rank*E/P ...).  `forward` takes this rank's tokens with their
    routing (device [T][K] ids and fp16 weights, as tf_router_topk_batched
    writes them) and returns the routed output h2 [T][d] for those tokens.
    """

    def __init__(self, experts_local, num_experts: int, top_k: int, group=None, ops=None,
                 context: Context | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.E = num_experts
        self.per_rank = num_experts // self.world
        self.K = top_k
        self.pool = experts_local
        if ops is None:
            ops = CudaOps(context or Context.get(torch.cuda.current_device()))
        self.ops = ops
        self.last = None

    def forward(self, hidden, expert_ids, weights, h2):
        T = hidden.shape[0]
        routes = self.ops.route(expert_ids, weights, T, self.K, self.E)
        send = self.ops.send_counts(routes, self.E, self.per_rank, self.world)
        recv = exchange_counts(send, self.group, device=hidden.device)
        rows, local = self.ops.pack(hidden, routes, T * self.K, T, self.per_rank)
        r_rows = exchange_rows(rows, send, recv, self.group)
        r_local = exchange_rows(local, send, recv, self.group)
        out = self.ops.experts(self.pool, r_rows, r_local)
        back = exchange_rows(out, recv, send, self.group)
        self.ops.combine(routes, back, weights, h2, T, self.K)
        self.last = EPStats(send, recv)
        return h2
