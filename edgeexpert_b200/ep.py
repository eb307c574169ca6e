"""Expert-parallel routed MoE: routed experts sharded over the ranks of a
process group in contiguous id ranges (rank r owns experts
[r*E/P, (r+1)*E/P)), tokens owned by the rank that routed them.

The reference has no multi-GPU path (one Apple GPU, experts streamed from
SSD); this is the B200 layout for 2/4/8 GPUs.  The exchange has a fixed
capacity: every rank sends every rank exactly `capacity` rows per layer, one
slot per (owner, token), so the all-to-all splits are equal and known on the
host.  Nothing is read back to the host and every buffer is allocated once,
so a whole layer (or a stack of them) can be captured in one CUDA graph.

One layer on every rank:

1. tf_ep_dispatch_pack: slot (r, t) carries token t's fp16 row and a header
   with its routing slots that live on rank r (local expert id, weight);
   a token reaches an owner once, however many of its experts live there;
2. all-to-all (equal splits) to the owners;
3. tf_ep_dispatch_unpack: received headers -> [rows][top_k] routing, with
   UINT32_MAX for slots of other ranks;
4. tf_moe_route_sort + tf_moe_grouped_routed over the received rows: the
   reference's grouped gate/up/GELU and down (prefill.metal:336-440,598-670),
   one fp16 partial per (row, slot);
5. tf_ep_expert_combine: per received row, fp32 sum in slot order of
   fma(w, partial) over its slots on this rank;
6. all-to-all of the fp32 rows back to their senders;
7. tf_ep_return_reduce: h2[t] = half(sum over owner ranks in rank order).

Compared with the single-GPU token-major reduce (prefill.metal:575-596, one
fp32 fma chain over the k slots in rank order) the fp32 sum is regrouped by
owner rank, so results agree to fp32 rounding, not bit for bit.

The collectives go through torch.distributed (NCCL between GPUs, gloo in the
CPU tests); the device work goes through `ops`, by default the CUDA kernels
of libtfcuda.so.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ._lib import Context, lib, ptr, stream_ptr

ROW_HEADER_BYTES = 64  # sizeof(tf_ep_row_header)
EMPTY_SLOT = 0xFFFFFFFF


def row_bytes(d: int) -> int:
    """Bytes of one dispatch row: d fp16 values + tf_ep_row_header."""
    return 2 * d + ROW_HEADER_BYTES


def exchange_equal(send: torch.Tensor, recv: torch.Tensor, group=None) -> torch.Tensor:
    """All-to-all with equal splits along dim 0 (world blocks of the same size).
    With one rank (or no process group) the send buffer is returned as is."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return send
    dist.all_to_all_single(recv, send, group=group)
    return recv


@dataclass
class EPBuffers:
    """Every device buffer of one expert-parallel layer, allocated once."""

    send: torch.Tensor      # uint8 [world*capacity, row_bytes]
    recv: torch.Tensor      # uint8 [world*capacity, row_bytes]
    ids: torch.Tensor       # int32 [world*capacity, K]
    w: torch.Tensor         # fp16  [world*capacity, K]
    act: torch.Tensor       # fp16  [world*capacity*K, f]
    part: torch.Tensor      # fp16  [world*capacity*K, d]
    ret: torch.Tensor       # fp32  [world*capacity, d]
    back: torch.Tensor      # fp32  [world*capacity, d]
    routes: object          # DeviceRoutes of the received rows
    # local pairs the grouped experts should expect: each sender's tokens
    # spread their K slots over every rank, so capacity * K (not rows * K)
    expected_pairs: int = 0


class CudaOps:
    """The device work of an expert-parallel layer on one GPU (libtfcuda.so)."""

    def __init__(self, context: Context):
        self.ctx = context

    def alloc(self, world, capacity, K, d, f, num_local, device) -> EPBuffers:
        from .prefill import DeviceRoutes
        rows = world * capacity
        rb = row_bytes(d)
        n = max(rows * K, 1)
        routes = DeviceRoutes(torch.empty(n, 4, dtype=torch.int32, device=device),
                              torch.empty(num_local, dtype=torch.int32, device=device),
                              torch.empty(num_local, dtype=torch.int32, device=device),
                              torch.empty(num_local, 3, dtype=torch.int32, device=device),
                              torch.empty(1, dtype=torch.int32, device=device),
                              torch.empty(num_local, 4, dtype=torch.int32, device=device),
                              torch.empty(1, dtype=torch.int32, device=device))
        return EPBuffers(torch.zeros(rows, rb, dtype=torch.uint8, device=device),
                         torch.zeros(rows, rb, dtype=torch.uint8, device=device),
                         torch.empty(rows, K, dtype=torch.int32, device=device),
                         torch.empty(rows, K, dtype=torch.float16, device=device),
                         torch.empty(n, f, dtype=torch.float16, device=device),
                         torch.empty(n, d, dtype=torch.float16, device=device),
                         torch.empty(rows, d, dtype=torch.float32, device=device),
                         torch.empty(rows, d, dtype=torch.float32, device=device),
                         routes, capacity * K)

    def dispatch_pack(self, hidden, expert_ids, weights, T, K, E, per_rank, world, capacity, send, stream=None):
        d = hidden.shape[1]
        st = lib().tf_ep_dispatch_pack(self.ctx.handle, ptr(hidden), hidden.stride(0), ptr(expert_ids), ptr(weights),
                                       T, K, E, per_rank, world, capacity, d, ptr(send), stream_ptr(stream))
        self.ctx.check(st, "tf_ep_dispatch_pack")

    def unpack(self, recv, rows, d, K, ids, w, stream=None):
        st = lib().tf_ep_dispatch_unpack(self.ctx.handle, ptr(recv), rows, d, K, ptr(ids), ptr(w), stream_ptr(stream))
        self.ctx.check(st, "tf_ep_dispatch_unpack")

    def experts(self, pool, buf: EPBuffers, recv, rows, K, stream=None):
        """buf.ret[i] = sum over row i's slots here of w * down(gelu(gate.x)*up.x)."""
        from .prefill import PrefillGroupedRoutedMoE, route_sort
        d = pool.d
        route_sort(buf.ids, buf.w, rows, K, pool.num_experts, 16, stream=stream, context=self.ctx, out=buf.routes)
        PrefillGroupedRoutedMoE(self.ctx).encode(pool, buf.routes, recv, buf.act, buf.part, rows, K,
                                                 hidden_stride=row_bytes(d) // 2, stream=stream,
                                                 expected_pairs=buf.expected_pairs)
        st = lib().tf_ep_expert_combine(self.ctx.handle, ptr(buf.part), ptr(buf.ids), ptr(buf.w), rows, K, d,
                                        ptr(buf.ret), stream_ptr(stream))
        self.ctx.check(st, "tf_ep_expert_combine")

    def reduce(self, back, world, capacity, T, h2, stream=None):
        d = h2.shape[1]
        st = lib().tf_ep_return_reduce(self.ctx.handle, ptr(back), world, capacity, T, d, ptr(h2), h2.stride(0),
                                       stream_ptr(stream))
        self.ctx.check(st, "tf_ep_return_reduce")


class P2PExchange:
    """Peer-memory buffers of the fixed-capacity exchange (one set, shared by
    every layer): this rank's receive rows, return rows and arrival counters,
    allocated once with tf_ep_ipc_alloc, and device arrays of every rank's
    buffer pointers (the peers' opened through CUDA IPC).  The data path then
    needs no collective: the dispatch and combine kernels store into the
    peers' buffers and signal their counters (tf_ep_*_p2p)."""

    def __init__(self, world: int, rank: int, capacity: int, d: int, group=None, context: Context | None = None,
                 device=None):
        self.ctx = context or Context.get(torch.cuda.current_device())
        self.world, self.rank, self.capacity, self.d = world, rank, capacity, d
        rows = world * capacity
        sizes = (rows * row_bytes(d), rows * d * 4, int(lib().tf_ep_flag_bytes(world)))
        self.own, handles = [], []
        for nbytes in sizes:
            ptr_out, h = C.c_void_p(), (C.c_uint8 * 64)()
            self.ctx.check(lib().tf_ep_ipc_alloc(self.ctx.handle, nbytes, C.byref(ptr_out), h), "tf_ep_ipc_alloc")
            self.own.append(ptr_out.value)
            handles.append(bytes(h))
        self.recv, self.back, self.flags = self.own
        allh = [None] * world
        if world > 1:
            dist.all_gather_object(allh, handles, group=group)
        else:
            allh = [handles]
        self.opened = []
        tables = []
        for i in range(3):
            ptrs = []
            for r in range(world):
                if r == rank:
                    ptrs.append(self.own[i])
                    continue
                pp = C.c_void_p()
                hb = (C.c_uint8 * 64).from_buffer_copy(allh[r][i])
                self.ctx.check(lib().tf_ep_ipc_open(self.ctx.handle, hb, C.byref(pp)), "tf_ep_ipc_open")
                self.opened.append(pp.value)
                ptrs.append(pp.value)
            tables.append(torch.tensor(ptrs, dtype=torch.int64, device=device))
        self.peer_recv, self.peer_back, self.peer_flags = tables

    def close(self):
        for pp in self.opened:
            lib().tf_ep_ipc_close(self.ctx.handle, C.c_void_p(pp))
        for pp in self.own:
            lib().tf_ep_ipc_free(self.ctx.handle, C.c_void_p(pp))
        self.opened, self.own = [], []


@dataclass
class EPStats:
    rows_per_rank: int  # slots sent to (and received from) every rank


class ExpertParallelMoE:
    """Routed experts of one MoE layer sharded over `group`.

    `experts_local` holds this rank's E/P experts (local ids 0..E/P-1 are
    global ids rank*E/P ...).  `forward` takes this rank's T <= capacity
    tokens with their routing (device [T][K] ids and fp16 weights, as
    tf_router_topk_batched writes them) and writes the routed output h2 [T][d]
    for those tokens.  Every rank must use the same capacity.
    """

    def __init__(self, experts_local, num_experts: int, top_k: int, capacity: int, d: int, f: int, group=None,
                 ops=None, context: Context | None = None, device=None, p2p: P2PExchange | None = None):
        """`p2p` (a P2PExchange of the same capacity and d) replaces the two
        NCCL all-to-alls with peer-memory stores; it may be shared by layers."""
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        if top_k > 8:
            raise ValueError("the dispatch header holds at most 8 routing slots")
        self.E = num_experts
        self.per_rank = num_experts // self.world
        self.K = top_k
        self.capacity = capacity
        self.d, self.f = d, f
        self.pool = experts_local
        if ops is None:
            ops = CudaOps(context or Context.get(torch.cuda.current_device()))
        self.ops = ops
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
        self.buf = ops.alloc(self.world, capacity, top_k, d, f, self.per_rank, device)
        self.p2p = p2p if self.world > 1 else None
        self.last = EPStats(capacity)

    def forward(self, hidden, expert_ids, weights, h2, stream=None):
        T = hidden.shape[0]
        if T > self.capacity:
            raise ValueError(f"{T} tokens exceed the dispatch capacity {self.capacity}")
        b, rows = self.buf, self.world * self.capacity
        if self.p2p is not None:
            return self._forward_p2p(hidden, expert_ids, weights, h2, T, rows, stream)
        self.ops.dispatch_pack(hidden, expert_ids, weights, T, self.K, self.E, self.per_rank, self.world,
                               self.capacity, b.send, stream)
        recv = exchange_equal(b.send, b.recv, self.group)
        self.ops.unpack(recv, rows, self.d, self.K, b.ids, b.w, stream)
        self.ops.experts(self.pool, b, recv, rows, self.K, stream)
        back = exchange_equal(b.ret, b.back, self.group)
        self.ops.reduce(back, self.world, self.capacity, T, h2, stream)
        return h2

    def _forward_p2p(self, hidden, expert_ids, weights, h2, T, rows, stream):
        x, b, ctx = self.p2p, self.buf, self.ops.ctx
        sp = stream_ptr(stream)
        d, K = self.d, self.K
        ctx.check(lib().tf_ep_dispatch_p2p(ctx.handle, ptr(hidden), hidden.stride(0) if T else d, ptr(expert_ids),
                                           ptr(weights), T, K, self.E, self.per_rank, self.world, self.rank,
                                           self.capacity, d, ptr(x.peer_recv), ptr(x.peer_flags), C.c_void_p(x.flags),
                                           sp), "tf_ep_dispatch_p2p")
        ctx.check(lib().tf_ep_dispatch_unpack_p2p(ctx.handle, C.c_void_p(x.recv), C.c_void_p(x.flags), self.world,
                                                  self.capacity, d, K, ptr(b.ids), ptr(b.w), sp),
                  "tf_ep_dispatch_unpack_p2p")
        from .prefill import PrefillGroupedRoutedMoE, route_sort
        route_sort(b.ids, b.w, rows, K, self.pool.num_experts, 16, stream=stream, context=ctx, out=b.routes)
        PrefillGroupedRoutedMoE(ctx).encode(self.pool, b.routes, x.recv, b.act, b.part, rows, K,
                                            hidden_stride=row_bytes(d) // 2, stream=stream,
                                            expected_pairs=b.expected_pairs)
        ctx.check(lib().tf_ep_combine_p2p(ctx.handle, ptr(b.part), ptr(b.ids), ptr(b.w), self.world, self.rank,
                                          self.capacity, K, d, ptr(x.peer_back), ptr(x.peer_flags),
                                          C.c_void_p(x.flags), sp), "tf_ep_combine_p2p")
        ctx.check(lib().tf_ep_return_reduce_p2p(ctx.handle, C.c_void_p(x.back), C.c_void_p(x.flags), self.world,
                                                self.capacity, T, d, ptr(h2) if T else C.c_void_p(0),
                                                h2.stride(0) if T else d, sp), "tf_ep_return_reduce_p2p")
        return h2
