"""Batched / prefill MoE operators (mirror of Sources/TurboFieldfare/Kernels/Prefill/MoE).

* ``PrefillMoEGrouping.group_token_expert_pairs`` -> PrefillMoEGrouping.groupTokenExpertPairs
  (PrefillMoEGrouping.swift:91-192), host memory, same validation errors.
* ``route_sort``                                  -> the same grouping on the device from the
  router's token-major ids/weights (no host round trip).
* ``PrefillRouter.make_token_expert_pairs``       -> PrefillRouter.makeTokenExpertPairs (host).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import (TF_ERR_GROUPING, TF_OK, Context, GroupingError as _GE, MoEGroup, MoETile, TFError,
                   TokenExpertPair, lib, ptr, stream_ptr)

PAIR_DTYPE = np.dtype([("token", "<u4"), ("expert", "<u4"), ("rank", "<u4"), ("weight_bits", "<u4")])
GROUP_DTYPE = np.dtype([("expert", "<u4"), ("pair_start", "<u4"), ("pair_count", "<u4")])
TILE_DTYPE = np.dtype([("group_start", "<u4"), ("group_count", "<u4"), ("pair_start", "<u4"),
                       ("pair_count", "<u4")])

GROUPING_ERRORS = {
    1: "invalidQueryCount", 2: "invalidTopK", 3: "invalidNumExperts", 4: "invalidTileExpertCount",
    5: "pairCountMismatch", 6: "tokenOutOfRange", 7: "rankOutOfRange", 8: "expertOutOfRange",
    9: "duplicateTokenRank", 10: "expertSortKeyCountMismatch",
}


class PrefillMoEGroupingError(ValueError):
    """PrefillMoEGroupingError (PrefillMoEGrouping.swift:52-88)."""

    def __init__(self, code: int, a: int, b: int):
        self.code, self.a, self.b = code, a, b
        self.name = GROUPING_ERRORS.get(code, str(code))
        super().__init__(f"{self.name}({a}, {b})")


@dataclass
class PrefillMoEGroupedRoutes:
    sorted_pairs: np.ndarray
    per_expert_offsets: np.ndarray
    per_expert_counts: np.ndarray
    groups: np.ndarray
    tiles: np.ndarray
    query_count: int

    @property
    def max_pairs_per_expert(self) -> int:
        return int(self.groups["pair_count"].max()) if len(self.groups) else 0

    @property
    def max_pairs_per_tile(self) -> int:
        return int(self.tiles["pair_count"].max()) if len(self.tiles) else 0

    @property
    def max_live_experts_per_tile(self) -> int:
        return int(self.tiles["group_count"].max()) if len(self.tiles) else 0


class PrefillMoEGrouping:
    @staticmethod
    def group_token_expert_pairs(pairs: np.ndarray, query_count: int, top_k: int, num_experts: int,
                                 tile_expert_count: int = 16, expert_sort_keys=None) -> PrefillMoEGroupedRoutes:
        pairs = np.ascontiguousarray(pairs, PAIR_DTYPE)
        n = pairs.size
        E = max(int(num_experts), 1)
        sorted_ = np.zeros(max(n, 1), PAIR_DTYPE)
        offsets = np.zeros(E, np.uint32)
        counts = np.zeros(E, np.uint32)
        groups = np.zeros(E, GROUP_DTYPE)
        tiles = np.zeros(E, TILE_DTYPE)
        ng, nt = C.c_uint32(0), C.c_uint32(0)
        err = _GE()
        keys = None if expert_sort_keys is None else np.ascontiguousarray(expert_sort_keys, np.uint64)
        st = lib().tf_group_token_expert_pairs(
            C.c_void_p(pairs.ctypes.data if n else 0), n, query_count, top_k, num_experts, tile_expert_count,
            C.c_void_p(0 if keys is None else keys.ctypes.data), 0 if keys is None else keys.size,
            C.c_void_p(sorted_.ctypes.data), C.c_void_p(offsets.ctypes.data), C.c_void_p(counts.ctypes.data),
            C.c_void_p(groups.ctypes.data), C.byref(ng), C.c_void_p(tiles.ctypes.data), C.byref(nt), C.byref(err))
        if st == TF_ERR_GROUPING:
            raise PrefillMoEGroupingError(err.code, err.a, err.b)
        if st != TF_OK:
            raise TFError(st, "tf_group_token_expert_pairs")
        return PrefillMoEGroupedRoutes(sorted_[:n], offsets[:num_experts], counts[:num_experts],
                                       groups[:ng.value], tiles[:nt.value], query_count)

    groupTokenExpertPairs = group_token_expert_pairs


class PrefillRouter:
    @staticmethod
    def make_token_expert_pairs(indices: np.ndarray, weights_f16: np.ndarray, query_count: int,
                                top_k: int) -> np.ndarray:
        """Token-major pairs {token, expert, rank, weightBits} (PrefillRouter.swift:91-111)."""
        idx = np.asarray(indices, np.uint32).reshape(query_count, top_k)
        w = np.asarray(weights_f16).view(np.uint16).reshape(query_count, top_k)
        out = np.zeros(query_count * top_k, PAIR_DTYPE)
        out["token"] = np.repeat(np.arange(query_count, dtype=np.uint32), top_k)
        out["expert"] = idx.reshape(-1)
        out["rank"] = np.tile(np.arange(top_k, dtype=np.uint32), query_count)
        out["weight_bits"] = w.reshape(-1).astype(np.uint32)
        return out

    makeTokenExpertPairs = make_token_expert_pairs

    def __init__(self, context: Context | None = None):
        import torch
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode_gemma4_block(self, weights, scales, biases, hidden, effective_scale, per_expert_scale, out_indices,
                            out_weights, query_count: int, num_experts: int, d: int, top_k: int,
                            hidden_stride_elements: int | None = None, stream=None, out_logits=None):
        """Router + top-k for `query_count` tokens (PrefillRouter.encodeGemma4Block).
        `out_logits` (optional, float32[query_count][num_experts] on the device)
        receives every token's fp32 logits."""
        from .quant import scale_type_of
        hs = hidden_stride_elements if hidden_stride_elements is not None else d
        head = (self.ctx.handle, ptr(weights), ptr(scales), ptr(biases), ptr(hidden), hs, ptr(effective_scale),
                ptr(per_expert_scale), ptr(out_indices), ptr(out_weights))
        tail = (query_count, num_experts, d, top_k, scale_type_of(scales), stream_ptr(stream))
        if out_logits is not None:
            st = lib().tf_router_topk_batched_with_logits(*head, ptr(out_logits), *tail)
        else:
            st = lib().tf_router_topk_batched(*head, *tail)
        self.ctx.check(st, "PrefillRouter.encodeGemma4Block")

    encodeGemma4Block = encode_gemma4_block


@dataclass
class DeviceRoutes:
    """Device-resident grouping outputs (torch tensors)."""

    sorted_pairs: "object"  # int32 [T*K, 4]
    offsets: "object"
    counts: "object"
    groups: "object"        # int32 [E, 3]
    n_groups: "object"
    tiles: "object"         # int32 [E, 4]
    n_tiles: "object"


def route_sort(expert_ids, weights, T: int, top_k: int, num_experts: int, tile_expert_count: int = 16,
               sort_keys=None, stream=None, context: Context | None = None, out: DeviceRoutes | None = None):
    """Device grouping of the router's [T][top_k] routing (tf_moe_route_sort)."""
    import torch
    ctx = context or Context.get(expert_ids.device.index or 0)
    dev = expert_ids.device
    if out is None:
        n = max(T * top_k, 1)
        out = DeviceRoutes(torch.empty(n, 4, dtype=torch.int32, device=dev),
                           torch.empty(num_experts, dtype=torch.int32, device=dev),
                           torch.empty(num_experts, dtype=torch.int32, device=dev),
                           torch.empty(num_experts, 3, dtype=torch.int32, device=dev),
                           torch.empty(1, dtype=torch.int32, device=dev),
                           torch.empty(num_experts, 4, dtype=torch.int32, device=dev),
                           torch.empty(1, dtype=torch.int32, device=dev))
    st = lib().tf_moe_route_sort(ctx.handle, ptr(expert_ids), ptr(weights), T, top_k, num_experts,
                                 tile_expert_count, ptr(sort_keys), ptr(out.sorted_pairs), ptr(out.offsets),
                                 ptr(out.counts), ptr(out.groups), ptr(out.n_groups), ptr(out.tiles),
                                 ptr(out.n_tiles), stream_ptr(stream))
    ctx.check(st, "tf_moe_route_sort")
    return out


class PrefillInt4QMM:
    """Dense int4 x fp16 GEMM on the tensor cores (PrefillInt4QMM.encode,
    PrefillPrimitives.swift:73-122; MPPPrefillInt4QMM.encode, MPPPrefillInt4QMM.swift:34-78)."""

    def __init__(self, context: Context | None = None):
        import torch
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, weights, scales, biases, x, y, t: int, n: int, k: int, bits: int = 4,
               x_stride: int = 0, y_stride: int = 0, stream=None):
        from .quant import scale_type_of
        if bits != 4:
            raise TFError(3, f"unsupported prefill QMM bits {bits}")
        st = lib().tf_int4_qmm(self.ctx.handle, ptr(weights), ptr(scales), ptr(biases), ptr(x), ptr(y), t, n, k,
                               x_stride, y_stride, scale_type_of(scales), stream_ptr(stream))
        self.ctx.check(st, "PrefillInt4QMM.encode")


class PrefillSharedExpert:
    """Shared expert over T prefill tokens (per-token SharedExpertRuntime arithmetic)."""

    def __init__(self, context: Context | None = None):
        import torch
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, x, gate, up, down, act_scratch, y, t: int, x_stride: int = 0, y_stride: int = 0, stream=None):
        from .quant import scale_type_of
        g, u, dn = gate.as_c(), up.as_c(), down.as_c()
        st = lib().tf_prefill_shared_expert(self.ctx.handle, ptr(x), x_stride, C.byref(g), C.byref(u), C.byref(dn),
                                            ptr(act_scratch), ptr(y), y_stride, t, scale_type_of(gate.scales),
                                            stream_ptr(stream))
        self.ctx.check(st, "PrefillSharedExpert.encode")


class PrefillGroupedRoutedMoE:
    """Grouped routed experts for a prefill chunk (PrefillGroupedRoutedMoE.encodeStreamedBatched,
    PrefillGroupedRoutedMoE.swift:446-527): every group of the device routes in one pair of launches."""

    def __init__(self, context: Context | None = None):
        import torch
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, experts, routes: "DeviceRoutes", hidden, act_scratch, route_partials, t: int, top_k: int,
               hidden_stride: int = 0, stream=None, expected_pairs: int = 0):
        """`expected_pairs` (0: t * top_k) is the caller's estimate of the
        pairs the groups hold; it only selects the kernel."""
        st = lib().tf_moe_grouped_routed_expected(
            self.ctx.handle, ptr(experts.blob), experts.stride, experts.num_experts, C.byref(experts.offsets),
            ptr(routes.sorted_pairs), ptr(routes.groups), ptr(routes.n_groups), ptr(hidden), hidden_stride,
            ptr(act_scratch), ptr(route_partials), t, experts.d, experts.f, top_k, expected_pairs,
            0 if experts.scale_dtype == _bf16() else 1, stream_ptr(stream))
        self.ctx.check(st, "PrefillGroupedRoutedMoE.encodeStreamedBatched")

    encodeStreamedBatched = encode


class PrefillMoE:
    @staticmethod
    def encode_reduce_token_major(route_partials, routing_weights, h2, t: int, top_k: int, d: int, stream=None,
                                  context: Context | None = None):
        """PrefillMoE.encodeReduceTokenMajor (PrefillMoE.swift:11-40)."""
        ctx = context or Context.get(h2.device.index or 0)
        st = lib().tf_moe_reduce_token_major(ctx.handle, ptr(route_partials), ptr(routing_weights), ptr(h2), t, top_k,
                                             d, stream_ptr(stream))
        ctx.check(st, "PrefillMoE.encodeReduceTokenMajor")

    encodeReduceTokenMajor = encode_reduce_token_major


def _bf16():
    import torch
    return torch.bfloat16
