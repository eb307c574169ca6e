"""Decode-time MoE operators (mirror of Sources/TurboFieldfare/Kernels/MoE).

* ``MoE.encode_router_gemma4``            -> MoE.encodeRouterGemma4 (MoE.swift:147-197)
* ``MoE.encode_routed_phase1``            -> encodeRoutedPersistentPhase1U16Load (MoE.swift:234-266)
* ``MoE.encode_routed_phase2_reduce``     -> encodeRoutedPersistentPhase2Reduce (MoE.swift:312-362)
* ``SharedExpertRuntime.encode``          -> SharedExpertRuntime.encode (SharedExpertInt4.swift:97-137)
* ``moe_decode_layer``                    -> the MoE section of RealForwardRunner.produceToken
                                             with HBM-resident experts (no SSD fetch, no host readback)

Routed experts come either as an :class:`ExpertPool` (one device buffer of
``num_experts`` blobs, addressed by device-side ids) or as a list of per-slot
blob tensors, the reference's ``routedBlobs``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from ._lib import (AffineMatrix, Context, ExpertOffsets, MoELayer, TFError, TF_ERR_INVALID_ARG, lib, ptr,
                   stream_ptr)
from .quant import scale_type_of


@dataclass
class SharedExpertProjection:
    """weights/scales/biases for one projection (SharedExpertInt8.swift:9-31)."""

    weights: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    rows: int
    cols: int
    bits: int = 4

    def as_c(self) -> AffineMatrix:
        return AffineMatrix(self.weights.data_ptr(), self.scales.data_ptr(), self.biases.data_ptr(),
                            self.rows, self.cols, self.bits)


@dataclass
class ExpertPool:
    """HBM-resident routed experts: expert e's blob at ``blob + e*stride``."""

    blob: torch.Tensor  # uint8, num_experts * stride bytes
    stride: int
    num_experts: int
    offsets: ExpertOffsets
    d: int
    f: int
    scale_dtype: torch.dtype = torch.bfloat16
    bits: int = 4  # packed routed-weight width: 4, or 2 / 3 (the rebits output)


class MoE:
    max_streamed_experts = 8

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode_router_gemma4(self, weights, scales, biases, hidden, effective_scale, per_expert_scale,
                             out_indices, out_weights, num_experts: int, d: int, top_k: int, stream=None,
                             out_logits=None):
        """Router + top-k (MoE.encodeRouterGemma4).  `out_logits` (optional,
        float32[num_experts] on the device) receives the fp32 router logits."""
        if out_logits is not None:
            st = lib().tf_router_topk_with_logits(
                self.ctx.handle, ptr(weights), ptr(scales), ptr(biases), ptr(hidden), ptr(effective_scale),
                ptr(per_expert_scale), ptr(out_indices), ptr(out_weights), ptr(out_logits), num_experts, d, top_k,
                scale_type_of(scales), stream_ptr(stream))
        else:
            st = lib().tf_router_topk(self.ctx.handle, ptr(weights), ptr(scales), ptr(biases), ptr(hidden),
                                      ptr(effective_scale), ptr(per_expert_scale), ptr(out_indices),
                                      ptr(out_weights), num_experts, d, top_k, scale_type_of(scales),
                                      stream_ptr(stream))
        self.ctx.check(st, "MoE.encodeRouterGemma4")

    encodeRouterGemma4 = encode_router_gemma4

    @staticmethod
    def _source(experts, expert_ids, top_k):
        if isinstance(experts, ExpertPool):
            if expert_ids is None:
                raise TFError(TF_ERR_INVALID_ARG, "an ExpertPool needs device expert_ids")
            return (ptr(experts.blob), experts.stride, experts.num_experts, ptr(expert_ids), None,
                    experts.offsets, experts.scale_dtype)
        blobs, offsets, scale_dtype = experts
        arr = (C.c_void_p * max(1, len(blobs)))(*[b.data_ptr() for b in blobs])
        return (C.c_void_p(0), 0, 0, C.c_void_p(0), arr, offsets, scale_dtype)

    @staticmethod
    def _stype(dt):
        return 1 if dt == torch.float16 else 0

    def encode_routed_phase1(self, experts, x, acts, d: int, f: int, top_k: int, expert_ids=None, stream=None,
                             bits: int = 4):
        """bits 2 / 3: moe_phase1_gate_up_act_b2/_b3 (the `bits` argument of MoE.swift:244)."""
        pool, stride, ne, ids, blobs, off, sdt = self._source(experts, expert_ids, top_k)
        if bits == 4:
            st = lib().tf_moe_phase1(self.ctx.handle, pool, stride, ne, ids, blobs, C.byref(off), ptr(x), ptr(acts),
                                     d, f, top_k, self._stype(sdt), stream_ptr(stream))
        else:
            st = lib().tf_moe_phase1_bits(self.ctx.handle, bits, pool, stride, ne, ids, blobs, C.byref(off), ptr(x),
                                          ptr(acts), d, f, top_k, self._stype(sdt), stream_ptr(stream))
        self.ctx.check(st, "MoE.encodeRoutedPersistentPhase1U16Load")

    def encode_routed_phase2_reduce(self, experts, acts, routing_weights, residual, y, d: int, f: int, top_k: int,
                                    expert_ids=None, stream=None, bits: int = 4):
        """bits 2 / 3: moe_phase2_down_reduce_b2/_b3 (the `bits` argument of MoE.swift:324)."""
        pool, stride, ne, ids, blobs, off, sdt = self._source(experts, expert_ids, top_k)
        if bits == 4:
            st = lib().tf_moe_phase2(self.ctx.handle, pool, stride, ne, ids, blobs, C.byref(off), ptr(acts),
                                     ptr(routing_weights), ptr(residual), ptr(y), d, f, top_k, self._stype(sdt),
                                     stream_ptr(stream))
        else:
            st = lib().tf_moe_phase2_bits(self.ctx.handle, bits, pool, stride, ne, ids, blobs, C.byref(off),
                                          ptr(acts), ptr(routing_weights), ptr(residual), ptr(y), d, f, top_k,
                                          self._stype(sdt), stream_ptr(stream))
        self.ctx.check(st, "MoE.encodeRoutedPersistentPhase2Reduce")


class SharedExpertRuntime:
    """Shared (dense) expert: int4 or int8 weights (SharedExpertInt4.swift:97-137)."""

    def __init__(self, weight_bits: int, context: Context | None = None):
        if weight_bits not in (4, 8):
            raise TFError(3, f"SharedExpert unsupported weight bits: {weight_bits}")
        self.weight_bits = weight_bits
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, x, gate: SharedExpertProjection, up: SharedExpertProjection, down: SharedExpertProjection,
               y, scratch_act, stream=None):
        g, u, dn = gate.as_c(), up.as_c(), down.as_c()
        st = lib().tf_shared_expert(self.ctx.handle, ptr(x), C.byref(g), C.byref(u), C.byref(dn), ptr(y),
                                    ptr(scratch_act), scale_type_of(gate.scales), stream_ptr(stream))
        self.ctx.check(st, "SharedExpertRuntime.encode")


@dataclass
class MoELayerWeights:
    """Everything one decode MoE layer reads, resident on one GPU."""

    router_w: torch.Tensor
    router_s: torch.Tensor
    router_b: torch.Tensor
    eff_scale: torch.Tensor  # bf16 [d]
    per_expert_scale: torch.Tensor  # bf16 [E]
    experts: ExpertPool
    shared_gate: SharedExpertProjection | None
    shared_up: SharedExpertProjection | None
    shared_down: SharedExpertProjection | None
    top_k: int = 8

    def as_c(self) -> MoELayer:
        L = MoELayer()
        L.router_w, L.router_s, L.router_b = (self.router_w.data_ptr(), self.router_s.data_ptr(),
                                              self.router_b.data_ptr())
        L.eff_scale = self.eff_scale.data_ptr()
        L.per_expert_scale = self.per_expert_scale.data_ptr()
        L.expert_pool = self.experts.blob.data_ptr()
        L.expert_stride = self.experts.stride
        L.num_experts = self.experts.num_experts
        L.offsets = self.experts.offsets
        if self.shared_gate is not None:
            L.shared_gate, L.shared_up, L.shared_down = (self.shared_gate.as_c(), self.shared_up.as_c(),
                                                         self.shared_down.as_c())
        L.d, L.f, L.top_k = self.experts.d, self.experts.f, self.top_k
        L.scale_type = 1 if self.experts.scale_dtype == torch.float16 else 0
        return L


def moe_decode_layer(layer: MoELayerWeights, router_x, x, y, residual=None, out_indices=None, out_weights=None,
                     stream=None, context: Context | None = None, c_layer: MoELayer | None = None):
    """router -> routed gate/up -> down + combine (+ shared), 3 launches, no host sync."""
    ctx = context or Context.get(torch.cuda.current_device())
    L = c_layer if c_layer is not None else layer.as_c()
    st = lib().tf_moe_decode_layer(ctx.handle, C.byref(L), ptr(router_x), ptr(x), ptr(residual), ptr(y),
                                   ptr(out_indices), ptr(out_weights), stream_ptr(stream))
    ctx.check(st, "moe_decode_layer")
