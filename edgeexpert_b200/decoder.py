"""The dense decode stack around the MoE FFN: one Gemma 4 decoder layer per
call (RealForwardRunner.produceToken,
Sources/TurboFieldfare/Runtime/Inference/RealForwardRunner.swift:2240-2480)
and the LM head with greedy selection, on HBM-resident weights and an fp16
KV cache.  Every step is device work enqueued on one stream; nothing is read
back, so a whole step (all layers + LM head) is captured in one CUDA graph.

Per layer, for T tokens (T independent sequences at the same position):

  normed  = rmsnorm_bf16w(h, input_norm)                       tf_rmsnorm
  q, k, v = int4 GEMVs of normed (k, v written into the cache)  tf_affine_gemv_batched / tf_int4_qmm
  q, k, v = per-head norms + NeoX RoPE                          tf_qkv_epilogue
  attn    = split-KV GQA attention over [0, pos]                tf_attention_decode
  o       = o_proj(attn)                                        int4 GEMV / GEMM
  h, dense_x, routed_x, router_x = post-attention setup         tf_post_attn_setup
  h1      = shared expert(dense_x)                              tf_shared_expert / tf_prefill_shared_expert
  h2      = routed experts(routed_x, router(router_x))          tf_moe_decode_layer (T = 1) or the grouped path
  h       = layer tail(h2, h1)   (the a16 combine)              tf_layer_tail

then tokens = argmax(W_lm . rmsnorm_bf16w(h, final_norm))        tf_lm_head_greedy.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from ._lib import Context, lib, ptr, stream_ptr
from .quant import scale_type_of

EPS = 1e-6


# ------------------------------------------------------------- operators ----
class RMSNorm:
    """RMSNorm.encodeBF16W / encodeNoScale (Metal/Primitives/rmsnorm.metal)."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, x, weight, out, rows: int, d: int, eps: float = EPS, x_stride: int = 0, out_stride: int = 0,
               stream=None):
        st = lib().tf_rmsnorm(self.ctx.handle, ptr(x), x_stride, ptr(weight), ptr(out), out_stride, rows, d, eps,
                              stream_ptr(stream))
        self.ctx.check(st, "RMSNorm.encode")


class FusedQKVEpilogue:
    """fused_qkv_epilogue (Metal/Fusions/fused.metal:84-170)."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, q, k, v, q_weight, k_weight, head_dim, num_q_heads, num_kv_heads, T, position, theta,
               rotated_pairs, eps=EPS, q_stride=0, kv_stride=0, stream=None):
        st = lib().tf_qkv_epilogue(self.ctx.handle, ptr(q), q_stride, ptr(k), ptr(v), kv_stride, ptr(q_weight),
                                   ptr(k_weight), head_dim, num_q_heads, num_kv_heads, T, position, theta,
                                   rotated_pairs, eps, stream_ptr(stream))
        self.ctx.check(st, "FusedQKVEpilogue.encode")


class Attention:
    """Split-KV decode attention (Metal/Attention/attention.metal:135-312)."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def workspace_bytes(self, T, head_dim, num_q_heads, num_kv_heads, seq_len) -> int:
        return int(lib().tf_attention_workspace_bytes(self.ctx.handle, T, head_dim, num_q_heads, num_kv_heads,
                                                      seq_len))

    def encode(self, q, k_cache, v_cache, out, head_dim, num_q_heads, num_kv_heads, T, seq_len, workspace,
               scale=1.0, kv_start=0, seq_stride=0, q_stride=0, out_stride=0, stream=None):
        st = lib().tf_attention_decode(self.ctx.handle, ptr(q), q_stride, ptr(k_cache), ptr(v_cache), seq_stride,
                                       ptr(out), out_stride, head_dim, num_q_heads, num_kv_heads, T, seq_len,
                                       kv_start, scale, ptr(workspace), workspace.numel() * workspace.element_size(),
                                       stream_ptr(stream))
        self.ctx.check(st, "Attention.encode")


class FusedPostAttentionSetup:
    """fused_post_attn_setup (Metal/Fusions/fused.metal:190-269)."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, hidden, attn, dense_x, routed_x, router_x, w_post_attn, w_pre_ffn, w_pre_ffn2, rows, d,
               eps=EPS, stream=None):
        st = lib().tf_post_attn_setup(self.ctx.handle, ptr(hidden), ptr(attn), ptr(dense_x), ptr(routed_x),
                                      ptr(router_x), ptr(w_post_attn), ptr(w_pre_ffn), ptr(w_pre_ffn2), rows, d, eps,
                                      stream_ptr(stream))
        self.ctx.check(st, "FusedPostAttentionSetup.encode")


class FusedLayerTail:
    """fused_layer_tail (Metal/Fusions/fused.metal:271-375), with the shared
    expert's post-FFN-1 norm folded in when w_post_ffn1 is given."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, h2, h1, hidden, w_post_ffn1, w_post_ffn2, w_post_ffn, layer_scalar, rows, d, eps=EPS,
               stream=None):
        st = lib().tf_layer_tail(self.ctx.handle, ptr(h2), ptr(h1), ptr(hidden), ptr(w_post_ffn1), ptr(w_post_ffn2),
                                 ptr(w_post_ffn), float(layer_scalar), rows, d, eps, stream_ptr(stream))
        self.ctx.check(st, "FusedLayerTail.encode")


class EmbedLookupInt4:
    """embed_lookup_int4 (Metal/Quant/dequant_int4.metal:65-84)."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, table, scales, biases, token_ids, out, T, vocab, d, out_scale=1.0, stream=None):
        st = lib().tf_embed_int4(self.ctx.handle, ptr(table), ptr(scales), ptr(biases), ptr(token_ids), T, vocab, d,
                                 float(out_scale), ptr(out), 0, scale_type_of(scales), stream_ptr(stream))
        self.ctx.check(st, "EmbedLookupInt4.encode")


class LMHeadChainInt4:
    """Final norm + int4 LM head + greedy argmax (Kernels/Fusions/LMHeadChainInt4.swift)."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, hidden, norm_weight, W, scales, biases, vocab, d, T, x_normed, logits, out_tokens, eps=EPS,
               hidden_stride=0, stream=None):
        st = lib().tf_lm_head_greedy(self.ctx.handle, ptr(hidden), hidden_stride, ptr(norm_weight), eps, ptr(W),
                                     ptr(scales), ptr(biases), vocab, d, T, ptr(x_normed), ptr(logits),
                                     ptr(out_tokens), scale_type_of(scales), stream_ptr(stream))
        self.ctx.check(st, "LMHeadChainInt4.encode")


# ------------------------------------------------------------ the model -----
@dataclass
class DecoderConfig:
    """Config-4 shape (BASELINE): the config-1 MoE layer, 16 query / 8 KV heads
    of 256, fp16 KV cache, vocab 262144 with an int4 LM head."""

    d: int = 2816
    f: int = 704
    fs: int = 2112
    num_experts: int = 128
    top_k: int = 8
    num_q_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 256
    vocab: int = 262144
    layers: int = 30
    max_context: int = 4096
    rope_theta: float = 10000.0
    eps: float = EPS


@dataclass
class AffineWeight:
    """One int4 affine matrix [rows][cols] (weights, scales, biases)."""

    W: torch.Tensor
    S: torch.Tensor
    B: torch.Tensor
    rows: int
    cols: int

    def nbytes(self) -> int:
        return self.W.numel() + 2 * self.S.numel() * 2


@dataclass
class DecoderLayerWeights:
    input_norm: torch.Tensor
    q: AffineWeight
    k: AffineWeight
    v: AffineWeight
    o: AffineWeight
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    post_attn_norm: torch.Tensor
    pre_ffn: torch.Tensor
    pre_ffn2: torch.Tensor
    post_ffn1: torch.Tensor
    post_ffn2: torch.Tensor
    post_ffn: torch.Tensor
    layer_scalar: float
    moe: object  # MoELayerWeights

    def attn_bytes(self) -> int:
        return sum(w.nbytes() for w in (self.q, self.k, self.v, self.o))


@dataclass
class DecoderWeights:
    cfg: DecoderConfig
    layers: list
    embed: AffineWeight  # [vocab][d], also the LM head (tied)
    final_norm: torch.Tensor


def synthetic_decoder(cfg: DecoderConfig, device, gen: torch.Generator, scale_dtype=torch.bfloat16,
                      moe_layers=None) -> DecoderWeights:
    """Random-initialised weights with the benchmark distributions (int4 codes
    U{0..15}, scale |N(0, 0.02)|, bias -8 scale + N(0, 0.002)); norms near 1.
    `moe_layers` reuses already-built MoE layer weights."""
    from .format import synthetic_affine, synthetic_moe_layer
    d, hd = cfg.d, cfg.head_dim

    def aff(rows, cols):
        W, S, B = synthetic_affine(rows, cols, 4, scale_dtype, device, gen)
        return AffineWeight(W, S, B, rows, cols)

    def norm(n):
        return (1.0 + 0.1 * torch.randn(n, device=device, generator=gen)).to(torch.bfloat16)

    layers = []
    for i in range(cfg.layers):
        moe = moe_layers[i] if moe_layers is not None else synthetic_moe_layer(
            d, cfg.f, cfg.fs, cfg.num_experts, cfg.top_k, 4, scale_dtype, device, gen)
        layers.append(DecoderLayerWeights(
            norm(d), aff(cfg.num_q_heads * hd, d), aff(cfg.num_kv_heads * hd, d), aff(cfg.num_kv_heads * hd, d),
            aff(d, cfg.num_q_heads * hd), norm(hd), norm(hd), norm(d), norm(d), norm(d), norm(d), norm(d), norm(d),
            0.5 + 0.5 * float(torch.rand(1, device=device, generator=gen).item()), moe))
    return DecoderWeights(cfg, layers, aff(cfg.vocab, d), norm(d))


class KVCache:
    """fp16 KV cache: [layer][T][max_context][num_kv_heads][head_dim] for K and V."""

    def __init__(self, cfg: DecoderConfig, T: int, device, context_len: int | None = None):
        n = context_len or cfg.max_context
        self.ctx_len = n
        self.k = torch.zeros(cfg.layers, T, n, cfg.num_kv_heads, cfg.head_dim, dtype=torch.float16, device=device)
        self.v = torch.zeros_like(self.k)

    def fill_random(self, gen: torch.Generator, upto: int):
        """Synthetic history for positions [0, upto): N(0, 1) fp16."""
        self.k[:, :, :upto].normal_(generator=gen)
        self.v[:, :, :upto].normal_(generator=gen)

    def nbytes_per_token(self, seq_len: int) -> int:
        L, _, _, nkv, hd = self.k.shape
        return 2 * L * seq_len * nkv * hd * 2


class Decoder:
    """T-token decode step through every layer and the LM head.  All scratch
    is allocated here once; `step` only enqueues work."""

    def __init__(self, weights: DecoderWeights, T: int, cache: KVCache, context: Context | None = None,
                 device=None, ep_layers: list | None = None, overlap_shared: bool = True):
        """`ep_layers` (one ExpertParallelMoE per layer) routes the experts over
        the process group; the router, shared expert and attention stay local.
        T may be 0 on a rank that only serves experts."""
        cfg = weights.cfg
        self.w, self.cfg, self.T, self.cache = weights, cfg, T, cache
        self.ep = ep_layers
        Ta = max(T, 1)  # buffers of a rank without tokens (it still serves experts)
        self.ctx = context or Context.get(torch.cuda.current_device())
        dev = device or torch.device("cuda", torch.cuda.current_device())
        d, hd, nq, nkv = cfg.d, cfg.head_dim, cfg.num_q_heads, cfg.num_kv_heads
        f16 = dict(dtype=torch.float16, device=dev)
        self.h = torch.zeros(Ta, d, **f16)
        self.normed = torch.empty(Ta, d, **f16)
        self.q = torch.empty(Ta, nq * hd, **f16)
        self.attn = torch.empty(Ta, nq * hd, **f16)
        self.o = torch.empty(Ta, d, **f16)
        self.dense_x = torch.empty(Ta, d, **f16)
        self.routed_x = torch.empty(Ta, d, **f16)
        self.router_x = torch.empty(Ta, d, **f16)
        self.h1 = torch.empty(Ta, d, **f16)
        self.h2 = torch.empty(Ta, d, **f16)
        self.idx = torch.empty(Ta, cfg.top_k, dtype=torch.int32, device=dev)
        self.wts = torch.empty(Ta, cfg.top_k, dtype=torch.float16, device=dev)
        self.sact = torch.empty(Ta, cfg.fs, **f16)
        self.x_normed = torch.empty(Ta, d, **f16)
        self.logits = torch.empty(Ta, cfg.vocab, dtype=torch.float32, device=dev)
        self.tokens = torch.zeros(Ta, dtype=torch.int32, device=dev)
        self.ws_bytes = int(lib().tf_attention_workspace_bytes(self.ctx.handle, Ta, hd, nq, nkv, cache.ctx_len))
        self.attn_ws = torch.empty(max(self.ws_bytes, 16) // 4 + 4, dtype=torch.float32, device=dev)
        if T > 1 and ep_layers is None:
            from .prefill import DeviceRoutes
            E = cfg.num_experts
            i32 = dict(dtype=torch.int32, device=dev)
            self.routes = DeviceRoutes(torch.empty(Ta * cfg.top_k, 4, **i32), torch.empty(E, **i32),
                                       torch.empty(E, **i32), torch.empty(E, 3, **i32), torch.empty(1, **i32),
                                       torch.empty(E, 4, **i32), torch.empty(1, **i32))
            self.ract = torch.empty(Ta * cfg.top_k, cfg.f, **f16)
            self.rpart = torch.empty(Ta * cfg.top_k, d, **f16)
        self.c_moe = [L.moe.as_c() for L in weights.layers]
        self.launches = 0
        # the shared expert's stream (None: run it after the routed path)
        self.side = torch.cuda.Stream(device=dev) if overlap_shared else None

    # int4 projection of T rows (row t of y at y + t*y_stride): the GEMV
    # engines for up to 8 tokens, the tcgen05 GEMM beyond
    def _proj(self, w: AffineWeight, x, y, stream, y_stride: int = 0):
        y_stride = y_stride or w.rows
        if self.T <= 8:
            from .quant import affine_gemv_batched
            affine_gemv_batched(w.W, w.S, w.B, x, y, bits=4, m=w.rows, n=w.cols, ntok=self.T, x_row_stride=w.cols,
                                y_row_stride=y_stride, stream=stream, context=self.ctx)
        else:
            from .prefill import PrefillInt4QMM
            PrefillInt4QMM(self.ctx).encode(w.W, w.S, w.B, x, y, self.T, w.rows, w.cols, y_stride=y_stride,
                                            stream=stream)
        self.launches += 1

    def layer(self, i: int, position: int, stream=None):
        """One decoder layer for the T tokens at `position` (cache slot)."""
        cfg, L, T = self.cfg, self.w.layers[i], self.T
        if T == 0:  # no tokens here: only serve this rank's experts
            self._moe(i, stream)
            return
        d, hd, nq, nkv = cfg.d, cfg.head_dim, cfg.num_q_heads, cfg.num_kv_heads
        ctx = self.ctx
        seq_stride = self.cache.ctx_len * nkv * hd
        kslot = self.cache.k[i, :, position]  # [T][nkv][hd], token stride seq_stride
        vslot = self.cache.v[i, :, position]
        RMSNorm(ctx).encode(self.h, L.input_norm, self.normed, T, d, cfg.eps, stream=stream)
        self._proj(L.q, self.normed, self.q, stream)
        # K and V land straight in this position's cache slots (token stride = one sequence)
        self._proj(L.k, self.normed, kslot, stream, y_stride=seq_stride)
        self._proj(L.v, self.normed, vslot, stream, y_stride=seq_stride)
        FusedQKVEpilogue(ctx).encode(self.q, kslot, vslot, L.q_norm, L.k_norm, hd, nq, nkv, T, position,
                                     cfg.rope_theta, hd // 2, cfg.eps, kv_stride=seq_stride, stream=stream)
        Attention(ctx).encode(self.q, self.cache.k[i], self.cache.v[i], self.attn, hd, nq, nkv, T, position + 1,
                              self.attn_ws, seq_stride=seq_stride, stream=stream)
        self._proj(L.o, self.attn, self.o, stream)
        FusedPostAttentionSetup(ctx).encode(self.h, self.o, self.dense_x, self.routed_x, self.router_x,
                                            L.post_attn_norm, L.pre_ffn, L.pre_ffn2, T, d, cfg.eps, stream=stream)
        self.launches += 8
        self._moe(i, stream)
        FusedLayerTail(ctx).encode(self.h2, self.h1, self.h, L.post_ffn1, L.post_ffn2, L.post_ffn, L.layer_scalar, T,
                                   d, cfg.eps, stream=stream)
        self.launches += 1

    def _shared(self, M, T, stream):
        from .moe import SharedExpertRuntime
        from .prefill import PrefillSharedExpert
        if T == 1:
            SharedExpertRuntime(4, self.ctx).encode(self.dense_x[0], M.shared_gate, M.shared_up, M.shared_down,
                                                    self.h1[0], self.sact[0], stream=stream)
            self.launches += 2
        elif T:
            PrefillSharedExpert(self.ctx).encode(self.dense_x, M.shared_gate, M.shared_up, M.shared_down, self.sact,
                                                 self.h1, T, stream=stream)
            self.launches += 2

    def _moe(self, i: int, stream):
        """h1 = shared(dense_x), h2 = routed(routed_x) with the router on router_x.
        The shared expert reads only dense_x, so it runs on a stream forked from
        `stream` beside the routed path (which is latency-bound for most of its
        length) and the two join before the layer tail."""
        from .moe import moe_decode_layer
        from .prefill import PrefillGroupedRoutedMoE, PrefillMoE, PrefillRouter, route_sort
        cfg, M, T, ctx = self.cfg, self.w.layers[i].moe, self.T, self.ctx
        main = stream if stream is not None else torch.cuda.current_stream()
        fork = T > 0 and self.side is not None
        if fork:
            self.side.wait_stream(main)
            self._shared(M, T, self.side)
        if self.ep is not None:
            if T:
                PrefillRouter(ctx).encode_gemma4_block(M.router_w, M.router_s, M.router_b, self.router_x, M.eff_scale,
                                                       M.per_expert_scale, self.idx, self.wts, T, cfg.num_experts,
                                                       cfg.d, cfg.top_k, stream=main)
            self.ep[i].forward(self.routed_x[:T], self.idx[:T], self.wts[:T], self.h2[:T], stream=main)
            self.launches += 11
        elif T == 1:
            moe_decode_layer(M, self.router_x[0], self.routed_x[0], self.h2[0], out_indices=self.idx[0],
                             out_weights=self.wts[0], stream=main, context=ctx, c_layer=self._routed_only(i))
            self.launches += 3
        else:
            PrefillRouter(ctx).encode_gemma4_block(M.router_w, M.router_s, M.router_b, self.router_x, M.eff_scale,
                                                   M.per_expert_scale, self.idx, self.wts, T, cfg.num_experts, cfg.d,
                                                   cfg.top_k, stream=main)
            route_sort(self.idx, self.wts, T, cfg.top_k, cfg.num_experts, 16, stream=main, context=ctx,
                       out=self.routes)
            PrefillGroupedRoutedMoE(ctx).encode(M.experts, self.routes, self.routed_x, self.ract, self.rpart, T,
                                                cfg.top_k, stream=main)
            PrefillMoE.encode_reduce_token_major(self.rpart, self.wts, self.h2, T, cfg.top_k, cfg.d, stream=main,
                                                 context=ctx)
            self.launches += 8
        if fork:
            main.wait_stream(self.side)
        else:
            self._shared(M, T, main)

    def _routed_only(self, i: int):
        """The C layer struct with the shared expert switched off (rows = 0)."""
        from ._lib import AffineMatrix
        if not hasattr(self, "_c_routed"):
            self._c_routed = {}
        if i not in self._c_routed:
            c = self.w.layers[i].moe.as_c()
            c.shared_gate = AffineMatrix()
            c.shared_up = AffineMatrix()
            c.shared_down = AffineMatrix()
            self._c_routed[i] = c
        return self._c_routed[i]

    def embed(self, token_ids, stream=None):
        if self.T == 0:
            return
        cfg = self.cfg
        e = self.w.embed
        EmbedLookupInt4(self.ctx).encode(e.W, e.S, e.B, token_ids, self.h, self.T, cfg.vocab, cfg.d,
                                         float(cfg.d) ** 0.5, stream=stream)
        self.launches += 1

    def lm_head(self, stream=None):
        if self.T == 0:
            return
        cfg, e = self.cfg, self.w.embed
        LMHeadChainInt4(self.ctx).encode(self.h, self.w.final_norm, e.W, e.S, e.B, cfg.vocab, cfg.d, self.T,
                                         self.x_normed, self.logits, self.tokens, cfg.eps, stream=stream)
        self.launches += 3

    def step(self, token_ids, position: int, stream=None):
        """Embed -> every layer at `position` -> LM head; next tokens in self.tokens."""
        self.launches = 0
        self.embed(token_ids, stream)
        for i in range(self.cfg.layers):
            self.layer(i, position, stream)
        self.lm_head(stream)
        return self.tokens

    def weight_bytes_per_step(self, distinct_experts_per_layer: float) -> float:
        """Algorithmic HBM bytes of one step's weights: attention + router +
        shared expert + the distinct routed experts hit, per layer, plus the LM head."""
        from .format import affine_bytes
        cfg = self.cfg
        expert = 2 * affine_bytes(cfg.f, cfg.d) + affine_bytes(cfg.d, cfg.f)
        shared = 2 * affine_bytes(cfg.fs, cfg.d) + affine_bytes(cfg.d, cfg.fs)
        router = affine_bytes(cfg.num_experts, cfg.d, 8)
        per_layer = self.w.layers[0].attn_bytes() + router + shared + distinct_experts_per_layer * expert
        return cfg.layers * per_layer + self.w.embed.nbytes()
