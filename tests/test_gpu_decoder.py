"""GPU parity of the dense decode stack (attention, norms, RoPE, layer tail,
embedding, LM head) against the C oracle, through the C ABI.

Tolerances: RelError (RelError.swift:7-16) <= 2e-3 for fp16 outputs and
<= 1e-4 for the LM head's fp32 logits of one token; the greedy token is
bit-exact unless the top-2 logit gap is a near tie (<= 1e-5 max|logit|).
The embedding lookup is bit-exact (same rounding points).
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
FP16_TOL = 2e-3
FP32_TOL = 1e-4


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.view(dtype) if dtype is not None else t


def f16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def norm_w(rng, n):
    return O.bf16_bits((1.0 + 0.1 * np.asarray(rng.uniform(-1, 1, n))).astype(np.float32))


@pytest.mark.parametrize("rows,d,scaled", [(1, 2816, True), (5, 2816, False), (3, 256, True)])
def test_rmsnorm(cuda, rows, d, scaled):
    from edgeexpert_b200.decoder import RMSNorm
    rng = O.seed_tree(rows * d, "rms")
    x = rng.normal_f16(rows * d, 3.0)
    w = norm_w(rng, d) if scaled else None
    ref = O.rmsnorm(x, w, rows, d)
    out = torch.empty(rows, d, dtype=torch.float16, device="cuda")
    RMSNorm().encode(dev(x, torch.float16), None if w is None else dev(w, torch.bfloat16), out, rows, d)
    torch.cuda.synchronize()
    assert O.rel_error(O.f16_to_f32(f16(out)), O.f16_to_f32(ref)) < FP16_TOL


@pytest.mark.parametrize("T,position", [(1, 0), (1, 4095), (3, 77)])
def test_qkv_epilogue(cuda, T, position):
    from edgeexpert_b200.decoder import FusedQKVEpilogue
    nq, nkv, hd = 16, 8, 256
    rng = O.seed_tree(T * 7 + position, "qkv")
    q = rng.normal_f16(T * nq * hd, 2.0)
    k = rng.normal_f16(T * nkv * hd, 2.0)
    v = rng.normal_f16(T * nkv * hd, 2.0)
    qw, kw = norm_w(rng, hd), norm_w(rng, hd)
    ref_q, ref_k, ref_v = [], [], []
    for t in range(T):
        a, b, c = O.qkv_epilogue(q[t * nq * hd:(t + 1) * nq * hd], k[t * nkv * hd:(t + 1) * nkv * hd],
                                 v[t * nkv * hd:(t + 1) * nkv * hd], qw, kw, hd, nq, nkv, position, 10000.0, hd // 2)
        ref_q.append(a), ref_k.append(b), ref_v.append(c)
    qd, kd, vd = dev(q, torch.float16), dev(k, torch.float16), dev(v, torch.float16)
    FusedQKVEpilogue().encode(qd, kd, vd, dev(qw, torch.bfloat16), dev(kw, torch.bfloat16), hd, nq, nkv, T, position,
                              10000.0, hd // 2)
    torch.cuda.synchronize()
    for got, ref in ((qd, ref_q), (kd, ref_k), (vd, ref_v)):
        assert O.rel_error(O.f16_to_f32(f16(got)), O.f16_to_f32(np.concatenate(ref))) < FP16_TOL


@pytest.mark.parametrize("T,nq,nkv,hd,seq,start", [(1, 16, 8, 256, 4096, 0), (1, 16, 8, 256, 1, 0),
                                                   (2, 16, 8, 256, 300, 0), (3, 8, 1, 128, 77, 5),
                                                   (1, 4, 4, 512, 513, 0), (1, 16, 2, 64, 1000, 0),
                                                   (4, 16, 4, 128, 2000, 7), (2, 8, 8, 64, 333, 0),
                                                   (3, 12, 4, 256, 901, 900), (8, 16, 8, 256, 4096, 0)])
def test_attention_decode(cuda, T, nq, nkv, hd, seq, start):
    """Split-KV attention (config 4: 16 query / 8 KV heads of 256 at 4096
    context) against the oracle's two-pass softmax in double."""
    from edgeexpert_b200.decoder import Attention
    ctx_len = seq + 3
    rng = np.random.default_rng(seq + hd)
    K = rng.standard_normal((T, ctx_len, nkv, hd)).astype(np.float16)
    V = rng.standard_normal((T, ctx_len, nkv, hd)).astype(np.float16)
    q = (rng.standard_normal((T, nq, hd)) * 0.08).astype(np.float16)
    att = Attention()
    ws = torch.empty(att.workspace_bytes(T, hd, nq, nkv, seq) // 4 + 4, dtype=torch.float32, device="cuda")
    out = torch.empty(T, nq * hd, dtype=torch.float16, device="cuda")
    att.encode(dev(q.view(np.uint16), torch.float16), dev(K.view(np.uint16), torch.float16),
               dev(V.view(np.uint16), torch.float16), out, hd, nq, nkv, T, seq, ws, kv_start=start,
               seq_stride=ctx_len * nkv * hd)
    torch.cuda.synchronize()
    got = O.f16_to_f32(f16(out)).reshape(T, nq * hd)
    for t in range(T):
        _, ref32 = O.attention_decode(q[t].view(np.uint16), K[t].view(np.uint16), V[t].view(np.uint16), hd, nq, nkv,
                                      seq, start, 1.0)
        assert O.rel_error(got[t], ref32) < FP16_TOL, t


def test_post_attn_setup_and_layer_tail(cuda):
    from edgeexpert_b200.decoder import FusedLayerTail, FusedPostAttentionSetup
    rows, d = 3, 2816
    rng = O.seed_tree(11, "post")
    hidden = rng.normal_f16(rows * d, 2.0)
    attn = rng.normal_f16(rows * d, 0.5)
    w = [norm_w(rng, d) for _ in range(6)]
    h_ref, dx_ref, rx_ref, rt_ref = O.post_attn_setup(hidden, attn, w[0], w[1], w[2], rows, d)
    h = dev(hidden, torch.float16)
    outs = [torch.empty(rows, d, dtype=torch.float16, device="cuda") for _ in range(3)]
    FusedPostAttentionSetup().encode(h, dev(attn, torch.float16), *outs, *[dev(x, torch.bfloat16) for x in w[:3]],
                                     rows, d)
    torch.cuda.synchronize()
    for got, ref in zip([h] + outs, [h_ref, dx_ref, rx_ref, rt_ref]):
        assert O.rel_error(O.f16_to_f32(f16(got)), O.f16_to_f32(ref)) < FP16_TOL
    # the layer tail on the oracle's hidden (isolates the kernel), with and without post-FFN-1
    h1 = rng.normal_f16(rows * d, 4.0)
    h2 = rng.normal_f16(rows * d, 0.3)
    for w1 in (w[3], None):
        ref = O.layer_tail(h2, h1, h_ref, w1, w[4], w[5], 0.7, rows, d)
        hh = dev(h_ref, torch.float16)
        FusedLayerTail().encode(dev(h2, torch.float16), dev(h1, torch.float16), hh,
                                None if w1 is None else dev(w1, torch.bfloat16), dev(w[4], torch.bfloat16),
                                dev(w[5], torch.bfloat16), 0.7, rows, d)
        torch.cuda.synchronize()
        assert O.rel_error(O.f16_to_f32(f16(hh)), O.f16_to_f32(ref)) < FP16_TOL


def test_embed_lookup_bit_exact(cuda):
    from edgeexpert_b200.decoder import EmbedLookupInt4
    vocab, d = 1000, 2816
    rng = O.seed_tree(3, "embed")
    W, S, B = rng.synthetic_affine(vocab, d, 4, 0)
    toks = np.array([0, 999, 17, 17, 512], np.uint32)
    ref = O.embed_int4(W, S, B, toks, d, d ** 0.5)
    out = torch.empty(len(toks), d, dtype=torch.float16, device="cuda")
    EmbedLookupInt4().encode(dev(W), dev(S, torch.bfloat16), dev(B, torch.bfloat16), dev(toks.view(np.int32)), out,
                             len(toks), vocab, d, d ** 0.5)
    torch.cuda.synchronize()
    assert np.array_equal(f16(out).reshape(-1), ref)


@pytest.mark.parametrize("vocab,T", [(262144, 1), (5000, 1), (20000, 4)])
def test_lm_head_greedy(cuda, vocab, T):
    """Config 4's int4 LM head (262144 x 2816) for one token on the ring GEMV
    (fp32 logits within 1e-4 of the oracle, token bit-exact), and several
    tokens on the tcgen05 GEMM (w rounded to fp16 before the MMA: logits within
    the fp16 bar, token bit-exact when the top-2 gap exceeds that error)."""
    from edgeexpert_b200.decoder import LMHeadChainInt4
    d = 2816
    rng = O.seed_tree(vocab + T, "lmhead")
    W, S, B = rng.synthetic_affine(vocab, d, 4, 0)
    hidden = rng.normal_f16(T * d, 2.0)
    nw = norm_w(rng, d)
    xn = O.rmsnorm(hidden, nw, T, d)
    x_normed = torch.empty(T, d, dtype=torch.float16, device="cuda")
    logits = torch.empty(T, vocab, dtype=torch.float32, device="cuda")
    toks = torch.full((T,), -1, dtype=torch.int32, device="cuda")
    LMHeadChainInt4().encode(dev(hidden, torch.float16), dev(nw, torch.bfloat16), dev(W), dev(S, torch.bfloat16),
                             dev(B, torch.bfloat16), vocab, d, T, x_normed, logits, toks)
    torch.cuda.synchronize()
    assert O.rel_error(O.f16_to_f32(f16(x_normed)), O.f16_to_f32(xn)) < FP16_TOL
    lg = logits.cpu().numpy()
    got = toks.cpu().numpy()
    for t in range(T):
        # the oracle on the kernel's normalised input isolates the head
        ref_tok, ref_lg = O.lm_head_greedy(W, S, B, f16(x_normed)[t], vocab, d, want_logits=True)
        tol = FP32_TOL if T == 1 else FP16_TOL
        assert O.rel_error(lg[t], ref_lg) <= tol, t
        srt = np.sort(ref_lg)[::-1]
        gap_tol = (1e-5 if T == 1 else 4e-3) * np.max(np.abs(ref_lg))
        if srt[0] - srt[1] > gap_tol:
            assert int(got[t]) == ref_tok, t
        # always: the token is the argmax of the kernel's own logits, ties to the lower row
        assert int(got[t]) == int(np.argmax(lg[t])), t


def _host(t):
    """A device tensor's raw bytes/bits as numpy (uint8 / uint16)."""
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return t.contiguous().cpu().numpy()


def _oracle_layer(L, cfg, h, Kc, Vc, position, gpu_idx=None, gpu_w=None):
    """One decoder layer on the oracle (the reference's step order,
    RealForwardRunner.swift:2240-2480), for one token with hidden h (fp16
    bits); Kc/Vc [ctx][nkv][hd] fp16 bits are updated at `position`."""
    d, hd, nq, nkv = cfg.d, cfg.head_dim, cfg.num_q_heads, cfg.num_kv_heads

    def gemv(w, x):
        _, y16 = O.int4_gemv_kernel_order(_host(w.W), _host(w.S), _host(w.B), x, 0)
        return y16

    normed = O.rmsnorm(h, _host(L.input_norm), 1, d, cfg.eps)
    q, k, v = gemv(L.q, normed), gemv(L.k, normed), gemv(L.v, normed)
    q, k, v = O.qkv_epilogue(q, k, v, _host(L.q_norm), _host(L.k_norm), hd, nq, nkv, position, cfg.rope_theta,
                             hd // 2, cfg.eps)
    Kc[position] = k.reshape(nkv, hd)
    Vc[position] = v.reshape(nkv, hd)
    attn, _ = O.attention_decode(q, Kc, Vc, hd, nq, nkv, position + 1, 0, 1.0)
    o = gemv(L.o, attn)
    h, dense_x, routed_x, router_x = O.post_attn_setup(h, o, _host(L.post_attn_norm), _host(L.pre_ffn),
                                                       _host(L.pre_ffn2), 1, d, cfg.eps)
    M = L.moe
    sg, su, sd = ((_host(p.weights), _host(p.scales), _host(p.biases)) for p in (M.shared_gate, M.shared_up,
                                                                                M.shared_down))
    _, h1, _ = O.shared_expert(sg, su, sd, dense_x, d, cfg.fs, 4)
    _, l64 = O.router_logits(_host(M.router_w), _host(M.router_s), _host(M.router_b), router_x, _host(M.eff_scale))
    idx, w16, _ = O.router_topk(l64.astype(np.float32), _host(M.per_expert_scale), cfg.top_k)
    srt = np.sort(l64)[::-1]
    near_tie = srt[cfg.top_k - 1] - srt[cfg.top_k] <= 1e-5 * np.max(np.abs(l64))
    if near_tie and gpu_idx is not None:
        idx, w16 = gpu_idx, gpu_w
    pool = _host(M.experts.blob)
    stride = M.experts.stride
    blobs = [pool[int(e) * stride:(int(e) + 1) * stride] for e in idx]
    off = O.Offsets(*[getattr(M.experts.offsets, n) for n, _ in O.Offsets._fields_])
    acts = O.moe_phase1(blobs, off, routed_x, d, cfg.f)
    h2, _ = O.moe_phase2(blobs, off, acts, w16, None, d, cfg.f)
    h = O.layer_tail(h2, h1, h, _host(L.post_ffn1), _host(L.post_ffn2), _host(L.post_ffn), L.layer_scalar, 1, d,
                     cfg.eps)
    return h, idx, near_tie


def test_decoder_step_matches_oracle_layer_by_layer(cuda):
    """A small decoder (d=256, 16 experts, 4/2 heads of 64, vocab 1000, two
    layers) decoding one token at position 20 over a random 20-token cache:
    every layer's output hidden within 2e-3 of the oracle's layer run on the
    GPU's input (and cache), routing bit-exact (or a near tie), and the greedy
    token equal to the oracle LM head's."""
    from edgeexpert_b200.decoder import Decoder, DecoderConfig, KVCache, synthetic_decoder
    cfg = DecoderConfig(d=256, f=128, fs=128, num_experts=16, top_k=8, num_q_heads=4, num_kv_heads=2, head_dim=64,
                        vocab=1000, layers=2, max_context=32)
    devc = torch.device("cuda", 0)
    gen = torch.Generator(device=devc)
    gen.manual_seed(7)
    w = synthetic_decoder(cfg, devc, gen)
    cache = KVCache(cfg, 1, devc)
    cache.fill_random(gen, 20)
    dec = Decoder(w, 1, cache)
    pos = 20
    tok = torch.tensor([123], dtype=torch.int32, device=devc)
    dec.embed(tok)
    torch.cuda.synchronize()
    h = _host(dec.h)[0].copy()
    ref_h = O.embed_int4(_host(w.embed.W), _host(w.embed.S), _host(w.embed.B), np.array([123], np.uint32), cfg.d,
                         cfg.d ** 0.5)
    assert np.array_equal(h, ref_h)
    for i in range(cfg.layers):
        Kc = _host(cache.k[i, 0]).copy()
        Vc = _host(cache.v[i, 0]).copy()
        dec.layer(i, pos)
        torch.cuda.synchronize()
        got = _host(dec.h)[0]
        ref, idx, tie = _oracle_layer(w.layers[i], cfg, h, Kc, Vc, pos, _host(dec.idx)[0].astype(np.uint32),
                                      _host(dec.wts)[0])
        if not tie:
            assert _host(dec.idx)[0].astype(np.uint32).tolist() == idx.tolist(), i
        # the cache slot written by the layer (normed + RoPE'd K, normed V)
        assert O.rel_error(O.f16_to_f32(_host(cache.k[i, 0, pos])), O.f16_to_f32(Kc[pos])) < FP16_TOL
        assert O.rel_error(O.f16_to_f32(got), O.f16_to_f32(ref)) < FP16_TOL, i
        h = got.copy()
    dec.lm_head()
    torch.cuda.synchronize()
    xn = O.rmsnorm(h, _host(w.final_norm), 1, cfg.d, cfg.eps)
    ref_tok, lg = O.lm_head_greedy(_host(w.embed.W), _host(w.embed.S), _host(w.embed.B), xn, cfg.vocab, cfg.d,
                                   want_logits=True)
    srt = np.sort(lg)[::-1]
    if srt[0] - srt[1] > 1e-3 * np.max(np.abs(lg)):
        assert int(dec.tokens[0].item()) == ref_tok
    assert dec.launches > 0
