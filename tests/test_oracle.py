"""CPU tests: pin the oracle against the reference's own known answers and
self-tests (no GPU).  Each test names the reference test it restates."""
import json
import math
import struct
from pathlib import Path

import numpy as np
import pytest

import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


# --------------------------------------------------------------- PRNG -------
def _py_splitmix(seed, n):
    out, s = [], seed
    for _ in range(n):
        s = (s + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        z = s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        out.append(z ^ (z >> 31))
    return out


def test_splitmix64_matches_independent_restatement_and_snapshot():
    snap = json.loads((GOLDEN / "oracle_snapshots.json").read_text())
    r = O.Rng(0)
    got = [r.next() for _ in range(4)]
    assert got == _py_splitmix(0, 4) == snap["splitmix64_seed0"]
    assert got[0] == 0xE220A8397B1DCDAF  # the published first SplitMix64 output for seed 0


def test_seedtree_fnv1a():
    h = 0xCBF29CE484222325
    for b in b"abc":
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    assert O.lib().orc_seedtree_seed(0, b"abc") == h
    assert O.lib().orc_seedtree_seed(5, b"abc") == h ^ 5


def test_uniform_is_24_bit_grid():
    r = O.Rng(123)
    ref = _py_splitmix(123, 3)
    for v in ref:
        assert O.Rng(0) is not None
    vals = O.Rng(123).uniform(-1.0, 1.0, 3)
    exp = [np.float32(-1.0) + np.float32(2.0) * np.float32((v >> 40) / (1 << 24)) for v in ref]
    assert np.allclose(vals, exp, rtol=0, atol=1e-7)


# --------------------------------------------------------------- formats ----
def test_bf16_round_half_even_matches_reference_formula():
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(4000).astype(np.float32),
                         np.array([1.0, -2.5, 3.0e-5, 65504.0, 1.00390625, 1.01171875], np.float32)])
    for x in xs:
        bits = struct.unpack("<I", struct.pack("<f", float(x)))[0]
        lsb = (bits >> 16) & 1
        exp = ((bits + 0x7FFF + lsb) & 0xFFFFFFFF) >> 16   # Quantization.swift:17-23
        assert O.lib().orc_bf16_bits(float(x)) == exp


def test_f16_conversion_matches_ieee_numpy():
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10.0,
                         rng.standard_normal(2000).astype(np.float32) * 1e-5,
                         np.array([65504.0, 65520.0, 1e9, -0.0, 6e-8, 2.98e-8], np.float32)])
    got = O.f32_to_f16(xs)
    assert np.array_equal(got, xs.astype(np.float16).view(np.uint16))
    back = O.f16_to_f32(got)
    assert np.array_equal(back, got.view(np.float16).astype(np.float32))


def test_nibble_layout_low_is_even():
    # QuantizationTests.swift:36-50
    row = (np.arange(64, dtype=np.float32) - 31.5).reshape(1, 64)
    W, S, B = O.quantize_affine(row, 4)
    b0 = int(W[0, 0])
    s = float(O.scale_to_f32(S[0, 0], 0))
    b = float(O.scale_to_f32(B[0, 0], 0))
    assert abs((b0 & 0x0F) * s + b - row[0, 0]) <= s + 1e-3
    assert abs((b0 >> 4) * s + b - row[0, 1]) <= s + 1e-3
    assert O.unpack_code(W[0], 0, 4) == (b0 & 0x0F) and O.unpack_code(W[0], 1, 4) == (b0 >> 4)


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_affine_round_trip_bound(bits):
    # DequantInt4GEMVReferenceTests.swift:59-76: |w_hat - w| <= scale + 1e-4
    rng = O.seed_tree(0x55, f"roundtrip-b{bits}")
    w = rng.uniform(-0.5, 0.5, 4 * 256).reshape(4, 256)
    W, S, B = O.quantize_affine(w, bits)
    rec = O.dequantize_affine(W, S, B, 256, bits)
    sc = np.repeat(O.scale_to_f32(S, 0), 64, axis=1)
    assert np.all(np.abs(rec - w) <= sc + 1e-4)


def test_constant_group_is_exact():
    # QuantizationAffineTests.swift:60-88 (constant group -> scale 1, bias = value)
    w = np.full((1, 64), 0.25, np.float32)
    W, S, B = O.quantize_affine(w, 4)
    assert np.all(O.dequantize_affine(W, S, B, 64, 4) == 0.25)


def test_gelu_known_answers():
    kat = json.loads((GOLDEN / "gelu_kat.json").read_text())
    y = [O.gelu(v) for v in kat["x"]]
    assert abs(y[0]) < 1e-7
    assert abs(y[1] - kat["at1"]) < 1e-5
    assert y[1] > 0 and y[2] < 0 and y[3] > y[1]
    assert O.gelu(1e4) == pytest.approx(1e4) and O.gelu(-1e4) == 0.0  # clamp keeps it finite


# --------------------------------------------------------------- GEMV -------
@pytest.mark.parametrize("m,n", [(128, 128), (64, 64), (65, 192), (129, 512), (96, 2816)])
def test_kernel_order_gemv_within_reference_tolerance(m, n):
    # DequantInt4GEMVTests.swift:41-100: kernel vs DequantInt4GemvRef, rel < 5e-3
    rng = O.seed_tree(0xC1, f"int4-gemv-kernel-m{m}-n{n}")
    w = rng.uniform(-0.5, 0.5, m * n).reshape(m, n)
    W, S, B = O.quantize_affine(w, 4)
    x16 = O.f32_to_f16(rng.uniform(-1.0, 1.0, n))
    y32, y16 = O.int4_gemv_kernel_order(W, S, B, x16)
    ref = O.affine_gemv_ref(W, S, B, O.f16_to_f32(x16), 4)
    assert O.rel_error(O.f16_to_f32(y16), ref) < 5e-3
    assert O.rel_error(y32, ref) < 1e-5  # the two fp32 orders agree closely


def test_gemv_snapshot_is_stable():
    snap = json.loads((GOLDEN / "oracle_snapshots.json").read_text())["int4_gemv_m64_n256"]
    rng = O.seed_tree(0, snap["seed_label"])
    W, S, B = rng.synthetic_affine(snap["m"], snap["n"], 4, 0)
    x = rng.normal_f16(snap["n"])
    _, y16 = O.int4_gemv_kernel_order(W, S, B, x, 0, nthreads=1)
    assert y16.tolist() == snap["y_kernel_order_f16"]


def test_int8_kernel_order_vs_ref():
    rng = O.seed_tree(0xD1, "int8")
    W, S, B = rng.synthetic_affine(128, 2816, 8, 0)
    x = rng.normal_f16(2816)
    y32, _ = O.int8_gemv_kernel_order(W, S, B, x)
    ref = O.affine_gemv_ref(W, S, B, O.f16_to_f32(x), 8)
    assert O.rel_error(y32, ref) < 1e-4


# --------------------------------------------------------------- router -----
def _router_reference(weights, hidden, eff, expert_scale, k=8):
    """RouterTopKTests.swift:72-97 restated: quantize int8, DequantInt8GemvRef
    on hidden*effective_scale (fp32), sort desc (ties -> lower id), softmax."""
    scaled = (hidden.astype(np.float32) * eff.astype(np.float32)).astype(np.float32)
    W, S, B = O.quantize_affine(weights, 8)
    logits = O.affine_gemv_ref(W, S, B, scaled, 8)
    order = sorted(range(len(logits)), key=lambda e: (-logits[e], e))[:k]
    mx = logits[order[0]]
    ex = np.array([math.exp(logits[e] - mx) for e in order], np.float32)
    w = ex / ex.sum() * np.array([expert_scale[e] for e in order], np.float32)
    return np.array(order, np.uint32), w, (W, S, B)


def test_router_matches_reference_test_case():
    # RouterTopKTests.productionRouterMatchesReference (:17-44), data from the same SplitMix64 stream
    rng = O.Rng(0xA5B61234)
    E, D = 16, 128
    weights = np.array([[rng.uniform(-0.05, 0.05) + e * 0.01 for _ in range(D)] for e in range(E)], np.float32)
    hidden = np.array([rng.uniform(-1.0, 1.0) for _ in range(D)], np.float32)
    inv = 1.0 / math.sqrt(D)
    eff = np.array([rng.uniform(0.5, 1.5) * inv for _ in range(D)], np.float32)
    es = np.array([rng.uniform(0.6, 1.4) for _ in range(E)], np.float32)
    # kernel inputs: hidden as half, eff/expert scale as bf16 (RouterTopKTests.swift:122-130)
    h16 = O.f32_to_f16(hidden)
    eff_b = O.bf16_bits(eff)
    es_b = O.bf16_bits(es)
    exp_idx, exp_w, (W, S, B) = _router_reference(weights, O.f16_to_f32(h16), O.scale_to_f32(eff_b, 0),
                                                  O.scale_to_f32(es_b, 0))
    l32, l64 = O.router_logits(W, S, B, h16, eff_b)
    idx, w16, _ = O.router_topk(l32, es_b, 8)
    assert idx.tolist() == exp_idx.tolist()
    assert np.max(np.abs(O.f16_to_f32(w16) - exp_w)) < 5e-3


def test_router_near_tie_resolves_like_reference():
    # RouterTopKTests.productionRouterResolvesNearTieLikeReference (:46-70)
    rng = O.Rng(0x71E0F4A)
    E, D = 16, 128
    pattern = np.array([rng.uniform(0.2, 1.0) for _ in range(D)], np.float32)
    hidden = np.array([rng.uniform(0.5, 1.5) for _ in range(D)], np.float32)
    gains = np.zeros(E, np.float32)
    for e in range(7):
        gains[e] = 1.0 - e * 0.05
    gains[7] = 0.5
    gains[8] = np.float32(0.5 * (1.0 + 1e-4))
    for e in range(9, E):
        gains[e] = 0.4 - (e - 9) * 0.02
    weights = np.outer(gains, pattern).astype(np.float32)
    h16 = O.f32_to_f16(hidden)
    ones_b = O.bf16_bits(np.ones(D, np.float32))
    exp_idx, _, (W, S, B) = _router_reference(weights, O.f16_to_f32(h16), np.ones(D, np.float32), np.ones(E))
    l32, _ = O.router_logits(W, S, B, h16, ones_b)
    idx, _, _ = O.router_topk(l32, O.bf16_bits(np.ones(E, np.float32)), 8)
    assert idx.tolist() == exp_idx.tolist()


def test_topk_tie_goes_to_lower_id():
    logits = np.array([1.0, 3.0, 3.0, 2.0, 3.0, 0.5, 0.5, 0.5, 0.5, 0.5], np.float32)
    idx, _, w = O.router_topk(logits, O.bf16_bits(np.ones(10, np.float32)), 8)
    assert idx.tolist() == [1, 2, 4, 3, 0, 5, 6, 7]
    assert abs(float(w.sum()) - 1.0) < 1e-5


# --------------------------------------------------------------- grouping ---
def _pairs(lst):
    a = np.zeros(len(lst), O.PAIR_DTYPE)
    for i, (t, e, r, w) in enumerate(lst):
        a[i] = (t, e, r, w)
    return a


def test_grouping_known_answers():
    kat = json.loads((GOLDEN / "grouping_kat.json").read_text())
    c = kat["cases"][0]
    g = O.group_pairs(_pairs(c["pairs"]), c["query_count"], c["top_k"], c["num_experts"], c["tile_expert_count"])
    e = c["expect"]
    assert g["sorted"]["expert"].tolist() == e["sorted_experts"]
    assert [[int(p["token"]), int(p["rank"])] for p in g["sorted"]] == e["sorted_token_rank"]
    assert g["offsets"].tolist() == e["offsets"]
    assert g["counts"].tolist() == e["counts"]
    assert [list(map(int, x)) for x in g["groups"].tolist()] == e["groups"]
    assert [list(map(int, x)) for x in g["tiles"].tolist()] == e["tiles"]
    assert max(g["groups"]["pair_count"]) == e["max_pairs_per_expert"]
    assert max(g["tiles"]["pair_count"]) == e["max_pairs_per_tile"]
    assert max(g["tiles"]["group_count"]) == e["max_live_experts_per_tile"]


def test_grouping_order_independent_and_keeps_weight_bits():
    kat = json.loads((GOLDEN / "grouping_kat.json").read_text())
    c = kat["cases"][1]
    a = O.group_pairs(_pairs(c["pairs"]), c["query_count"], c["top_k"], c["num_experts"], c["tile_expert_count"])
    sh = [c["pairs"][i] for i in c["shuffle"]]
    b = O.group_pairs(_pairs(sh), c["query_count"], c["top_k"], c["num_experts"], c["tile_expert_count"])
    for k in a:
        assert np.array_equal(a[k], b[k])
    assert a["sorted"]["weight_bits"].tolist() == c["expect"]["sorted_weight_bits"]


def test_grouping_sort_keys():
    kat = json.loads((GOLDEN / "grouping_kat.json").read_text())
    c = kat["cases"][2]
    g = O.group_pairs(_pairs(c["pairs"]), c["query_count"], c["top_k"], c["num_experts"], c["tile_expert_count"],
                      c["sort_keys"])
    e = c["expect"]
    assert g["groups"]["expert"].tolist() == e["group_experts"]
    assert g["sorted"]["expert"].tolist() == e["sorted_experts"]
    assert g["offsets"].tolist() == e["offsets"]
    assert [list(map(int, x)) for x in g["tiles"].tolist()] == e["tiles"]


def test_grouping_rejects_invalid_metadata():
    kat = json.loads((GOLDEN / "grouping_kat.json").read_text())
    for r in kat["rejects"]:
        with pytest.raises(O.GroupingError) as ei:
            O.group_pairs(_pairs(r["pairs"]), r["query_count"], r["top_k"], r["num_experts"],
                          r["tile_expert_count"], r["sort_keys"])
        assert O.GROUP_ERRORS[ei.value.code] == r["error"]
        assert ei.value.a == r["a"]
        if "b" in r:
            assert ei.value.b == r["b"]


def test_grouping_real_trace_pressure_t32():
    # PrefillMoEGroupingTests.swift:175-203
    lst = [(t, (t + r * 7) % 74, r, t * 8 + r) for t in range(32) for r in range(8)]
    g = O.group_pairs(_pairs(lst), 32, 8, 128, 16)
    assert g["sorted"].size == 256
    assert len(g["groups"]) <= 74
    assert all(t["group_count"] <= 16 and t["pair_count"] > 0 for t in g["tiles"])


# --------------------------------------------------------------- MoE --------
def test_moe_oracle_matches_reference_composition():
    # MoEFusedFFNTests vs MoeRef.applyStreamedRouted (rel < 1e-2), D=128 F=64 top-8
    D, F, K = 128, 64, 8
    rng = O.seed_tree(0x181, "moe-ffn")
    blobs, mats = [], []
    for _ in range(K):
        g = O.quantize_affine(rng.uniform(-0.3, 0.3, F * D).reshape(F, D), 4)
        u = O.quantize_affine(rng.uniform(-0.3, 0.3, F * D).reshape(F, D), 4)
        d = O.quantize_affine(rng.uniform(-0.3, 0.3, D * F).reshape(D, F), 4)
        parts = [g[0], g[1], g[2], u[0], u[1], u[2], d[0], d[1], d[2]]
        offs, cur, chunks = [], 0, []
        for p in parts:
            b = np.ascontiguousarray(p).view(np.uint8).reshape(-1)
            offs.append(cur)
            chunks.append(b)
            cur += b.size
        blobs.append(np.concatenate(chunks))
        mats.append((g, u, d))
    off = O.Offsets(*offs)
    x16 = O.f32_to_f16(rng.uniform(-1, 1, D))
    w = rng.uniform(0.05, 0.3, K)
    w16 = O.f32_to_f16(w)
    acts = O.moe_phase1(blobs, off, x16, D, F)
    y16, y32 = O.moe_phase2(blobs, off, acts, w16, None, D, F)
    # MoeRef: fp32 FFN per expert, no intermediate rounding, weighted sum
    x = O.f16_to_f32(x16)
    ref = np.zeros(D, np.float32)
    for s, (g, u, d) in enumerate(mats):
        gv = O.affine_gemv_ref(*g, x, 4)
        uv = O.affine_gemv_ref(*u, x, 4)
        act = np.array([O.gelu(float(a)) for a in gv], np.float32) * uv
        ref += O.f16_to_f32(w16)[s] * O.affine_gemv_ref(*d, act, 4)
    assert O.rel_error(O.f16_to_f32(y16), ref) < 1e-2
