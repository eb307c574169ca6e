"""Host-side grouping (tf_group_token_expert_pairs, CPU) against the
reference's known answers (PrefillMoEGroupingTests.swift:5-203) and the oracle."""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from edgeexpert_b200.prefill import PAIR_DTYPE, PrefillMoEGrouping, PrefillMoEGroupingError, PrefillRouter

GOLDEN = Path(__file__).resolve().parent / "golden"


def _pairs(lst):
    a = np.zeros(len(lst), PAIR_DTYPE)
    for i, (t, e, r, w) in enumerate(lst):
        a[i] = (t, e, r, w)
    return a


def test_host_grouping_known_answers():
    kat = json.loads((GOLDEN / "grouping_kat.json").read_text())
    c = kat["cases"][0]
    g = PrefillMoEGrouping.group_token_expert_pairs(_pairs(c["pairs"]), c["query_count"], c["top_k"],
                                                    c["num_experts"], c["tile_expert_count"])
    e = c["expect"]
    assert g.sorted_pairs["expert"].tolist() == e["sorted_experts"]
    assert [[int(p["token"]), int(p["rank"])] for p in g.sorted_pairs] == e["sorted_token_rank"]
    assert g.per_expert_offsets.tolist() == e["offsets"]
    assert g.per_expert_counts.tolist() == e["counts"]
    assert [list(map(int, x)) for x in g.groups.tolist()] == e["groups"]
    assert [list(map(int, x)) for x in g.tiles.tolist()] == e["tiles"]
    assert g.max_pairs_per_expert == e["max_pairs_per_expert"]
    assert g.max_pairs_per_tile == e["max_pairs_per_tile"]
    assert g.max_live_experts_per_tile == e["max_live_experts_per_tile"]


def test_host_grouping_order_independent_and_sort_keys():
    kat = json.loads((GOLDEN / "grouping_kat.json").read_text())
    c = kat["cases"][1]
    a = PrefillMoEGrouping.group_token_expert_pairs(_pairs(c["pairs"]), 3, 2, 3, 2)
    b = PrefillMoEGrouping.group_token_expert_pairs(_pairs([c["pairs"][i] for i in c["shuffle"]]), 3, 2, 3, 2)
    assert np.array_equal(a.sorted_pairs, b.sorted_pairs)
    assert a.sorted_pairs["weight_bits"].tolist() == c["expect"]["sorted_weight_bits"]
    c = kat["cases"][2]
    g = PrefillMoEGrouping.group_token_expert_pairs(_pairs(c["pairs"]), 3, 2, 4, 2, c["sort_keys"])
    assert g.groups["expert"].tolist() == c["expect"]["group_experts"]
    assert g.per_expert_offsets.tolist() == c["expect"]["offsets"]
    assert [list(map(int, x)) for x in g.tiles.tolist()] == c["expect"]["tiles"]


def test_host_grouping_rejects_like_reference():
    kat = json.loads((GOLDEN / "grouping_kat.json").read_text())
    for r in kat["rejects"]:
        with pytest.raises(PrefillMoEGroupingError) as ei:
            PrefillMoEGrouping.group_token_expert_pairs(_pairs(r["pairs"]), r["query_count"], r["top_k"],
                                                        r["num_experts"], r["tile_expert_count"], r["sort_keys"])
        assert ei.value.name == r["error"]
        assert ei.value.a == r["a"]
        if "b" in r:
            assert ei.value.b == r["b"]


@pytest.mark.parametrize("seed", range(5))
def test_host_grouping_matches_oracle_random(seed):
    rng = np.random.default_rng(seed)
    T, K, E = 37, 8, 128
    idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.uint32)
    w = rng.random((T, K)).astype(np.float16)
    pairs = PrefillRouter.make_token_expert_pairs(idx, w, T, K)
    rng.shuffle(pairs)
    keys = rng.integers(0, 5, E).astype(np.uint64) if seed % 2 else None
    g = PrefillMoEGrouping.group_token_expert_pairs(pairs, T, K, E, 16, keys)
    o = O.group_pairs(pairs.view(O.PAIR_DTYPE), T, K, E, 16, keys)
    assert np.array_equal(g.sorted_pairs.view(np.uint32), o["sorted"].view(np.uint32))
    assert np.array_equal(g.per_expert_offsets, o["offsets"])
    assert np.array_equal(g.per_expert_counts, o["counts"])
    assert np.array_equal(g.groups.view(np.uint32), o["groups"].view(np.uint32))
    assert np.array_equal(g.tiles.view(np.uint32), o["tiles"].view(np.uint32))


def test_host_grouping_empty_query():
    g = PrefillMoEGrouping.group_token_expert_pairs(np.zeros(0, PAIR_DTYPE), 0, 8, 128)
    assert g.sorted_pairs.size == 0 and len(g.groups) == 0 and len(g.tiles) == 0
    assert (g.per_expert_offsets == 0xFFFFFFFF).all()
