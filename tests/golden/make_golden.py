"""Generate tests/golden/*.json.

Two kinds of fixtures:

1. Known-answer cases transcribed, as data, from the reference's own test
   suite (read as text; the Swift code cannot run here):
   - PrefillMoEGroupingTests.swift:5-53   (sorted pairs, offsets, counts, groups, tiles)
   - PrefillMoEGroupingTests.swift:55-82  (order independence, preserved weight bits)
   - PrefillMoEGroupingTests.swift:84-115 (expert sort keys)
   - PrefillMoEGroupingTests.swift:117-173 (rejected metadata)
   - QuantizationTests.swift:36-50        (nibble layout: low nibble = even index)
   - MoEReferenceTests.swift:7-17         (gelu_pytorch_tanh at 0, 1, -1, 2)
2. Oracle snapshots (seeded, small) used to detect drift of the oracle
   itself and as fixed vectors for the GPU parity tests.

Run: python tests/golden/make_golden.py
"""
import json
import math
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "oracle"))

import numpy as np  # noqa: E402

import oracle as O  # noqa: E402


def grouping_kats():
    main_pairs = [  # (token, expert, rank, weightBits), then reversed as in the test
        (0, 3, 0, 10), (0, 1, 1, 11), (0, 4, 2, 12), (1, 1, 0, 13), (1, 3, 1, 14), (1, 2, 2, 15),
        (2, 4, 0, 16), (2, 3, 1, 17), (2, 1, 2, 18), (3, 5, 0, 19), (3, 1, 1, 20), (3, 4, 2, 21)]
    cases = [
        {
            "name": "groupingSortsPairsAndBuildsOffsetsCountsAndTiles",
            "pairs": list(reversed(main_pairs)), "query_count": 4, "top_k": 3, "num_experts": 6,
            "tile_expert_count": 2, "sort_keys": None,
            "expect": {
                "sorted_experts": [1, 1, 1, 1, 2, 3, 3, 3, 4, 4, 4, 5],
                "sorted_token_rank": [[0, 1], [1, 0], [2, 2], [3, 1], [1, 2], [0, 0], [1, 1], [2, 1], [0, 2],
                                      [2, 0], [3, 2], [3, 0]],
                "offsets": [4294967295, 0, 4, 5, 8, 11],
                "counts": [0, 4, 1, 3, 3, 1],
                "groups": [[1, 0, 4], [2, 4, 1], [3, 5, 3], [4, 8, 3], [5, 11, 1]],
                "tiles": [[0, 2, 0, 5], [2, 2, 5, 6], [4, 1, 11, 1]],
                "max_pairs_per_expert": 4, "max_pairs_per_tile": 6, "max_live_experts_per_tile": 2,
            },
        },
        {
            "name": "groupingIsDeterministicAcrossInputOrderAndPreservesWeightBits",
            "pairs": [(0, 2, 0, 101), (0, 1, 1, 102), (1, 2, 0, 103), (1, 0, 1, 104), (2, 1, 0, 105),
                      (2, 2, 1, 106)],
            "shuffle": [5, 1, 3, 0, 4, 2],
            "query_count": 3, "top_k": 2, "num_experts": 3, "tile_expert_count": 2, "sort_keys": None,
            "expect": {"sorted_weight_bits": [104, 102, 105, 101, 103, 106]},
        },
        {
            "name": "groupingCanOrderTilesByExpertSortKeysWhileKeepingPairRangesContiguous",
            "pairs": [(0, 1, 0, 10), (0, 2, 1, 20), (1, 3, 0, 30), (1, 1, 1, 11), (2, 2, 0, 21), (2, 3, 1, 31)],
            "query_count": 3, "top_k": 2, "num_experts": 4, "tile_expert_count": 2, "sort_keys": [0, 30, 10, 20],
            "expect": {
                "group_experts": [2, 3, 1],
                "sorted_experts": [2, 2, 3, 3, 1, 1],
                "offsets": [4294967295, 4, 0, 2],
                "tiles": [[0, 2, 0, 4], [2, 1, 4, 2]],
            },
        },
    ]
    rejects = [
        {"pairs": [(0, 0, 0, 1)], "query_count": 1, "top_k": 1, "num_experts": 1, "tile_expert_count": 17,
         "sort_keys": None, "error": "invalidTileExpertCount", "a": 17},
        {"pairs": [(0, 2, 0, 1)], "query_count": 1, "top_k": 1, "num_experts": 2, "tile_expert_count": 1,
         "sort_keys": None, "error": "expertOutOfRange", "a": 2},
        {"pairs": [(0, 0, 0, 1), (0, 1, 0, 2)], "query_count": 1, "top_k": 2, "num_experts": 2,
         "tile_expert_count": 1, "sort_keys": None, "error": "duplicateTokenRank", "a": 0, "b": 0},
        {"pairs": [(0, 0, 0, 1)], "query_count": 1, "top_k": 1, "num_experts": 2, "tile_expert_count": 1,
         "sort_keys": [0], "error": "expertSortKeyCountMismatch", "a": 2, "b": 1},
    ]
    return {"cases": cases, "rejects": rejects,
            "source": "Tests/TurboFieldfare/Core/Kernels/Prefill/PrefillMoEGroupingTests.swift:5-173"}


def gelu_kat():
    # gelu_pytorch_tanh(1) as the reference test computes it (MoEReferenceTests.swift:12)
    return {"x": [0.0, 1.0, -1.0, 2.0],
            "at1": 0.5 * (1 + math.tanh(0.7978845608028654 * (1 + 0.044715))),
            "source": "Tests/TurboFieldfare/Core/Validation/Reference/MoEReferenceTests.swift:7-17"}


def oracle_snapshots():
    out = {}
    # int4 GEMV, config-0 distributions at a small size
    rng = O.seed_tree(0, "golden.int4.gemv.m64.n256")
    W, S, B = rng.synthetic_affine(64, 256, 4, 0)
    x = rng.normal_f16(256)
    y32, y16 = O.int4_gemv_kernel_order(W, S, B, x, 0, nthreads=1)
    yref = O.affine_gemv_ref(W, S, B, O.f16_to_f32(x), 4, 0, nthreads=1)
    out["int4_gemv_m64_n256"] = {"seed_label": "golden.int4.gemv.m64.n256", "m": 64, "n": 256,
                                 "y_kernel_order_f16": y16.tolist(), "y_ref_f32": yref.tolist()}
    # router: 16 experts, D=128
    rng = O.seed_tree(0, "golden.router.e16.d128")
    W8, S8, B8 = rng.synthetic_affine(16, 128, 8, 0)
    h = rng.normal_f16(128)
    es = O.bf16_bits(np.full(128, 128 ** -0.5, np.float32))
    pes = O.bf16_bits(rng.uniform(0.6, 1.4, 16))
    l32, l64 = O.router_logits(W8, S8, B8, h, es)
    idx, w16, _ = O.router_topk(l64.astype(np.float32), pes, 8)
    out["router_e16_d128"] = {"seed_label": "golden.router.e16.d128", "indices": idx.tolist(),
                              "weights_f16": w16.tolist(), "logits_f64": l64.tolist()}
    # SplitMix64 stream of seed 0 and SeedTree(0).key("abc")
    r = O.Rng(0)
    out["splitmix64_seed0"] = [r.next() for _ in range(4)]
    out["seedtree_0_abc"] = O.lib().orc_seedtree_seed(0, b"abc")
    return out


def main():
    HERE.mkdir(exist_ok=True)
    (HERE / "grouping_kat.json").write_text(json.dumps(grouping_kats(), indent=1))
    (HERE / "gelu_kat.json").write_text(json.dumps(gelu_kat(), indent=1))
    (HERE / "oracle_snapshots.json").write_text(json.dumps(oracle_snapshots()))
    print("wrote", sorted(p.name for p in HERE.glob("*.json")))


if __name__ == "__main__":
    main()
