"""A repacked layer directory loaded into HBM (edgeexpert_b200.gturbo) runs
through the grouped routed experts and matches the oracle on the file's own
experts (both the aligned layout and the 16-byte realignment)."""
import numpy as np
import pytest
import torch

import oracle as O
from test_gturbo import D, E, F, make_experts, write_packed

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("gap", [0, 2])
def test_loaded_pool_runs_grouped_experts(cuda, tmp_path, gap):
    from edgeexpert_b200.gturbo import OFFSET_FIELDS, load_layer_host, load_layer_pool
    from edgeexpert_b200.prefill import PrefillGroupedRoutedMoE, PrefillRouter, route_sort
    layers = [make_experts(7)]
    write_packed(tmp_path, layers, gap=gap, order=[2, 4, 0, 1, 5, 3])
    pool = load_layer_pool(tmp_path, 0, torch.device("cuda", 0))
    host, stride, offsets, _, _, _ = load_layer_host(tmp_path, 0)
    T, K = 20, 2
    rng = np.random.default_rng(gap)
    idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.uint32)
    w = (rng.random((T, K)) * 0.5 + 0.1).astype(np.float16)
    X = O.seed_tree(gap, "gturbo-x").normal_f16(T * D).reshape(T, D)
    ref = O.group_pairs(PrefillRouter.make_token_expert_pairs(idx, w, T, K), T, K, E, 16)
    off = O.Offsets(*[getattr(offsets, n) for n in OFFSET_FIELDS])
    part_ref = O.grouped_routed(host, stride, off, ref["sorted"], X, D, D, F, K, T, 0)
    routes = route_sort(torch.from_numpy(idx.view(np.int32)).cuda(), torch.from_numpy(w).cuda(), T, K, E, 16)
    act = torch.empty(T * K, F, dtype=torch.float16, device="cuda")
    part = torch.empty(T * K, D, dtype=torch.float16, device="cuda")
    PrefillGroupedRoutedMoE().encode(pool, routes, torch.from_numpy(X.view(np.float16)).cuda(), act, part, T, K)
    torch.cuda.synchronize()
    got = part.view(torch.int16).cpu().numpy().view(np.uint16)
    assert O.rel_error(O.f16_to_f32(got), O.f16_to_f32(part_ref)) < 2e-3
