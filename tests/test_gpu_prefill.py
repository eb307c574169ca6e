"""GPU parity of the batched/prefill path: device grouping and batched router."""
import numpy as np
import pytest
import torch

import oracle as O
from edgeexpert_b200.prefill import PAIR_DTYPE, PrefillMoEGrouping, PrefillRouter, route_sort

pytestmark = pytest.mark.gpu


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.view(dtype) if dtype is not None else t


@pytest.mark.parametrize("T,K,E,tile,keys", [(64, 8, 128, 16, False), (3, 2, 16, 2, False), (4096, 8, 128, 16, False),
                                             (37, 8, 128, 4, True), (1, 8, 128, 16, False)])
def test_device_route_sort_matches_reference_grouping(cuda, T, K, E, tile, keys):
    rng = np.random.default_rng(T * 7 + K)
    # skewed histogram: popular experts more likely
    p = rng.random(E) ** 4
    p /= p.sum()
    idx = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T)]).astype(np.uint32)
    w = rng.random((T, K)).astype(np.float16)
    sk = rng.integers(0, 7, E).astype(np.uint64) if keys else None
    pairs = PrefillRouter.make_token_expert_pairs(idx, w, T, K)
    ref = PrefillMoEGrouping.group_token_expert_pairs(pairs, T, K, E, tile, sk)
    out = route_sort(dev(idx.view(np.int32)), dev(w), T, K, E, tile, None if sk is None else dev(sk.view(np.int64)))
    torch.cuda.synchronize()
    assert np.array_equal(out.sorted_pairs.cpu().numpy().view(np.uint32).reshape(-1),
                          ref.sorted_pairs.view(np.uint32).reshape(-1))
    assert np.array_equal(out.offsets.cpu().numpy().view(np.uint32), ref.per_expert_offsets)
    assert np.array_equal(out.counts.cpu().numpy().view(np.uint32), ref.per_expert_counts)
    ng, nt = int(out.n_groups.item()), int(out.n_tiles.item())
    assert ng == len(ref.groups) and nt == len(ref.tiles)
    assert np.array_equal(out.groups.cpu().numpy()[:ng].view(np.uint32).reshape(-1), ref.groups.view(np.uint32).reshape(-1))
    assert np.array_equal(out.tiles.cpu().numpy()[:nt].view(np.uint32).reshape(-1), ref.tiles.view(np.uint32).reshape(-1))


@pytest.mark.parametrize("T,E,D,K", [(3, 16, 128, 2), (64, 128, 2816, 8), (257, 128, 2816, 8), (5, 64, 256, 64)])
def test_batched_router(cuda, T, E, D, K):
    rng = O.seed_tree(T, f"prefill-router-{E}-{D}")
    W8, S8, B8 = rng.synthetic_affine(E, D, 8, 0)
    H = rng.normal_f16(T * D).reshape(T, D)
    es = O.bf16_bits(np.full(D, D ** -0.5, np.float32))
    pes = O.bf16_bits(rng.uniform(0.8, 1.2, E))
    idx = torch.empty(T, K, dtype=torch.int32, device="cuda")
    w = torch.empty(T, K, dtype=torch.float16, device="cuda")
    PrefillRouter().encode_gemma4_block(dev(W8), dev(S8, torch.bfloat16), dev(B8, torch.bfloat16),
                                        dev(H, torch.float16), dev(es, torch.bfloat16), dev(pes, torch.bfloat16),
                                        idx, w, T, E, D, K)
    torch.cuda.synchronize()
    gi = idx.cpu().numpy().astype(np.uint32)
    gw = w.float().cpu().numpy()
    near = 0
    for t in range(T):
        _, l64 = O.router_logits(W8, S8, B8, H[t], es)
        ri, rw16, _ = O.router_topk(l64.astype(np.float32), pes, K)
        srt = np.sort(l64)[::-1]
        if K < E and srt[K - 1] - srt[K] <= 1e-5 * np.max(np.abs(l64)):
            near += 1
            continue
        assert gi[t].tolist() == ri.tolist(), t
        assert np.max(np.abs(gw[t] - O.f16_to_f32(rw16))) < 2e-3
    assert near <= max(1, T // 20)
