"""GPU test of tf_router_topk_noalloc, the router entry point for callers that
cannot allocate device memory (for example a host whose allocator owns every
device byte).  It must select the same experts, with the same weights, as
tf_router_topk on identical inputs, on two calls in a row (the second call
reuses the library's fixed scratch array left by the first).

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def _dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.view(dtype) if dtype is not None else t


def test_router_noalloc_matches_router_twice(cuda):
    from edgeexpert_b200._lib import TF_OK, lib, ptr, stream_ptr
    from edgeexpert_b200.moe import MoE

    E, D, K = 128, 2816, 8
    moe = MoE()
    for call in range(2):
        rng = O.seed_tree(call, "noalloc-router")
        W8, S8, B8 = rng.synthetic_affine(E, D, 8, 0)
        h = _dev(rng.normal_f16(D), torch.float16)
        es = _dev(O.bf16_bits(np.full(D, D ** -0.5, np.float32)), torch.bfloat16)
        pes = _dev(O.bf16_bits(rng.uniform(0.8, 1.2, E)), torch.bfloat16)
        W, S, B = _dev(W8), _dev(S8, torch.bfloat16), _dev(B8, torch.bfloat16)

        idx_ref = torch.empty(K, dtype=torch.int32, device="cuda")
        w_ref = torch.empty(K, dtype=torch.float16, device="cuda")
        moe.encode_router_gemma4(W, S, B, h, es, pes, idx_ref, w_ref, E, D, K)

        idx = torch.full((K,), -1, dtype=torch.int32, device="cuda")
        w = torch.zeros(K, dtype=torch.float16, device="cuda")
        st = lib().tf_router_topk_noalloc(ptr(W), ptr(S), ptr(B), ptr(h), ptr(es), ptr(pes), ptr(idx), ptr(w),
                                          E, D, K, 0, stream_ptr(None))
        assert st == TF_OK
        torch.cuda.synchronize()
        assert idx.tolist() == idx_ref.tolist(), call
        diff = (w.float() - w_ref.float()).abs().max().item()
        assert diff <= 2e-3 * max(1.0, w_ref.float().abs().max().item()), call


def test_router_noalloc_rejects_too_many_experts(cuda):
    from edgeexpert_b200._lib import TF_ERR_UNSUPPORTED_SHAPE, lib
    z = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    p = C.c_void_p(z.data_ptr())
    st = lib().tf_router_topk_noalloc(p, p, p, p, p, p, p, p, 257, 64, 8, 0, C.c_void_p(0))
    assert st == TF_ERR_UNSUPPORTED_SHAPE
