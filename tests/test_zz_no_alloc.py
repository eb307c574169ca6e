"""GPU test of tf_router_topk_noalloc, the router entry point for callers that
cannot allocate device memory (for example a host whose allocator owns every
device byte, or a process that must not allocate after start-up).  On two
calls in a row (the second reuses the library's fixed scratch array left by
the first) it must select the same experts as the oracle's router top-k, bit
for bit, with weights within the fp16 tolerance, and agree with
tf_router_topk.  tf_router_topk_noalloc_check must then report no device
error.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
FP16_TOL = 2e-3


def _dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.view(dtype) if dtype is not None else t


@pytest.mark.parametrize("E,K,st", [(128, 8, 0), (128, 8, 1), (100, 32, 0), (256, 16, 1), (24, 24, 0)])
def test_router_noalloc_matches_oracle_twice(cuda, E, K, st):
    from edgeexpert_b200._lib import TF_OK, lib, ptr, stream_ptr
    from edgeexpert_b200.moe import MoE

    D = 2816 if E <= 128 else 1024
    sdt = torch.float16 if st == 1 else torch.bfloat16
    moe = MoE()
    for call in range(2):
        rng = O.seed_tree(call * 1000 + E, f"noalloc-router-{st}")
        W8, S8, B8 = rng.synthetic_affine(E, D, 8, st)
        h16 = rng.normal_f16(D)
        es_b = O.bf16_bits(np.full(D, D ** -0.5, np.float32))
        pes_b = O.bf16_bits(rng.uniform(0.8, 1.2, E))
        W, S, B = _dev(W8), _dev(S8, sdt), _dev(B8, sdt)
        h, es, pes = _dev(h16, torch.float16), _dev(es_b, torch.bfloat16), _dev(pes_b, torch.bfloat16)

        idx = torch.full((K,), -1, dtype=torch.int32, device="cuda")
        w = torch.zeros(K, dtype=torch.float16, device="cuda")
        rc = lib().tf_router_topk_noalloc(ptr(W), ptr(S), ptr(B), ptr(h), ptr(es), ptr(pes), ptr(idx), ptr(w),
                                          E, D, K, st, stream_ptr(None))
        assert rc == TF_OK
        flags = C.c_uint32(0xFFFF)
        assert lib().tf_router_topk_noalloc_check(stream_ptr(None), C.byref(flags)) == TF_OK
        assert flags.value == 0
        got_idx = idx.cpu().numpy().astype(np.uint32)
        got_w = w.float().cpu().numpy()

        # oracle: fp64 logits, the reference's selection rule (ties to the lower id)
        _, l64 = O.router_logits(W8, S8, B8, h16, es_b, st)
        srt = np.sort(l64)[::-1]
        if K < E and srt[K - 1] - srt[K] <= 1e-5 * np.max(np.abs(l64)):
            pytest.skip("near tie at the k-th logit for this seed")
        exp_idx, exp_w16, _ = O.router_topk(l64.astype(np.float32), pes_b, K)
        assert got_idx.tolist() == exp_idx.tolist(), call
        assert np.max(np.abs(got_w - O.f16_to_f32(exp_w16))) <= FP16_TOL, call

        # and the context entry point on the same inputs
        idx_ref = torch.empty(K, dtype=torch.int32, device="cuda")
        w_ref = torch.empty(K, dtype=torch.float16, device="cuda")
        moe.encode_router_gemma4(W, S, B, h, es, pes, idx_ref, w_ref, E, D, K)
        torch.cuda.synchronize()
        assert idx.tolist() == idx_ref.tolist(), call
        assert (w.float() - w_ref.float()).abs().max().item() <= FP16_TOL, call


def test_router_noalloc_rejects_bad_arguments(cuda):
    from edgeexpert_b200._lib import TF_ERR_INVALID_ARG, TF_ERR_UNSUPPORTED_SHAPE, lib
    z = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    p = C.c_void_p(z.data_ptr())
    assert lib().tf_router_topk_noalloc(p, p, p, p, p, p, p, p, 257, 64, 8, 0, C.c_void_p(0)) == \
        TF_ERR_UNSUPPORTED_SHAPE
    assert lib().tf_router_topk_noalloc(p, p, p, p, p, p, p, p, 16, 64, 8, 7, C.c_void_p(0)) == TF_ERR_INVALID_ARG
