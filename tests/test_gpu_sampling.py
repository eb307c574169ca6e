"""GPU parity of the output-head sampling kernels against the oracle
(logit.metal:42-617): the softcap softmax within RelError 2e-3 (fp16 out),
and the sampled token bit-exact for greedy, Gumbel-max, top-k / top-p and
top-64 draws on the same probabilities and seeds (the draws depend only on
the probabilities, the candidate order and the seeded generators)."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
FP16_TOL = 2e-3


def f16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("V,rows,fp32", [(262144, 1, True), (1000, 3, False), (70000, 2, True)])
def test_softcap_softmax(cuda, V, rows, fp32):
    from edgeexpert_b200.sampling import LogitSoftcapSoftmax
    lg = (np.random.default_rng(V).standard_normal((rows, V)) * 8).astype(np.float32)
    if not fp32:
        lg = lg.astype(np.float16).astype(np.float32)
    t = torch.from_numpy(lg).cuda() if fp32 else torch.from_numpy(lg.astype(np.float16)).cuda()
    probs = torch.empty(rows, V, dtype=torch.float16, device="cuda")
    LogitSoftcapSoftmax().encode(t, probs, V, 30.0, rows)
    torch.cuda.synchronize()
    got = O.f16_to_f32(f16(probs)).reshape(rows, V)
    for r in range(rows):
        ref = O.f16_to_f32(O.softcap_softmax(lg[r], 30.0))
        assert O.rel_error(got[r], ref) < FP16_TOL


def _probs(V, seed, sharp=4.0):
    lg = (np.random.default_rng(seed).standard_normal(V) * sharp).astype(np.float32)
    return O.softcap_softmax(lg, 30.0)


@pytest.mark.parametrize("V", [262144, 777])
@pytest.mark.parametrize("temperature,top_k,top_p,seed", [(0.0, 0, 1.0, 0), (1.0, 0, 1.0, 11), (0.7, 0, 1.0, 12),
                                                         (0.8, 40, 1.0, 13), (1.0, 0, 0.9, 14), (1.3, 64, 0.95, 15),
                                                         (0.6, 200, 0.5, 16), (1.0, 1, 1.0, 17)])
def test_sample_matches_oracle(cuda, V, temperature, top_k, top_p, seed):
    from edgeexpert_b200.sampling import Sample
    p = _probs(V, seed + V)
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    pd = torch.from_numpy(p.view(np.float16)).cuda()
    Sample().encode(pd, out, V, temperature, top_k, top_p, seed, position=5)
    torch.cuda.synchronize()
    assert int(out.item()) == O.sample(p, temperature, top_k, top_p, seed, 5)


@pytest.mark.parametrize("V,temperature,top_p,seed", [(262144, 1.0, 0.95, 3), (262144, 0.7, 1.0, 4), (100, 1.0, 0.5, 5)])
def test_sample_topk64_matches_oracle(cuda, V, temperature, top_p, seed):
    from edgeexpert_b200.sampling import SampleTopK64
    p = _probs(V, seed, 3.0)
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    SampleTopK64().encode(torch.from_numpy(p.view(np.float16)).cuda(), out, V, temperature, top_p, seed)
    torch.cuda.synchronize()
    assert int(out.item()) == O.sample_topk64(p, temperature, top_p, seed)


def test_sample_is_deterministic_and_seed_dependent(cuda):
    from edgeexpert_b200.sampling import Sample
    V = 50000
    p = torch.from_numpy(_probs(V, 99, 1.0).view(np.float16)).cuda()
    outs = []
    for seed in (1, 1, 2, 3, 4, 5):
        o = torch.zeros(1, dtype=torch.int32, device="cuda")
        Sample().encode(p, o, V, 1.0, 0, 1.0, seed)
        outs.append(int(o.item()))
    assert outs[0] == outs[1]
    assert len(set(outs[1:])) > 1
