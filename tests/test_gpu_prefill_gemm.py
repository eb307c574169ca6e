"""GPU parity of the tensor-core prefill GEMMs against the C oracle.

* tf_int4_qmm              vs orc_int4_qmm (PrefillInt4QMM, prefill.metal:672-709)
* tf_prefill_shared_expert vs the per-token shared expert (SharedExpertRuntime arithmetic)
* tf_moe_grouped_routed    vs orc_grouped_routed (prefill.metal:336-440,598-670)
* tf_moe_reduce_token_major vs orc_reduce_token_major (bit-exact: same fma order)
Tolerance: RelError (RelError.swift:7-16) <= 2e-3 for fp16 outputs.
"""
import numpy as np
import pytest
import torch

import oracle as O
from edgeexpert_b200.prefill import (PrefillGroupedRoutedMoE, PrefillInt4QMM, PrefillMoE, PrefillRouter,
                                     PrefillSharedExpert, route_sort)

pytestmark = pytest.mark.gpu
FP16_TOL = 2e-3


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.view(dtype) if dtype is not None else t


def f16(t):
    return t.cpu().numpy().view(np.uint16)


def sdt(scale_type):
    return torch.bfloat16 if scale_type == 0 else torch.float16


@pytest.mark.parametrize("T,N,K,st", [(1, 128, 64, 0), (17, 200, 128, 0), (300, 2112, 2816, 0), (256, 384, 704, 0),
                                      (257, 128, 256, 1), (513, 136, 192, 0)])
def test_int4_qmm(cuda, T, N, K, st):
    rng = O.seed_tree(T * 31 + N, f"qmm-{K}-{st}")
    W, S, B = rng.synthetic_affine(N, K, 4, st)
    X = rng.normal_f16(T * K).reshape(T, K)
    _, y32 = O.int4_qmm(W, S, B, X, T, N, K, st)
    y = torch.empty(T, N, dtype=torch.float16, device="cuda")
    PrefillInt4QMM().encode(dev(W), dev(S, sdt(st)), dev(B, sdt(st)), dev(X, torch.float16), y, T, N, K)
    torch.cuda.synchronize()
    assert O.rel_error(O.f16_to_f32(f16(y)), y32) < FP16_TOL


@pytest.mark.parametrize("T,N,K", [(300, 2112, 2816), (17, 200, 128)])
def test_int4_qmm_cta_pairs(cuda, T, N, K, monkeypatch):
    """The 2-SM (CTA pair) variant, selected with TFCUDA_QMM_PAIR=1."""
    monkeypatch.setenv("TFCUDA_QMM_PAIR", "1")
    rng = O.seed_tree(T * 7 + N, f"qmm-pair-{K}")
    W, S, B = rng.synthetic_affine(N, K, 4, 0)
    X = rng.normal_f16(T * K).reshape(T, K)
    _, y32 = O.int4_qmm(W, S, B, X, T, N, K, 0)
    y = torch.empty(T, N, dtype=torch.float16, device="cuda")
    PrefillInt4QMM().encode(dev(W), dev(S, torch.bfloat16), dev(B, torch.bfloat16), dev(X, torch.float16), y, T, N, K)
    torch.cuda.synchronize()
    assert O.rel_error(O.f16_to_f32(f16(y)), y32) < FP16_TOL


@pytest.mark.parametrize("pair", ["0", "1"])
def test_grouped_routed_config1_shapes_both_variants(cuda, pair, monkeypatch):
    monkeypatch.setenv("TFCUDA_QMM_PAIR", pair)
    T, K, E, D, F = 48, 8, 16, 2816, 704
    ex = Experts(E, D, F, 0, "g-variants")
    idx, w = skewed_routing(T, K, E, 99)
    X = O.seed_tree(T, "gx-variants").normal_f16(T * D).reshape(T, D)
    pairs = PrefillRouter.make_token_expert_pairs(idx, w, T, K)
    ref = O.group_pairs(pairs, T, K, E, 16)
    part_ref = O.grouped_routed(ex.host.reshape(-1), ex.lay.stride, ex.off, ref["sorted"], X, D, D, F, K, T, 0)
    routes = route_sort(dev(idx.view(np.int32)), dev(w), T, K, E, 16)
    act = torch.empty(T * K, F, dtype=torch.float16, device="cuda")
    part = torch.empty(T * K, D, dtype=torch.float16, device="cuda")
    PrefillGroupedRoutedMoE().encode(ex.pool(), routes, dev(X, torch.float16), act, part, T, K)
    torch.cuda.synchronize()
    assert O.rel_error(O.f16_to_f32(f16(part)), O.f16_to_f32(part_ref)) < FP16_TOL


def test_int4_qmm_strided_rows(cuda):
    T, N, K, LX, LY = 40, 256, 256, 320, 272
    rng = O.seed_tree(5, "qmm-strided")
    W, S, B = rng.synthetic_affine(N, K, 4, 0)
    X = rng.normal_f16(T * K).reshape(T, K)
    Xs = np.zeros((T, LX), np.uint16)
    Xs[:, :K] = X
    _, y32 = O.int4_qmm(W, S, B, X, T, N, K, 0)
    y = torch.full((T, LY), 7.0, dtype=torch.float16, device="cuda")
    PrefillInt4QMM().encode(dev(W), dev(S, torch.bfloat16), dev(B, torch.bfloat16), dev(Xs, torch.float16), y, T,
                            N, K, x_stride=LX, y_stride=LY)
    torch.cuda.synchronize()
    out = y.cpu().float().numpy()
    assert O.rel_error(out[:, :N].reshape(-1), y32) < FP16_TOL
    assert np.all(out[:, N:] == 7.0)  # nothing written past n


def test_int4_qmm_deterministic(cuda):
    T, N, K = 300, 384, 512
    rng = O.seed_tree(8, "qmm-det")
    W, S, B = rng.synthetic_affine(N, K, 4, 0)
    X = rng.normal_f16(T * K).reshape(T, K)
    args = (dev(W), dev(S, torch.bfloat16), dev(B, torch.bfloat16), dev(X, torch.float16))
    ys = []
    for _ in range(2):
        y = torch.empty(T, N, dtype=torch.float16, device="cuda")
        PrefillInt4QMM().encode(*args, y, T, N, K)
        ys.append(f16(y))
    torch.cuda.synchronize()
    assert np.array_equal(ys[0], ys[1])


@pytest.mark.parametrize("T,D,Fs", [(5, 128, 64), (40, 2816, 2112)])
def test_prefill_shared_expert(cuda, T, D, Fs):
    from edgeexpert_b200.moe import SharedExpertProjection
    rng = O.seed_tree(T, f"pshared-{D}")
    g = rng.synthetic_affine(Fs, D, 4, 0)
    u = rng.synthetic_affine(Fs, D, 4, 0)
    d = rng.synthetic_affine(D, Fs, 4, 0)
    X = rng.normal_f16(T * D).reshape(T, D)
    act_ref = np.empty((T, Fs), np.uint16)
    y_ref = np.empty((T, D), np.float32)
    for t in range(T):
        a, _, y32 = O.shared_expert(g, u, d, X[t], D, Fs, 4)
        act_ref[t], y_ref[t] = a, y32

    def proj(m, rows, cols):
        return SharedExpertProjection(dev(m[0]), dev(m[1], torch.bfloat16), dev(m[2], torch.bfloat16), rows, cols, 4)
    act = torch.empty(T, Fs, dtype=torch.float16, device="cuda")
    y = torch.empty(T, D, dtype=torch.float16, device="cuda")
    PrefillSharedExpert().encode(dev(X, torch.float16), proj(g, Fs, D), proj(u, Fs, D), proj(d, D, Fs), act, y, T)
    torch.cuda.synchronize()
    assert O.rel_error(O.f16_to_f32(f16(act)), O.f16_to_f32(act_ref)) < FP16_TOL
    assert O.rel_error(O.f16_to_f32(f16(y)), y_ref) < FP16_TOL


class Experts:
    """num_experts random experts in the reference blob layout (host + pool)."""

    def __init__(self, E, D, F, scale_type=0, label="gexperts"):
        from edgeexpert_b200.format import expert_layout
        self.E, self.D, self.F, self.st = E, D, F, scale_type
        self.lay = expert_layout(D, F)
        rng = O.seed_tree(0xE1, label)
        o = self.lay.offsets
        self.host = np.zeros((E, self.lay.stride), np.uint8)
        for e in range(E):
            for proj, rows, cols in (("gate", F, D), ("up", F, D), ("down", D, F)):
                W, S, B = rng.synthetic_affine(rows, cols, 4, scale_type)
                for part, arr in (("w", W), ("s", S), ("b", B)):
                    b = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
                    off = getattr(o, f"{proj}_{part}")
                    self.host[e, off:off + b.size] = b
        self.off = O.Offsets(*[getattr(o, n) for n, _ in O.Offsets._fields_])

    def pool(self):
        from edgeexpert_b200.moe import ExpertPool
        return ExpertPool(dev(self.host.reshape(-1)), self.lay.stride, self.E, self.lay.offsets, self.D, self.F,
                          sdt(self.st))


def skewed_routing(T, K, E, seed):
    rng = np.random.default_rng(seed)
    p = rng.random(E) ** 3 + 1e-3
    p /= p.sum()
    idx = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T)]).astype(np.uint32)
    w = (rng.random((T, K)) * 0.3 + 0.05).astype(np.float16)
    return idx, w


@pytest.mark.parametrize("path", ["gemm", "gemv", "engine"])
@pytest.mark.parametrize("T,K,E,D,F,st", [(37, 4, 16, 128, 64, 0), (300, 2, 2, 128, 64, 0), (64, 8, 16, 2816, 704, 0),
                                          (9, 8, 32, 256, 128, 1), (64, 8, 128, 2816, 704, 0),
                                          (256, 8, 128, 2816, 704, 0), (40, 2, 2, 2816, 704, 1)])
def test_grouped_routed_and_reduce(cuda, T, K, E, D, F, st, path, monkeypatch):
    """Every device path: tcgen05 GEMMs (many tokens per expert), the grouped
    ring-streamed kernel (few tokens per expert, batched decode; config 2 is
    T = 64, K = 8 over 128 experts) and the older streaming-engine policy."""
    monkeypatch.setenv("TFCUDA_GROUPED", path)
    ex = Experts(E, D, F, st, f"g-{E}-{D}-{F}-{st}")
    idx, w = skewed_routing(T, K, E, T + E)
    X = O.seed_tree(T, f"gx-{D}").normal_f16(T * D).reshape(T, D)
    pairs = PrefillRouter.make_token_expert_pairs(idx, w, T, K)
    ref = O.group_pairs(pairs, T, K, E, 16)
    part_ref = O.grouped_routed(ex.host.reshape(-1), ex.lay.stride, ex.off, ref["sorted"], X, D, D, F, K, T, st)
    routes = route_sort(dev(idx.view(np.int32)), dev(w), T, K, E, 16)
    act = torch.empty(T * K, F, dtype=torch.float16, device="cuda")
    part = torch.empty(T * K, D, dtype=torch.float16, device="cuda")
    PrefillGroupedRoutedMoE().encode(ex.pool(), routes, dev(X, torch.float16), act, part, T, K)
    torch.cuda.synchronize()
    assert O.rel_error(O.f16_to_f32(f16(part)), O.f16_to_f32(part_ref)) < FP16_TOL
    # token-major reduce of the oracle's partials: same fma order, bit-exact
    h2 = torch.empty(T, D, dtype=torch.float16, device="cuda")
    PrefillMoE.encode_reduce_token_major(dev(part_ref, torch.float16), dev(w), h2, T, K, D)
    torch.cuda.synchronize()
    h2_ref = O.reduce_token_major(part_ref, w.view(np.uint16), T, K, D)
    assert np.array_equal(f16(h2).reshape(-1), h2_ref)


@pytest.mark.parametrize("expected", [0, 1024, 100000])
def test_grouped_routed_expected_pairs(cuda, expected, monkeypatch):
    """tf_moe_grouped_routed_expected: the pair estimate only picks the kernel
    (T*K = 2048 pairs over 64 experts selects the tcgen05 GEMMs; an estimate
    of 1024, as expert parallelism over 2 GPUs passes, the grouped
    ring-streamed kernel; an estimate above T*K is clamped to it), and every
    choice matches the oracle."""
    monkeypatch.delenv("TFCUDA_GROUPED", raising=False)
    T, K, E, D, F, st = 256, 8, 64, 2816, 704, 0
    ex = Experts(E, D, F, st, f"g-{E}-{D}-{F}-{st}")
    idx, w = skewed_routing(T, K, E, T + E)
    X = O.seed_tree(T, f"gx-{D}").normal_f16(T * D).reshape(T, D)
    pairs = PrefillRouter.make_token_expert_pairs(idx, w, T, K)
    ref = O.group_pairs(pairs, T, K, E, 16)
    part_ref = O.grouped_routed(ex.host.reshape(-1), ex.lay.stride, ex.off, ref["sorted"], X, D, D, F, K, T, st)
    routes = route_sort(dev(idx.view(np.int32)), dev(w), T, K, E, 16)
    act = torch.empty(T * K, F, dtype=torch.float16, device="cuda")
    part = torch.empty(T * K, D, dtype=torch.float16, device="cuda")
    PrefillGroupedRoutedMoE().encode(ex.pool(), routes, dev(X, torch.float16), act, part, T, K,
                                     expected_pairs=expected)
    torch.cuda.synchronize()
    assert O.rel_error(O.f16_to_f32(f16(part)), O.f16_to_f32(part_ref)) < FP16_TOL


@pytest.mark.parametrize("path", ["gemm", "gemv", "engine"])
def test_grouped_routed_empty_routes(cuda, path, monkeypatch):
    """A route table with no groups runs no tile; T = 0 touches nothing."""
    monkeypatch.setenv("TFCUDA_GROUPED", path)
    ex = Experts(4, 128, 64, 0, "g-empty")
    T, K = 3, 2
    routes = route_sort(dev(np.zeros((T, K), np.int32)), dev(np.zeros((T, K), np.float16)), T, K, 4, 16)
    routes.n_groups.zero_()
    part = torch.full((T * K, 128), 3.0, dtype=torch.float16, device="cuda")
    act = torch.empty(T * K, 64, dtype=torch.float16, device="cuda")
    PrefillGroupedRoutedMoE().encode(ex.pool(), routes, torch.zeros(T, 128, dtype=torch.float16, device="cuda"),
                                     act, part, T, K)
    torch.cuda.synchronize()
    part.fill_(3.0)
    PrefillGroupedRoutedMoE().encode(ex.pool(), routes, torch.zeros(T, 128, dtype=torch.float16, device="cuda"),
                                     act, part, 0, K)
    torch.cuda.synchronize()
    assert bool((part == 3.0).all())


def test_prefill_argument_validation(cuda):
    """Contract violations return a status (the reference traps); nothing launches."""
    from edgeexpert_b200._lib import TFError
    W = torch.zeros(128, 64, dtype=torch.uint8, device="cuda")
    S = torch.zeros(128, 2, dtype=torch.bfloat16, device="cuda")
    X = torch.zeros(4, 128, dtype=torch.float16, device="cuda")
    Y = torch.zeros(4, 128, dtype=torch.float16, device="cuda")
    q = PrefillInt4QMM()
    with pytest.raises(TFError) as ei:
        q.encode(W, S, S, X, Y, 4, 128, 100)  # k % 64 != 0
    assert ei.value.status == 3
    with pytest.raises(TFError) as ei:
        q.encode(W, S, S, X, Y, 4, 128, 128, x_stride=100)  # stride not a multiple of 8
    assert ei.value.status == 3
    Xu = torch.zeros(4 * 128 + 1, dtype=torch.float16, device="cuda")[1:].view(4, 128)  # 2-byte aligned only
    with pytest.raises(TFError) as ei:
        q.encode(W, S, S, Xu, Y, 4, 128, 128)
    assert ei.value.status == 2
    # T = 0: nothing to do
    q.encode(W, S, S, X, Y, 0, 128, 128)
    with pytest.raises(TFError) as ei:
        PrefillMoE.encode_reduce_token_major(Y, Y, Y, 4, 8, 100)  # d % 8 != 0
    assert ei.value.status == 3


def test_prefill_config3_t4096_values(cuda):
    """BASELINE config 3 at full size: 4096 tokens, 128 experts (D=2816, F=704),
    top-8, through the tcgen05 grouped GEMMs and the token-major reduce, plus
    the shared expert (Fs=2112) on the tcgen05 dense GEMMs.  Values are checked
    against the oracle (fp32 fma(fma(q,s,b),x,acc) per element, the reference's
    prefill.metal:336-440,598-709 arithmetic) on 256 token rows spread over the
    batch, and every expert is hit.  This settles the one rounding difference
    (w rounded to fp16 once before the tensor-core product) at the
    configuration BASELINE names."""
    from edgeexpert_b200.moe import SharedExpertProjection
    T, K, E, D, F, Fs = 4096, 8, 128, 2816, 704, 2112
    ex = Experts(E, D, F, 0, "cfg3-4096")
    rng = np.random.default_rng(4096)
    p = rng.random(E) ** 2 + 0.05
    p /= p.sum()
    idx = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T)]).astype(np.uint32)
    w = (rng.random((T, K)) * 0.3 + 0.05).astype(np.float16)
    X = rng.standard_normal((T, D)).astype(np.float16).view(np.uint16)
    routes = route_sort(dev(idx.view(np.int32)), dev(w), T, K, E, 16)
    act = torch.empty(T * K, F, dtype=torch.float16, device="cuda")
    part = torch.empty(T * K, D, dtype=torch.float16, device="cuda")
    PrefillGroupedRoutedMoE().encode(ex.pool(), routes, dev(X, torch.float16), act, part, T, K)
    h2 = torch.empty(T, D, dtype=torch.float16, device="cuda")
    PrefillMoE.encode_reduce_token_major(part, dev(w), h2, T, K, D)

    srng = O.seed_tree(5, "cfg3-shared")
    g = srng.synthetic_affine(Fs, D, 4, 0)
    u = srng.synthetic_affine(Fs, D, 4, 0)
    dn = srng.synthetic_affine(D, Fs, 4, 0)

    def proj(m, rows, cols):
        return SharedExpertProjection(dev(m[0]), dev(m[1], torch.bfloat16), dev(m[2], torch.bfloat16), rows, cols, 4)
    sact = torch.empty(T, Fs, dtype=torch.float16, device="cuda")
    sy = torch.empty(T, D, dtype=torch.float16, device="cuda")
    PrefillSharedExpert().encode(dev(X, torch.float16), proj(g, Fs, D), proj(u, Fs, D), proj(dn, D, Fs), sact, sy, T)
    torch.cuda.synchronize()
    assert int(np.count_nonzero(np.bincount(idx.reshape(-1), minlength=E))) == E

    sample = np.unique(np.linspace(0, T - 1, 256).astype(np.int64))
    pairs = PrefillRouter.make_token_expert_pairs(idx, w, T, K)
    ref = O.group_pairs(pairs, T, K, E, 16)
    srt = ref["sorted"]
    sub = srt[np.isin(srt["token"], sample)]
    part_ref = O.grouped_routed(ex.host.reshape(-1), ex.lay.stride, ex.off, sub, X, D, D, F, K, T, 0)
    part_ref = part_ref.reshape(T, K, D)[sample]
    got_part = f16(part).reshape(T, K, D)[sample]
    assert O.rel_error(O.f16_to_f32(got_part), O.f16_to_f32(part_ref)) < FP16_TOL
    h2_ref = O.reduce_token_major(part_ref.reshape(-1), w[sample].view(np.uint16), len(sample), K, D)
    got_h2 = f16(h2).reshape(T, D)[sample]
    assert O.rel_error(O.f16_to_f32(got_h2), O.f16_to_f32(h2_ref)) < FP16_TOL

    y_ref = np.empty((len(sample), D), np.float32)
    for i, t in enumerate(sample):
        _, _, y_ref[i] = O.shared_expert(g, u, dn, X[t], D, Fs, 4)
    assert O.rel_error(O.f16_to_f32(f16(sy).reshape(T, D)[sample]), y_ref) < FP16_TOL

    # the dense QMM alone (gate projection) on the same rows
    _, q32 = O.int4_qmm(g[0], g[1], g[2], X[sample], len(sample), Fs, D, 0)
    yq = torch.empty(T, Fs, dtype=torch.float16, device="cuda")
    PrefillInt4QMM().encode(dev(g[0]), dev(g[1], torch.bfloat16), dev(g[2], torch.bfloat16), dev(X, torch.float16), yq,
                            T, Fs, D)
    torch.cuda.synchronize()
    assert O.rel_error(O.f16_to_f32(f16(yq).reshape(T, Fs)[sample]), q32.reshape(len(sample), Fs)) < FP16_TOL
