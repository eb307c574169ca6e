"""GPU parity of the ring-streamed one-token int4 GEMVs (tf_gemv_tc.cu) against the oracle.

Both kernels are reached through the public entry points tf_int4_gemv and
tf_affine_gemv_batched: the integer mma.sync kernel ("stream", the default
when a call has at least one 128-row tile per SM) and the tcgen05 kernel
("tc", opt-in).  TFCUDA_GEMV forces either for any tile count.
Tolerance: max relative error (RelError) <= 2e-3 for fp16 outputs, the
reference's own kernel-vs-CPU bar (Tolerances.swift:4-21).
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

FP16_TOL = 2e-3


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.view(dtype) if dtype is not None else t


def f16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def sdt(scale_type):
    return torch.float16 if scale_type == 1 else torch.bfloat16


def single(m, n, scale_type, label, uniform=False):
    from edgeexpert_b200.quant import DequantInt4GEMV
    rng = O.seed_tree(0x7C, label)
    if uniform:
        W, S, B = O.quantize_affine(rng.uniform(-0.5, 0.5, m * n).reshape(m, n), 4)
        x = O.f32_to_f16(rng.uniform(-1.0, 1.0, n))
    else:
        W, S, B = rng.synthetic_affine(m, n, 4, scale_type)
        x = rng.normal_f16(n)
    y = torch.empty(m, dtype=torch.float16, device="cuda")
    DequantInt4GEMV().encode(dev(W), dev(S, sdt(scale_type)), dev(B, sdt(scale_type)), dev(x, torch.float16), y, m, n)
    torch.cuda.synchronize()
    ref = O.affine_gemv_ref(W, S, B, O.f16_to_f32(x), 4, scale_type if not uniform else 0)
    return O.f16_to_f32(f16(y)), ref


@pytest.mark.parametrize("m,n", [(128, 128), (1024, 2816), (64, 64), (1408, 2816), (2816, 2112), (704, 2816),
                                 (2816, 704)])
@pytest.mark.parametrize("kind", ["stream", "tc"])
def test_ring_gemv_shapes(cuda, m, n, kind, monkeypatch):
    monkeypatch.setenv("TFCUDA_GEMV", kind)
    y, ref = single(m, n, 0, f"tc-{m}-{n}", uniform=True)
    assert O.rel_error(y, ref) < FP16_TOL


@pytest.mark.parametrize("m", [1, 65, 129, 200])
@pytest.mark.parametrize("n", [64, 192, 448, 512, 576, 1088])
@pytest.mark.parametrize("kind", ["stream", "tc"])
def test_ring_gemv_ragged(cuda, m, n, kind, monkeypatch):
    # partial 128-row tiles (scale blocks that are not a multiple of 16 bytes),
    # stages with fewer than 8 groups, a second TMA box outside the row
    monkeypatch.setenv("TFCUDA_GEMV", kind)
    y, ref = single(m, n, 0, f"tc-ragged-{m}-{n}", uniform=True)
    assert O.rel_error(y, ref) < FP16_TOL


@pytest.mark.parametrize("kind", ["stream", "tc"])
@pytest.mark.parametrize("scale_type", [0, 1])
def test_ring_gemv_config0(cuda, scale_type, kind, monkeypatch):
    monkeypatch.setenv("TFCUDA_GEMV", kind)
    y, ref = single(1408, 2816, scale_type, f"tc-cfg0-{scale_type}")
    assert O.rel_error(y, ref) < FP16_TOL


def batched(batch, m, n, scale_type, label, pad_w=0, pad_s=0):
    from edgeexpert_b200.quant import affine_gemv_batched
    rng = O.seed_tree(0x7D, label)
    mats = [rng.synthetic_affine(m, n, 4, scale_type) for _ in range(batch)]
    x = rng.normal_f16(n)
    rb, ng = n // 2, n // 64
    ws, ss = m * rb + pad_w, m * ng + pad_s
    Wh = np.zeros(batch * ws, np.uint8)
    Sh = np.zeros(batch * ss, np.uint16)
    Bh = np.zeros(batch * ss, np.uint16)
    for b, (w, s, bb) in enumerate(mats):
        Wh[b * ws:b * ws + m * rb] = w.reshape(-1)
        Sh[b * ss:b * ss + m * ng] = s.reshape(-1)
        Bh[b * ss:b * ss + m * ng] = bb.reshape(-1)
    Y = torch.zeros(batch, m + 3, dtype=torch.float16, device="cuda")
    affine_gemv_batched(dev(Wh), dev(Sh, sdt(scale_type)), dev(Bh, sdt(scale_type)), dev(x, torch.float16), Y,
                        bits=4, m=m, n=n, batch=batch, w_stride_bytes=ws, sb_stride=ss, y_batch_stride=m + 3)
    torch.cuda.synchronize()
    Yh = O.f16_to_f32(f16(Y)).reshape(batch, m + 3)
    xf = O.f16_to_f32(x)
    for b, (w, s, bb) in enumerate(mats):
        ref = O.affine_gemv_ref(w, s, bb, xf, 4, scale_type)
        assert O.rel_error(Yh[b, :m], ref) < FP16_TOL, b
    assert np.all(Yh[:, m:] == 0.0)  # nothing written past a matrix's rows
    return Yh


@pytest.mark.parametrize("kind", ["", "tc"])
def test_ring_gemv_batched_many_tiles(cuda, kind, monkeypatch):
    # 160 tiles: more jobs than SMs, each CTA runs several (persistent loop);
    # "" = the default selection (the integer ring kernel)
    if kind:
        monkeypatch.setenv("TFCUDA_GEMV", kind)
    else:
        monkeypatch.delenv("TFCUDA_GEMV", raising=False)
    batched(160, 128, 2816, 1, "tc-batched-auto")


@pytest.mark.parametrize("kind", ["stream", "tc"])
@pytest.mark.parametrize("pad_w,pad_s", [(0, 0), (48, 8), (4096, 24)])
def test_ring_gemv_batched_strides(cuda, pad_w, pad_s, kind, monkeypatch):
    monkeypatch.setenv("TFCUDA_GEMV", kind)
    batched(5, 200, 1088, 0, f"tc-batched-{pad_w}-{pad_s}", pad_w, pad_s)


@pytest.mark.parametrize("kind", ["stream", "tc"])
def test_ring_gemv_matches_engine_and_is_deterministic(cuda, kind, monkeypatch):
    monkeypatch.setenv("TFCUDA_GEMV", kind)
    a, _ = single(1408, 2816, 1, "tc-det")
    b, _ = single(1408, 2816, 1, "tc-det")
    assert np.array_equal(a, b)
    monkeypatch.setenv("TFCUDA_GEMV", "engine")
    e, ref = single(1408, 2816, 1, "tc-det")
    # same activation quantisation as the engine's integer path: the two paths
    # differ only in fp32 summation order
    assert O.rel_error(a, e) < 1e-3
    assert O.rel_error(e, ref) < FP16_TOL


@pytest.mark.parametrize("batch,m,n", [(300, 128, 2816), (100, 200, 1088), (149, 1408, 704)])
def test_stream_gemv_many_jobs_per_cta(cuda, batch, m, n, monkeypatch):
    # several jobs per CTA, some shorter than the stage ring (K = 704: two
    # stages), so a consumer warp can run jobs ahead of its partner
    monkeypatch.delenv("TFCUDA_GEMV", raising=False)
    a = batched(batch, m, n, 1, f"many-{batch}-{m}-{n}")
    b = batched(batch, m, n, 1, f"many-{batch}-{m}-{n}")
    assert np.array_equal(a, b)
