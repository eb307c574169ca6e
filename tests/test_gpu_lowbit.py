"""GPU parity of the 2-bit and 3-bit paths (the rebits output) against the
oracle's kernel-order restatement of moe.metal:644-1180 and
dequant_int4.metal:512-717, through the C ABI:

* tf_affine_gemv_batched with bits 2 / 3: 1..8 tokens, several matrices,
  ragged row counts, groups past the last full 4-group block;
* tf_moe_phase1_bits / tf_moe_phase2_bits: pool (device ids) and blob
  addressing, BF16 and FP16 scales, the Gemma 4 shape (d 2816, f 704, top-8)
  and a small ragged one; a bad expert id raises the device flag.

Tolerance: max relative error (RelError) <= 2e-3 for the fp16 outputs; the
kernels compute the same products exactly and differ from the reference only
in the fp32 summation order.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
FP16_TOL = 2e-3


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.view(dtype) if dtype is not None else t


def sdt(st):
    return torch.float16 if st == 1 else torch.bfloat16


def f16(t):
    return O.f16_to_f32(t.view(torch.int16).cpu().numpy().view(np.uint16))


@pytest.mark.parametrize("bits", [2, 3])
@pytest.mark.parametrize("m,n,ntok,batch,st", [(2816, 704, 1, 1, 0), (704, 2816, 1, 3, 1), (100, 192, 3, 2, 0),
                                               (1408, 2816, 8, 1, 1), (37, 64, 2, 1, 0), (4096, 2816, 1, 1, 0)])
def test_lowbit_gemv_matches_oracle(cuda, bits, m, n, ntok, batch, st):
    from edgeexpert_b200.quant import affine_gemv_batched
    rng = O.seed_tree(bits * 1000 + m + n, f"lowbit-gemv-{ntok}-{batch}-{st}")
    mats = [rng.synthetic_affine(m, n, bits, st) for _ in range(batch)]
    X = np.stack([rng.normal_f16(n) for _ in range(ntok)])
    W = dev(np.stack([w for w, _, _ in mats]).reshape(-1))
    S = dev(np.stack([s for _, s, _ in mats]).reshape(-1), sdt(st))
    B = dev(np.stack([b for _, _, b in mats]).reshape(-1), sdt(st))
    x = dev(X, torch.float16)
    y = torch.full((batch, ntok, m), float("nan"), dtype=torch.float16, device="cuda")
    affine_gemv_batched(W, S, B, x, y, bits=bits, m=m, n=n, batch=batch, ntok=ntok,
                        w_stride_bytes=mats[0][0].size, sb_stride=mats[0][1].size, x_row_stride=n, y_row_stride=m,
                        y_batch_stride=ntok * m)
    torch.cuda.synchronize()
    got = f16(y)
    for i, (Wi, Si, Bi) in enumerate(mats):
        for t in range(ntok):
            ref32, _ = O.lowbit_gemv_kernel_order(Wi, Si, Bi, X[t], bits, st)
            err = O.rel_error(got[i, t], ref32)
            assert err <= FP16_TOL, (i, t, err)


def make_experts(E, d, f, bits, st, seed):
    from edgeexpert_b200.format import expert_layout
    lay = expert_layout(d, f, bits=bits)
    rng = O.seed_tree(seed, f"lowbit-experts-{bits}-{st}")
    o = lay.offsets
    host = np.zeros((E, lay.stride), np.uint8)
    for e in range(E):
        for proj, rows, cols in (("gate", f, d), ("up", f, d), ("down", d, f)):
            W, S, B = rng.synthetic_affine(rows, cols, bits, st)
            for part, arr in (("w", W), ("s", S), ("b", B)):
                b = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
                off = getattr(o, f"{proj}_{part}")
                host[e, off:off + b.size] = b
    return host, lay


def device_flags():
    from edgeexpert_b200._lib import Context, lib
    flags = C.c_uint32(0)
    lib().tf_context_check_device(Context.get(0).handle, C.c_void_p(0), C.byref(flags))
    return flags.value


@pytest.mark.parametrize("bits", [2, 3])
@pytest.mark.parametrize("E,d,f,top_k,st,pool", [(16, 2816, 704, 8, 0, True), (16, 2816, 704, 8, 1, False),
                                                 (5, 192, 128, 3, 0, True), (4, 320, 64, 2, 1, False)])
def test_lowbit_phases_match_oracle(cuda, bits, E, d, f, top_k, st, pool):
    from edgeexpert_b200.moe import MoE, ExpertPool
    device_flags()  # clear what earlier tests left
    host, lay = make_experts(E, d, f, bits, st, 17 + E)
    rng = O.seed_tree(E * 7 + d, f"lowbit-phase-{bits}-{st}")
    ids = np.array(rng.uniform(0, 1, E).argsort()[:top_k], np.uint32)
    x16 = rng.normal_f16(d)
    w16 = O.f32_to_f16(rng.uniform(0.05, 0.3, top_k))
    res16 = rng.normal_f16(d)
    off = O.Offsets(*[getattr(lay.offsets, n) for n, _ in O.Offsets._fields_])
    blobs_h = [np.ascontiguousarray(host[e]) for e in ids]
    acts_ref = O.moe_phase1_bits(blobs_h, off, x16, d, f, bits, st)
    y_ref16, y_ref32 = O.moe_phase2_bits(blobs_h, off, acts_ref, w16, res16, d, f, bits, st)

    moe = MoE()
    if pool:
        experts = ExpertPool(dev(host.reshape(-1)), lay.stride, E, lay.offsets, d, f, sdt(st), bits)
        kw = dict(expert_ids=dev(ids))
    else:
        blobs = [dev(host[e]) for e in ids]
        experts = (blobs, lay.offsets, sdt(st))
        kw = {}
    x = dev(x16, torch.float16)
    acts = torch.full((top_k * f,), float("nan"), dtype=torch.float16, device="cuda")
    moe.encode_routed_phase1(experts, x, acts, d, f, top_k, bits=bits, **kw)
    torch.cuda.synchronize()
    err1 = O.rel_error(f16(acts), O.f16_to_f32(acts_ref))
    assert err1 <= FP16_TOL, err1

    # phase 2 on the oracle's acts, so each phase is checked on its own
    acts_in = dev(acts_ref, torch.float16)
    y = torch.full((d,), float("nan"), dtype=torch.float16, device="cuda")
    moe.encode_routed_phase2_reduce(experts, acts_in, dev(w16, torch.float16), dev(res16, torch.float16), y, d, f,
                                    top_k, bits=bits, **kw)
    torch.cuda.synchronize()
    err2 = O.rel_error(f16(y), y_ref32)
    assert err2 <= FP16_TOL, err2
    assert device_flags() == 0


def test_lowbit_bad_expert_id_raises_flag(cuda):
    from edgeexpert_b200.moe import MoE, ExpertPool
    device_flags()
    E, d, f, k = 4, 192, 64, 2
    host, lay = make_experts(E, d, f, 3, 0, 5)
    experts = ExpertPool(dev(host.reshape(-1)), lay.stride, E, lay.offsets, d, f, torch.bfloat16, 3)
    ids = dev(np.array([1, 9], np.uint32))  # 9 >= num_experts
    x = torch.zeros(d, dtype=torch.float16, device="cuda")
    acts = torch.zeros(k * f, dtype=torch.float16, device="cuda")
    MoE().encode_routed_phase1(experts, x, acts, d, f, k, expert_ids=ids, bits=3)
    torch.cuda.synchronize()
    assert device_flags() & 2  # kErrBadExpert


def test_lowbit_rejects_bad_arguments(cuda):
    from edgeexpert_b200._lib import TF_ERR_MISALIGNED, TF_ERR_UNSUPPORTED_SHAPE, Context, ExpertOffsets, lib
    ctx = Context.get(0).handle
    z = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    p = C.c_void_p(z.data_ptr())
    off = ExpertOffsets(0, 4096, 8192, 12288, 16384, 20480, 24576, 28672, 32768)
    ids = C.c_void_p(z.data_ptr() + 60000)
    assert lib().tf_moe_phase1_bits(ctx, 5, p, 65536, 1, ids, None, C.byref(off), p, p, 64, 64, 1, 0,
                                    C.c_void_p(0)) == TF_ERR_UNSUPPORTED_SHAPE
    bad = ExpertOffsets(4, 4096, 8192, 12288, 16384, 20480, 24576, 28672, 32768)  # gate_w not 8-byte aligned
    assert lib().tf_moe_phase1_bits(ctx, 3, p, 65536, 1, ids, None, C.byref(bad), p, p, 64, 64, 1, 0,
                                    C.c_void_p(0)) == TF_ERR_MISALIGNED
