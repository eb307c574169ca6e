"""Packed weight format helpers: expert blob layout and HBM residency.

The routed-expert blob is the one the reference repacker writes
(RepackPlanner.swift:1-7,380-445; MoEExpertOffsets, MoE.swift:4-29):
gate{W,s,b}, up{W,s,b}, down{W,s,b} back to back, identical offsets for every
expert of a layer, the blob stride rounded up to 16 KiB pages.  Each
sub-tensor starts on a 16-byte boundary here so the kernels can use bulk
copies; the bytes themselves are unchanged.

Synthetic weights follow the benchmark configuration distributions:
codes uniform, scale = |N(0, 0.02)|, bias = -(2^bits/2)*scale + N(0, 0.002).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ._lib import ExpertOffsets
from .moe import ExpertPool, MoELayerWeights, SharedExpertProjection

PAGE = 16 * 1024


def row_bytes(cols: int, bits: int) -> int:
    return cols if bits == 8 else cols * bits // 8


def affine_bytes(rows: int, cols: int, bits: int = 4) -> int:
    """Weights + scales + biases (2 bytes each per 64-group)."""
    return rows * row_bytes(cols, bits) + 2 * rows * (cols // 64) * 2


def _align(v: int, a: int = 16) -> int:
    return (v + a - 1) // a * a


@dataclass
class ExpertLayout:
    d: int
    f: int
    offsets: ExpertOffsets
    used: int
    stride: int

    def sub(self, name: str) -> tuple[int, int]:
        """(offset, bytes) of one sub-tensor."""
        o = getattr(self.offsets, name)
        rows, cols = (self.f, self.d) if name.startswith(("gate", "up")) else (self.d, self.f)
        n = rows * (cols // 2) if name.endswith("_w") else rows * (cols // 64) * 2
        return o, n


def expert_layout(d: int, f: int, page: int = PAGE, bits: int = 4) -> ExpertLayout:
    """Blob order gate{W,s,b}, up{W,s,b}, down{W,s,b}, each 16-byte aligned;
    `bits` 2/3/4 sets the packed weight size (rows * cols * bits / 8)."""
    off = {}
    cur = 0
    for proj, rows, cols in (("gate", f, d), ("up", f, d), ("down", d, f)):
        off[f"{proj}_w"] = cur
        cur = _align(cur + rows * cols * bits // 8)
        off[f"{proj}_s"] = cur
        cur = _align(cur + rows * (cols // 64) * 2)
        off[f"{proj}_b"] = cur
        cur = _align(cur + rows * (cols // 64) * 2)
    offsets = ExpertOffsets(**off)
    return ExpertLayout(d, f, offsets, cur, _align(cur, page))


def _fill_affine_(W: torch.Tensor, S: torch.Tensor, B: torch.Tensor, bits: int, gen: torch.Generator):
    """In-place synthetic fill (device RNG) of one affine tensor's three parts."""
    W.copy_(torch.randint(0, 256, W.shape, dtype=torch.uint8, device=W.device, generator=gen))
    s = torch.randn(S.shape, device=S.device, generator=gen, dtype=torch.float32).abs_().mul_(0.02)
    b = torch.randn(B.shape, device=B.device, generator=gen, dtype=torch.float32).mul_(0.002)
    b.add_(s, alpha=-float(1 << (bits - 1)))
    S.copy_(s.to(S.dtype))
    B.copy_(b.to(B.dtype))


def synthetic_affine(rows: int, cols: int, bits: int, scale_dtype=torch.bfloat16, device="cuda",
                     gen: torch.Generator | None = None):
    W = torch.empty(rows, row_bytes(cols, bits), dtype=torch.uint8, device=device)
    S = torch.empty(rows, cols // 64, dtype=scale_dtype, device=device)
    B = torch.empty(rows, cols // 64, dtype=scale_dtype, device=device)
    _fill_affine_(W, S, B, bits, gen)
    return W, S, B


def synthetic_expert_pool(num_experts: int, d: int, f: int, scale_dtype=torch.bfloat16, device="cuda",
                          gen: torch.Generator | None = None) -> ExpertPool:
    lay = expert_layout(d, f)
    blob = torch.zeros(num_experts, lay.stride, dtype=torch.uint8, device=device)
    o = lay.offsets
    for proj, rows, cols in (("gate", f, d), ("up", f, d), ("down", d, f)):
        ow, os_, ob = getattr(o, f"{proj}_w"), getattr(o, f"{proj}_s"), getattr(o, f"{proj}_b")
        nw, ns = rows * cols // 2, rows * (cols // 64) * 2
        W = blob[:, ow:ow + nw]
        S = blob[:, os_:os_ + ns].view(scale_dtype)
        B = blob[:, ob:ob + ns].view(scale_dtype)
        tW = torch.empty_like(W)
        tS = torch.empty_like(S)
        tB = torch.empty_like(B)
        _fill_affine_(tW, tS, tB, 4, gen)
        W.copy_(tW)
        S.copy_(tS)
        B.copy_(tB)
    return ExpertPool(blob.view(-1), lay.stride, num_experts, o, d, f, scale_dtype)


def expert_pool_from_host(blobs: list, layout: ExpertLayout, scale_dtype=torch.bfloat16,
                          device="cuda") -> ExpertPool:
    """Upload host blobs (numpy uint8 arrays of layout.used bytes) into one pool."""
    import numpy as np
    n = len(blobs)
    host = np.zeros((n, layout.stride), np.uint8)
    for i, b in enumerate(blobs):
        host[i, :b.size] = b
    t = torch.from_numpy(host.reshape(-1)).to(device)
    return ExpertPool(t, layout.stride, n, layout.offsets, layout.d, layout.f, scale_dtype)


def synthetic_moe_layer(d: int = 2816, f: int = 704, fs: int = 2112, num_experts: int = 128, top_k: int = 8,
                        shared_bits: int = 4, scale_dtype=torch.bfloat16, device="cuda",
                        gen: torch.Generator | None = None) -> MoELayerWeights:
    """Random-initialised MoE decode layer with the benchmark distributions."""
    rw, rs, rb = synthetic_affine(num_experts, d, 8, scale_dtype, device, gen)
    es = torch.ones(d, dtype=torch.bfloat16, device=device)
    es.mul_(float(d) ** -0.5)  # effective scale = router.scale * D^-1/2 (RealForwardRunner.swift:604-628)
    pes = (1.0 + 0.05 * torch.randn(num_experts, device=device, generator=gen)).to(torch.bfloat16)
    pool = synthetic_expert_pool(num_experts, d, f, scale_dtype, device, gen)
    shared = [None, None, None]
    if fs:
        gW, gS, gB = synthetic_affine(fs, d, shared_bits, scale_dtype, device, gen)
        uW, uS, uB = synthetic_affine(fs, d, shared_bits, scale_dtype, device, gen)
        dW, dS, dB = synthetic_affine(d, fs, shared_bits, scale_dtype, device, gen)
        shared = [SharedExpertProjection(gW, gS, gB, fs, d, shared_bits),
                  SharedExpertProjection(uW, uS, uB, fs, d, shared_bits),
                  SharedExpertProjection(dW, dS, dB, d, fs, shared_bits)]
    return MoELayerWeights(rw, rs, rb, es, pes, pool, *shared, top_k=top_k)


def moe_layer_bytes(d: int = 2816, f: int = 704, fs: int = 2112, num_experts: int = 128, top_k: int = 8,
                    shared_bits: int = 4) -> int:
    """Algorithmic HBM bytes of one decode-layer step for one token: every
    weight byte read once (router, top_k routed experts, shared expert) plus
    activations in/out."""
    routed = 2 * affine_bytes(f, d) + affine_bytes(d, f)
    shared = 2 * affine_bytes(fs, d, shared_bits) + affine_bytes(d, fs, shared_bits) if fs else 0
    router = affine_bytes(num_experts, d, 8) + 2 * d + 2 * num_experts
    acts = 2 * d * 2 + 2 * d  # router_x, x in; y out
    return top_k * routed + shared + router + acts
