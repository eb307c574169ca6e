"""Dense affine GEMV operators (mirror of Sources/TurboFieldfare/Kernels/Quant).

``DequantInt4GEMV`` / ``DequantInt8GEMV`` keep the reference class names and
argument meaning (DequantInt4GEMV.swift:84-180, DequantInt8GEMV.swift:50-81):
``encode`` enqueues on a stream (the CommandBuffer analogue) and never syncs.
Buffers are torch CUDA tensors; byte offsets are expressed by slicing.
"""
from __future__ import annotations

import torch

from ._lib import TF_SCALE_BF16, TF_SCALE_F16, Context, lib, ptr, stream_ptr

GROUP_SIZE = 64


def scale_type_of(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return TF_SCALE_BF16
    if t.dtype == torch.float16:
        return TF_SCALE_F16
    raise TypeError(f"scales/biases must be bfloat16 (reference format) or float16, got {t.dtype}")


def _check_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("all buffers must be CUDA tensors")


class DequantInt4GEMV:
    """MLX-affine int4 matrix-vector product, y = W x (fp32 accumulate, fp16 out)."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, weights, scales, biases, x, y, m: int, n: int, stream=None) -> None:
        _check_cuda(weights, scales, biases, x, y)
        st = lib().tf_int4_gemv(self.ctx.handle, ptr(weights), ptr(scales), ptr(biases), ptr(x), ptr(y),
                                m, n, scale_type_of(scales), stream_ptr(stream))
        self.ctx.check(st, "DequantInt4GEMV.encode")

    # encodeTgx computes the same bits in the reference (GemvBench.swift:78);
    # here both names launch the same kernel.
    encodeTgx = encode
    encode_tgx = encode


class DequantInt8GEMV:
    """MLX-affine int8 matrix-vector product."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, weights, scales, biases, x, y, m: int, n: int, stream=None) -> None:
        _check_cuda(weights, scales, biases, x, y)
        st = lib().tf_int8_gemv(self.ctx.handle, ptr(weights), ptr(scales), ptr(biases), ptr(x), ptr(y),
                                m, n, scale_type_of(scales), stream_ptr(stream))
        self.ctx.check(st, "DequantInt8GEMV.encode")


def affine_gemv_batched(weights, scales, biases, x, y, *, bits: int, m: int, n: int, batch: int = 1,
                        w_stride_bytes: int = 0, sb_stride: int = 0, ntok: int = 1, x_row_stride: int | None = None,
                        y_row_stride: int | None = None, y_batch_stride: int = 0, stream=None,
                        context: Context | None = None) -> None:
    """`batch` matrices x `ntok` (<= 8) tokens in one launch (tf_affine_gemv_batched)."""
    ctx = context or Context.get(torch.cuda.current_device())
    _check_cuda(weights, scales, biases, x, y)
    st = lib().tf_affine_gemv_batched(
        ctx.handle, bits, ptr(weights), ptr(scales), ptr(biases), w_stride_bytes, sb_stride, batch, ptr(x), ntok,
        x_row_stride if x_row_stride is not None else n, ptr(y),
        y_row_stride if y_row_stride is not None else m, y_batch_stride, m, n, scale_type_of(scales),
        stream_ptr(stream))
    ctx.check(st, "affine_gemv_batched")
