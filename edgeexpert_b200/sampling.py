"""Output-head sampling, mirroring the reference's LogitSoftcapSoftmax,
Sample and SampleTopK64 encoders (Kernels/Sampling/LogitOutput.swift;
Metal/Sampling/logit.metal:42-617) on libtfcuda.so."""
from __future__ import annotations

import torch

from ._lib import Context, lib, ptr, stream_ptr


class LogitSoftcapSoftmax:
    """probs = softmax(softcap * tanh(logits / softcap)), fp16 out (Gemma 4: softcap 30)."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, logits, probs, v: int, softcap: float = 30.0, rows: int = 1, stream=None):
        fp32 = 1 if logits.dtype == torch.float32 else 0
        st = lib().tf_softcap_softmax(self.ctx.handle, ptr(logits), fp32, ptr(probs), v, rows, softcap,
                                      stream_ptr(stream))
        self.ctx.check(st, "LogitSoftcapSoftmax.encode")


class Sample:
    """Greedy / temperature / top-k / top-p sampler on fp16 probabilities."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, probs, out_token, v: int, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
               seed: int = 0, position: int = 0, stream=None):
        st = lib().tf_sample(self.ctx.handle, ptr(probs), v, temperature, top_k, top_p, seed & 0xFFFFFFFFFFFFFFFF,
                             position, ptr(out_token), stream_ptr(stream))
        self.ctx.check(st, "Sample.encode")


class SampleTopK64:
    """The three-stage top-64 sampler."""

    def __init__(self, context: Context | None = None):
        self.ctx = context or Context.get(torch.cuda.current_device())

    def encode(self, probs, out_token, v: int, temperature: float = 1.0, top_p: float = 1.0, seed: int = 0,
               stream=None):
        st = lib().tf_sample_topk64(self.ctx.handle, ptr(probs), v, temperature, top_p, seed & 0xFFFFFFFFFFFFFFFF,
                                    ptr(out_token), stream_ptr(stream))
        self.ctx.check(st, "SampleTopK64.encode")
