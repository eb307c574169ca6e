"""ctypes binding of ``libtfcuda.so`` (the C ABI in ``include/tfcuda.h``).

The library is the only compute path: there is no CPU or PyTorch fallback.
If the shared object is missing or cannot be loaded, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parent
import os

# TFCUDA_LIB selects another build of the same library (e.g. a debug build).
LIB_PATH = Path(os.environ.get("TFCUDA_LIB", str(_PKG / "libtfcuda.so")))

# tf_status codes (tfcuda.h)
TF_OK = 0
TF_ERR_INVALID_ARG = 1
TF_ERR_MISALIGNED = 2
TF_ERR_UNSUPPORTED_SHAPE = 3
TF_ERR_CUDA = 4
TF_ERR_NCCL = 5
TF_ERR_TIMEOUT = 6
TF_ERR_NO_DEVICE = 7
TF_ERR_GROUPING = 8

TF_SCALE_BF16 = 0
TF_SCALE_F16 = 1


class TFError(RuntimeError):
    """A non-zero tf_status returned by the C ABI."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[tf_status {status}] {message}")
        self.status = status
        self.message = message


class ExpertOffsets(C.Structure):
    """tf_expert_offsets == MoEExpertOffsets (MoE.swift:4-29)."""

    _fields_ = [(n, C.c_uint32) for n in (
        "gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b", "down_w", "down_s", "down_b")]


class AffineMatrix(C.Structure):
    """tf_affine_matrix == SharedExpertProjection (SharedExpertInt8.swift:9-31)."""

    _fields_ = [("weights", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p),
                ("rows", C.c_uint32), ("cols", C.c_uint32), ("bits", C.c_uint32)]


class TokenExpertPair(C.Structure):
    """tf_token_expert_pair == PrefillTokenExpertPair (PrefillRouter.swift:4-28)."""

    _fields_ = [("token", C.c_uint32), ("expert", C.c_uint32), ("rank", C.c_uint32), ("weight_bits", C.c_uint32)]


class MoEGroup(C.Structure):
    _fields_ = [("expert", C.c_uint32), ("pair_start", C.c_uint32), ("pair_count", C.c_uint32)]


class MoETile(C.Structure):
    _fields_ = [("group_start", C.c_uint32), ("group_count", C.c_uint32), ("pair_start", C.c_uint32),
                ("pair_count", C.c_uint32)]


class GroupingError(C.Structure):
    _fields_ = [("code", C.c_int), ("a", C.c_uint32), ("b", C.c_uint32)]


class MoELayer(C.Structure):
    """tf_moe_layer."""

    _fields_ = [
        ("router_w", C.c_void_p), ("router_s", C.c_void_p), ("router_b", C.c_void_p),
        ("eff_scale", C.c_void_p), ("per_expert_scale", C.c_void_p),
        ("expert_pool", C.c_void_p), ("expert_stride", C.c_uint64), ("num_experts", C.c_uint32),
        ("offsets", ExpertOffsets),
        ("shared_gate", AffineMatrix), ("shared_up", AffineMatrix), ("shared_down", AffineMatrix),
        ("d", C.c_uint32), ("f", C.c_uint32), ("top_k", C.c_uint32), ("scale_type", C.c_int),
    ]


_P = C.c_void_p
_U32 = C.c_uint32
_U64 = C.c_uint64
_I = C.c_int

# name -> argtypes (restype is tf_status = int unless noted)
_PROTOS = {
    "tf_status_string": ([_I], C.c_char_p),
    "tf_version": ([C.POINTER(_I), C.POINTER(_I)], None),
    "tf_context_create": ([_I, C.POINTER(_P)], _I),
    "tf_context_destroy": ([_P], None),
    "tf_context_last_error": ([_P], C.c_char_p),
    "tf_context_check_device": ([_P, _P, C.POINTER(_U32)], _I),
    "tf_int4_gemv": ([_P, _P, _P, _P, _P, _P, _U32, _U32, _I, _P], _I),
    "tf_int8_gemv": ([_P, _P, _P, _P, _P, _P, _U32, _U32, _I, _P], _I),
    "tf_affine_gemv_batched": ([_P, _U32, _P, _P, _P, _U64, _U64, _U32, _P, _U32, _U32, _P, _U32, _U64,
                                _U32, _U32, _I, _P], _I),
    "tf_router_topk": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _I, _P], _I),
    "tf_moe_phase1": ([_P, _P, _U64, _U32, _P, C.POINTER(_P), C.POINTER(ExpertOffsets), _P, _P, _U32, _U32,
                       _U32, _I, _P], _I),
    "tf_moe_phase2": ([_P, _P, _U64, _U32, _P, C.POINTER(_P), C.POINTER(ExpertOffsets), _P, _P, _P, _P, _U32,
                       _U32, _U32, _I, _P], _I),
    "tf_moe_phase1_bits": ([_P, _U32, _P, _U64, _U32, _P, C.POINTER(_P), C.POINTER(ExpertOffsets), _P, _P, _U32,
                            _U32, _U32, _I, _P], _I),
    "tf_moe_phase2_bits": ([_P, _U32, _P, _U64, _U32, _P, C.POINTER(_P), C.POINTER(ExpertOffsets), _P, _P, _P, _P,
                            _U32, _U32, _U32, _I, _P], _I),
    "tf_shared_expert": ([_P, _P, C.POINTER(AffineMatrix), C.POINTER(AffineMatrix), C.POINTER(AffineMatrix),
                          _P, _P, _I, _P], _I),
    "tf_moe_decode_layer": ([_P, C.POINTER(MoELayer), _P, _P, _P, _P, _P, _P, _P], _I),
    "tf_router_topk_noalloc": ([_P, _P, _P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _I, _P], _I),
    "tf_router_topk_noalloc_check": ([_P, C.POINTER(_U32)], _I),
    "tf_router_topk_with_logits": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _I, _P], _I),
    "tf_router_topk_batched_with_logits": ([_P, _P, _P, _P, _P, _U32, _P, _P, _P, _P, _P, _U32, _U32, _U32, _U32,
                                            _I, _P], _I),
    "tf_group_token_expert_pairs": ([_P, _U32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P, _U32, _P, _P, _P,
                                     _P, _P, _P, _P, C.POINTER(GroupingError)], _I),
    "tf_router_topk_batched": ([_P, _P, _P, _P, _P, _U32, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _I, _P], _I),
    "tf_moe_route_sort": ([_P, _P, _P, _U32, _U32, _U32, _U32, _P, _P, _P, _P, _P, _P, _P, _P, _P], _I),
    "tf_int4_qmm": ([_P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _I, _P], _I),
    "tf_prefill_shared_expert": ([_P, _P, _U32, C.POINTER(AffineMatrix), C.POINTER(AffineMatrix),
                                  C.POINTER(AffineMatrix), _P, _P, _U32, _U32, _I, _P], _I),
    "tf_moe_grouped_routed": ([_P, _P, _U64, _U32, C.POINTER(ExpertOffsets), _P, _P, _P, _P, _U32, _P, _P, _U32,
                               _U32, _U32, _U32, _I, _P], _I),
    "tf_moe_grouped_routed_expected": ([_P, _P, _U64, _U32, C.POINTER(ExpertOffsets), _P, _P, _P, _P, _U32, _P, _P,
                                        _U32, _U32, _U32, _U32, _U32, _I, _P], _I),
    "tf_moe_reduce_token_major": ([_P, _P, _P, _P, _U32, _U32, _U32, _P], _I),
    "tf_rmsnorm": ([_P, _P, _U32, _P, _P, _U32, _U32, _U32, C.c_float, _P], _I),
    "tf_qkv_epilogue": ([_P, _P, _U32, _P, _P, _U64, _P, _P, _U32, _U32, _U32, _U32, _U32, C.c_float, _U32,
                         C.c_float, _P], _I),
    "tf_attention_workspace_bytes": ([_P, _U32, _U32, _U32, _U32, _U32], C.c_size_t),
    "tf_attention_decode": ([_P, _P, _U32, _P, _P, _U64, _P, _U32, _U32, _U32, _U32, _U32, _U32, _U32,
                             C.c_float, _P, C.c_size_t, _P], _I),
    "tf_post_attn_setup": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _U32, _U32, C.c_float, _P], _I),
    "tf_layer_tail": ([_P, _P, _P, _P, _P, _P, _P, C.c_float, _U32, _U32, C.c_float, _P], _I),
    "tf_embed_int4": ([_P, _P, _P, _P, _P, _U32, _U32, _U32, C.c_float, _P, _U32, _I, _P], _I),
    "tf_lm_head_greedy": ([_P, _P, _U32, _P, C.c_float, _P, _P, _P, _U32, _U32, _U32, _P, _P, _P, _I, _P], _I),
    "tf_softcap_softmax": ([_P, _P, _I, _P, _U32, _U32, C.c_float, _P], _I),
    "tf_sample": ([_P, _P, _U32, C.c_float, _U32, C.c_float, _U64, _U32, _P, _P], _I),
    "tf_sample_topk64": ([_P, _P, _U32, C.c_float, C.c_float, _U64, _P, _P], _I),
    "tf_ep_flag_bytes": ([_U32], C.c_size_t),
    "tf_ep_ipc_alloc": ([_P, C.c_size_t, C.POINTER(_P), _P], _I),
    "tf_ep_ipc_open": ([_P, _P, C.POINTER(_P)], _I),
    "tf_ep_ipc_close": ([_P, _P], _I),
    "tf_ep_ipc_free": ([_P, _P], _I),
    "tf_ep_dispatch_p2p": ([_P, _P, _U32, _P, _P, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P],
                           _I),
    "tf_ep_dispatch_unpack_p2p": ([_P, _P, _P, _U32, _U32, _U32, _U32, _P, _P, _P], _I),
    "tf_ep_combine_p2p": ([_P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P], _I),
    "tf_ep_return_reduce_p2p": ([_P, _P, _P, _U32, _U32, _U32, _U32, _P, _U32, _P], _I),
    "tf_ep_dispatch_pack": ([_P, _P, _U32, _P, _P, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _P, _P], _I),
    "tf_ep_dispatch_unpack": ([_P, _P, _U32, _U32, _U32, _P, _P, _P], _I),
    "tf_ep_expert_combine": ([_P, _P, _P, _P, _U32, _U32, _U32, _P, _P], _I),
    "tf_ep_return_reduce": ([_P, _P, _U32, _U32, _U32, _U32, _P, _U32, _P], _I),
}

# Symbols of include/tfcuda.h added by later milestones register here too.
EXTRA_PROTOS: dict = {}

_lock = threading.Lock()
_lib = None


def _bind(lib, protos):
    for name, (args, res) in protos.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res


def lib():
    """Load (once) and return the ctypes handle.  Raises if the build is missing."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m edgeexpert_b200.build` "
                    "(there is no CPU fallback)")
            handle = C.CDLL(str(LIB_PATH))
            _bind(handle, _PROTOS)
            _bind(handle, EXTRA_PROTOS)
            _lib = handle
        return _lib


def exported_symbols() -> list[str]:
    return sorted(list(_PROTOS) + list(EXTRA_PROTOS))


def status_string(status: int) -> str:
    return lib().tf_status_string(status).decode()


class Context:
    """One tf_context per CUDA device (replaces MetalContext)."""

    _cache: dict = {}

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        st = lib().tf_context_create(device, C.byref(h))
        if st != TF_OK:
            raise TFError(st, f"tf_context_create(device={device}): {status_string(st)}")
        self.handle = h
        self.device = device

    @classmethod
    def get(cls, device: int = 0) -> "Context":
        ctx = cls._cache.get(device)
        if ctx is None:
            ctx = cls(device)
            cls._cache[device] = ctx
        return ctx

    def last_error(self) -> str:
        return lib().tf_context_last_error(self.handle).decode()

    def check(self, status: int, what: str = "") -> None:
        if status != TF_OK:
            raise TFError(status, f"{what}: {self.last_error()}")

    def check_device(self, stream=None) -> int:
        flags = C.c_uint32(0)
        st = lib().tf_context_check_device(self.handle, _stream_ptr(stream), C.byref(flags))
        self.check(st, "tf_context_check_device")
        return flags.value

    def __del__(self):  # contexts live for the process; destroy only if created standalone
        pass


def _stream_ptr(stream):
    if stream is None:
        import torch
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return C.c_void_p(stream)
    return C.c_void_p(stream.cuda_stream)


def ptr(t) -> C.c_void_p:
    """Device pointer of a torch tensor (or None -> NULL)."""
    if t is None:
        return C.c_void_p(0)
    if isinstance(t, int):
        return C.c_void_p(t)
    return C.c_void_p(t.data_ptr())


stream_ptr = _stream_ptr
