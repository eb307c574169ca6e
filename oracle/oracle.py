"""numpy/ctypes front end of the C oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py as the checker.  The product path
(edgeexpert_b200/) never imports this module.

All fp16/bf16 arrays are np.uint16 bit patterns.  scale_type 0 = BF16, 1 = fp16.
"""
from __future__ import annotations

import ctypes as C
import subprocess
import threading
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_lock = threading.Lock()
_lib = None

u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
VP = C.c_void_p
I = C.c_int


class Pair(C.Structure):
    _fields_ = [("token", C.c_uint32), ("expert", C.c_uint32), ("rank", C.c_uint32), ("weight_bits", C.c_uint32)]


class Group(C.Structure):
    _fields_ = [("expert", C.c_uint32), ("pair_start", C.c_uint32), ("pair_count", C.c_uint32)]


class Tile(C.Structure):
    _fields_ = [("group_start", C.c_uint32), ("group_count", C.c_uint32), ("pair_start", C.c_uint32),
                ("pair_count", C.c_uint32)]


class Offsets(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b", "down_w", "down_s", "down_b")]


PAIR_DTYPE = np.dtype([("token", "<u4"), ("expert", "<u4"), ("rank", "<u4"), ("weight_bits", "<u4")])


def build() -> Path:
    """Compile the oracle (make in oracle/) if the shared object is stale."""
    srcs = [HERE / n for n in ("oracle_core.c", "oracle_moe.c", "oracle.h", "Makefile")]
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < max(s.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                build()
            L = C.CDLL(str(LIB_PATH))
            sig = {
                "orc_sm64_next": ([C.POINTER(C.c_uint64)], C.c_uint64),
                "orc_sm64_uniform": ([C.POINTER(C.c_uint64), C.c_float, C.c_float], C.c_float),
                "orc_sm64_normal": ([C.POINTER(C.c_uint64)], C.c_double),
                "orc_seedtree_seed": ([C.c_uint64, C.c_char_p], C.c_uint64),
                "orc_fill_uniform": ([C.POINTER(C.c_uint64), C.c_float, C.c_float, f32p, C.c_size_t], None),
                "orc_fill_synthetic_affine": ([C.POINTER(C.c_uint64), I, I, I, I, u8p, u16p, u16p], None),
                "orc_fill_normal_f16": ([C.POINTER(C.c_uint64), C.c_float, u16p, C.c_size_t], None),
                "orc_bf16_bits": ([C.c_float], C.c_uint16),
                "orc_bf16_to_float": ([C.c_uint16], C.c_float),
                "orc_f16_bits": ([C.c_float], C.c_uint16),
                "orc_f16_to_float": ([C.c_uint16], C.c_float),
                "orc_f32_to_f16_array": ([f32p, u16p, C.c_size_t], None),
                "orc_f16_to_f32_array": ([u16p, f32p, C.c_size_t], None),
                "orc_packed_row_bytes": ([I, I], C.c_size_t),
                "orc_unpack_code": ([u8p, C.c_size_t, I, I], I),
                "orc_quantize_affine": ([f32p, I, I, I, u8p, u16p, u16p], I),
                "orc_dequantize_affine": ([u8p, u16p, u16p, I, I, I, I, f32p], None),
                "orc_affine_gemv_ref": ([u8p, u16p, u16p, I, I, f32p, f32p, I, I, I], None),
                "orc_int4_gemv_kernel_order": ([u8p, u16p, u16p, I, u16p, f32p, u16p, I, I, I], None),
                "orc_int8_gemv_kernel_order": ([u8p, u16p, u16p, I, u16p, f32p, u16p, I, I], None),
                "orc_router_logits": ([u8p, u16p, u16p, I, u16p, u16p, I, f32p, f64p, I, I], None),
                "orc_router_topk": ([f32p, I, u16p, I, I, u32p, u16p, f32p], None),
                "orc_gelu_tanh": ([C.c_float], C.c_float),
                "orc_moe_phase1": ([C.POINTER(VP), C.POINTER(Offsets), I, u16p, u16p, I, I, I, I], None),
                "orc_moe_phase2": ([C.POINTER(VP), C.POINTER(Offsets), I, u16p, u16p, VP, u16p, f32p, I, I, I, I],
                                   None),
                "orc_lowbit_gemv_kernel_order": ([u8p, u16p, u16p, I, I, u16p, f32p, u16p, I, I, I], None),
                "orc_moe_phase1_bits": ([C.POINTER(VP), C.POINTER(Offsets), I, I, u16p, u16p, I, I, I, I], None),
                "orc_moe_phase2_bits": ([C.POINTER(VP), C.POINTER(Offsets), I, I, u16p, u16p, VP, u16p, f32p, I, I,
                                         I, I], None),
                "orc_shared_expert": ([u8p, u16p, u16p, u8p, u16p, u16p, u8p, u16p, u16p, I, I, u16p, u16p, u16p,
                                       f32p, I, I, I], None),
                "orc_group_pairs": ([VP, I, I, I, I, I, VP, I, VP, u32p, u32p, VP, C.POINTER(I), VP, C.POINTER(I),
                                     C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)], I),
                "orc_reduce_token_major": ([u16p, u16p, u16p, I, I, I], None),
                "orc_grouped_routed": ([u8p, C.c_uint64, C.POINTER(Offsets), I, VP, I, u16p, I, u16p, I, I, I, I],
                                       None),
                "orc_int4_qmm": ([u8p, u16p, u16p, I, u16p, u16p, f32p, I, I, I, I], None),
                "orc_rel_error": ([f32p, f32p, C.c_size_t], C.c_float),
                "orc_max_threads": ([], I),
                "orc_rmsnorm": ([u16p, VP, u16p, I, I, C.c_float], None),
                "orc_qkv_epilogue": ([u16p, u16p, u16p, u16p, u16p, I, I, I, I, C.c_float, I, C.c_float], None),
                "orc_attention_decode": ([u16p, u16p, u16p, VP, VP, I, I, I, I, I, C.c_float], None),
                "orc_post_attn_setup": ([u16p, u16p, u16p, u16p, u16p, u16p, u16p, u16p, I, I, C.c_float], None),
                "orc_layer_tail": ([u16p, u16p, u16p, VP, u16p, u16p, C.c_float, I, I, C.c_float], None),
                "orc_embed_int4": ([u8p, u16p, u16p, I, u32p, I, I, C.c_float, u16p], None),
                "orc_lm_head_greedy": ([u8p, u16p, u16p, I, u16p, I, I, VP, I], C.c_uint32),
                "orc_softcap_softmax": ([f32p, u16p, I, C.c_float], None),
                "orc_gumbel": ([C.c_uint64, C.c_uint32, C.c_uint32], C.c_float),
                "orc_sample": ([u16p, I, C.c_float, C.c_uint32, C.c_float, C.c_uint64, C.c_uint32], C.c_uint32),
                "orc_sample_topk64": ([u16p, I, C.c_float, C.c_float, C.c_uint64], C.c_uint32),
            }
            for name, (args, res) in sig.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = res
            _lib = L
        return _lib


# ---------------------------------------------------------------- PRNG ------
class Rng:
    """SplitMix64 stream (SplitMix64.swift:11-23)."""

    def __init__(self, seed: int):
        self.state = C.c_uint64(seed & 0xFFFFFFFFFFFFFFFF)

    def next(self) -> int:
        return lib().orc_sm64_next(C.byref(self.state))

    def uniform(self, lo: float, hi: float, n: int | None = None):
        if n is None:
            return lib().orc_sm64_uniform(C.byref(self.state), lo, hi)
        out = np.empty(n, np.float32)
        lib().orc_fill_uniform(C.byref(self.state), lo, hi, out, n)
        return out

    def normal_f16(self, n: int, sigma: float = 1.0) -> np.ndarray:
        out = np.empty(n, np.uint16)
        lib().orc_fill_normal_f16(C.byref(self.state), sigma, out, n)
        return out

    def synthetic_affine(self, rows: int, cols: int, bits: int = 4, scale_type: int = 0):
        rb = packed_row_bytes(cols, bits)
        W = np.empty((rows, rb), np.uint8)
        S = np.empty((rows, cols // 64), np.uint16)
        B = np.empty((rows, cols // 64), np.uint16)
        lib().orc_fill_synthetic_affine(C.byref(self.state), rows, cols, bits, scale_type, W, S, B)
        return W, S, B


def seed_tree(root: int, label: str) -> Rng:
    """SeedTree(root).key(label) (SeedTree.swift:12-19)."""
    return Rng(lib().orc_seedtree_seed(root & 0xFFFFFFFFFFFFFFFF, label.encode()))


# ---------------------------------------------------------------- formats ---
def f16_to_f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.uint16).view(np.float16).astype(np.float32)


def f32_to_f16(a) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().orc_f32_to_f16_array(a.reshape(-1), out.reshape(-1), a.size)
    return out


def bf16_bits(a) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    return np.array([lib().orc_bf16_bits(float(v)) for v in a.reshape(-1)], np.uint16).reshape(a.shape)


def scale_to_f32(bits, scale_type: int) -> np.ndarray:
    b = np.ascontiguousarray(bits, np.uint16)
    if scale_type == 1:
        return b.view(np.float16).astype(np.float32)
    return (b.astype(np.uint32) << 16).view(np.float32)


def packed_row_bytes(n: int, bits: int) -> int:
    return int(lib().orc_packed_row_bytes(n, bits))


def quantize_affine(w: np.ndarray, bits: int):
    w = np.ascontiguousarray(w, np.float32)
    rows, n = w.shape
    W = np.empty((rows, packed_row_bytes(n, bits)), np.uint8)
    S = np.empty((rows, n // 64), np.uint16)
    B = np.empty((rows, n // 64), np.uint16)
    rc = lib().orc_quantize_affine(w, rows, n, bits, W, S, B)
    if rc != 0:
        raise ValueError(f"quantize_affine: rc={rc}")
    return W, S, B


def dequantize_affine(W, S, B, n: int, bits: int, scale_type: int = 0) -> np.ndarray:
    rows = W.shape[0]
    out = np.empty((rows, n), np.float32)
    lib().orc_dequantize_affine(np.ascontiguousarray(W), np.ascontiguousarray(S), np.ascontiguousarray(B),
                                scale_type, rows, n, bits, out)
    return out


def unpack_code(buf: np.ndarray, index: int, bits: int) -> int:
    b = np.ascontiguousarray(buf, np.uint8)
    return lib().orc_unpack_code(b, b.size, index, bits)


# ---------------------------------------------------------------- GEMVs -----
def _nt(nthreads):
    return nthreads if nthreads else lib().orc_max_threads()


def affine_gemv_ref(W, S, B, x_f32, bits: int, scale_type: int = 0, nthreads: int = 0) -> np.ndarray:
    m = W.shape[0]
    n = x_f32.shape[0]
    y = np.empty(m, np.float32)
    lib().orc_affine_gemv_ref(np.ascontiguousarray(W), np.ascontiguousarray(S), np.ascontiguousarray(B), scale_type,
                              bits, np.ascontiguousarray(x_f32, np.float32), y, m, n, _nt(nthreads))
    return y


def int4_gemv_kernel_order(W, S, B, x_f16, scale_type: int = 0, nthreads: int = 0):
    m = W.shape[0]
    n = x_f16.shape[0]
    y32 = np.empty(m, np.float32)
    y16 = np.empty(m, np.uint16)
    lib().orc_int4_gemv_kernel_order(np.ascontiguousarray(W), np.ascontiguousarray(S), np.ascontiguousarray(B),
                                     scale_type, np.ascontiguousarray(x_f16, np.uint16), y32, y16, m, n,
                                     _nt(nthreads))
    return y32, y16


def int8_gemv_kernel_order(W, S, B, x_f16, scale_type: int = 0):
    m = W.shape[0]
    n = x_f16.shape[0]
    y32 = np.empty(m, np.float32)
    y16 = np.empty(m, np.uint16)
    lib().orc_int8_gemv_kernel_order(np.ascontiguousarray(W), np.ascontiguousarray(S), np.ascontiguousarray(B),
                                     scale_type, np.ascontiguousarray(x_f16, np.uint16), y32, y16, m, n)
    return y32, y16


# ---------------------------------------------------------------- router ----
def router_logits(W8, S, B, hidden_f16, eff_scale_bf16, scale_type: int = 0, es_type: int = 0):
    E, D = W8.shape
    l32 = np.empty(E, np.float32)
    l64 = np.empty(E, np.float64)
    lib().orc_router_logits(np.ascontiguousarray(W8), np.ascontiguousarray(S), np.ascontiguousarray(B), scale_type,
                            np.ascontiguousarray(hidden_f16, np.uint16),
                            np.ascontiguousarray(eff_scale_bf16, np.uint16), es_type, l32, l64, E, D)
    return l32, l64


def router_topk(logits, pes_bits, k: int, pes_type: int = 0):
    logits = np.ascontiguousarray(logits, np.float32)
    idx = np.empty(k, np.uint32)
    w16 = np.empty(k, np.uint16)
    w32 = np.empty(k, np.float32)
    lib().orc_router_topk(logits, logits.size, np.ascontiguousarray(pes_bits, np.uint16), pes_type, k, idx, w16, w32)
    return idx, w16, w32


def gelu(x: float) -> float:
    return lib().orc_gelu_tanh(x)


# ---------------------------------------------------------------- decode MoE
def _blob_ptrs(blobs):
    arr = (VP * len(blobs))(*[b.ctypes.data for b in blobs])
    return arr


def moe_phase1(blobs, off: Offsets, x_f16, D: int, F: int, scale_type: int = 0, nthreads: int = 0):
    k = len(blobs)
    acts = np.empty(k * F, np.uint16)
    lib().orc_moe_phase1(_blob_ptrs(blobs), C.byref(off), scale_type, np.ascontiguousarray(x_f16, np.uint16), acts,
                         D, F, k, _nt(nthreads))
    return acts


def moe_phase2(blobs, off: Offsets, acts_f16, w_f16, residual_f16, D: int, F: int, scale_type: int = 0,
               nthreads: int = 0):
    k = len(blobs)
    y16 = np.empty(D, np.uint16)
    y32 = np.empty(D, np.float32)
    res = None if residual_f16 is None else np.ascontiguousarray(residual_f16, np.uint16)
    lib().orc_moe_phase2(_blob_ptrs(blobs), C.byref(off), scale_type, np.ascontiguousarray(acts_f16, np.uint16),
                         np.ascontiguousarray(w_f16, np.uint16), None if res is None else res.ctypes.data, y16, y32,
                         D, F, k, _nt(nthreads))
    return y16, y32


def lowbit_gemv_kernel_order(W, S, B, x_f16, bits: int, scale_type: int = 0, nthreads: int = 0):
    """moe_int2/int3 row order (moe.metal:644-757): (fp32 [m], fp16 bits [m])."""
    m = W.shape[0]
    n = S.shape[1] * 64
    y32 = np.empty(m, np.float32)
    y16 = np.empty(m, np.uint16)
    lib().orc_lowbit_gemv_kernel_order(np.ascontiguousarray(W), np.ascontiguousarray(S), np.ascontiguousarray(B),
                                       scale_type, bits, np.ascontiguousarray(x_f16, np.uint16), y32, y16, m, n,
                                       _nt(nthreads))
    return y32, y16


def moe_phase1_bits(blobs, off: Offsets, x_f16, D: int, F: int, bits: int, scale_type: int = 0, nthreads: int = 0):
    k = len(blobs)
    acts = np.empty(k * F, np.uint16)
    lib().orc_moe_phase1_bits(_blob_ptrs(blobs), C.byref(off), scale_type, bits,
                              np.ascontiguousarray(x_f16, np.uint16), acts, D, F, k, _nt(nthreads))
    return acts


def moe_phase2_bits(blobs, off: Offsets, acts_f16, w_f16, residual_f16, D: int, F: int, bits: int,
                    scale_type: int = 0, nthreads: int = 0):
    k = len(blobs)
    y16 = np.empty(D, np.uint16)
    y32 = np.empty(D, np.float32)
    res = None if residual_f16 is None else np.ascontiguousarray(residual_f16, np.uint16)
    lib().orc_moe_phase2_bits(_blob_ptrs(blobs), C.byref(off), scale_type, bits,
                              np.ascontiguousarray(acts_f16, np.uint16), np.ascontiguousarray(w_f16, np.uint16),
                              None if res is None else res.ctypes.data, y16, y32, D, F, k, _nt(nthreads))
    return y16, y32


def shared_expert(gate, up, down, x_f16, D: int, Fs: int, bits: int, scale_type: int = 0, nthreads: int = 0):
    act = np.empty(Fs, np.uint16)
    y16 = np.empty(D, np.uint16)
    y32 = np.empty(D, np.float32)
    c = np.ascontiguousarray
    lib().orc_shared_expert(c(gate[0]), c(gate[1]), c(gate[2]), c(up[0]), c(up[1]), c(up[2]), c(down[0]), c(down[1]),
                            c(down[2]), scale_type, bits, c(x_f16, np.uint16), act, y16, y32, D, Fs, _nt(nthreads))
    return act, y16, y32


# ---------------------------------------------------------------- grouping --
GROUP_ERRORS = {
    0: "ok", 1: "invalidQueryCount", 2: "invalidTopK", 3: "invalidNumExperts", 4: "invalidTileExpertCount",
    5: "pairCountMismatch", 6: "tokenOutOfRange", 7: "rankOutOfRange", 8: "expertOutOfRange",
    9: "duplicateTokenRank", 10: "expertSortKeyCountMismatch",
}


class GroupingError(ValueError):
    def __init__(self, code, a, b):
        super().__init__(f"{GROUP_ERRORS.get(code, code)} ({a}, {b})")
        self.code, self.a, self.b = code, a, b


def group_pairs(pairs: np.ndarray, query_count: int, top_k: int, num_experts: int, tile_expert_count: int = 16,
                sort_keys=None):
    """PrefillMoEGrouping.groupTokenExpertPairs -> dict of numpy arrays (raises GroupingError)."""
    pairs = np.ascontiguousarray(pairs, PAIR_DTYPE)
    n = pairs.size
    sorted_ = np.empty(max(n, 1), PAIR_DTYPE)
    E = max(num_experts, 1)
    offsets = np.empty(E, np.uint32)
    counts = np.empty(E, np.uint32)
    groups = np.empty(E, np.dtype([("expert", "<u4"), ("pair_start", "<u4"), ("pair_count", "<u4")]))
    tiles = np.empty(E, np.dtype([("group_start", "<u4"), ("group_count", "<u4"), ("pair_start", "<u4"),
                                  ("pair_count", "<u4")]))
    ng, nt = C.c_int(0), C.c_int(0)
    ea, eb = C.c_uint32(0), C.c_uint32(0)
    keys = None if sort_keys is None else np.ascontiguousarray(sort_keys, np.uint64)
    rc = lib().orc_group_pairs(pairs.ctypes.data if n else None, n, query_count, top_k, num_experts,
                               tile_expert_count, None if keys is None else keys.ctypes.data,
                               0 if keys is None else keys.size, sorted_.ctypes.data, offsets, counts,
                               groups.ctypes.data, C.byref(ng), tiles.ctypes.data, C.byref(nt), C.byref(ea),
                               C.byref(eb))
    if rc != 0:
        raise GroupingError(rc, ea.value, eb.value)
    return {"sorted": sorted_[:n], "offsets": offsets[:num_experts], "counts": counts[:num_experts],
            "groups": groups[:ng.value], "tiles": tiles[:nt.value]}


def reduce_token_major(partials_f16, w_f16, T: int, K: int, D: int) -> np.ndarray:
    out = np.empty(T * D, np.uint16)
    lib().orc_reduce_token_major(np.ascontiguousarray(partials_f16, np.uint16), np.ascontiguousarray(w_f16, np.uint16),
                                 out, T, K, D)
    return out


def grouped_routed(pool: np.ndarray, stride: int, off: Offsets, sorted_pairs, hidden_f16, hidden_stride: int,
                   D: int, F: int, top_k: int, T: int, scale_type: int = 0, nthreads: int = 0) -> np.ndarray:
    sp = np.ascontiguousarray(sorted_pairs, PAIR_DTYPE)
    part = np.zeros(T * top_k * D, np.uint16)
    lib().orc_grouped_routed(np.ascontiguousarray(pool, np.uint8), stride, C.byref(off), scale_type, sp.ctypes.data,
                             sp.size, np.ascontiguousarray(hidden_f16, np.uint16), hidden_stride, part, D, F, top_k,
                             _nt(nthreads))
    return part


def int4_qmm(W, S, B, X_f16, T: int, N: int, K: int, scale_type: int = 0, nthreads: int = 0):
    y16 = np.empty(T * N, np.uint16)
    y32 = np.empty(T * N, np.float32)
    lib().orc_int4_qmm(np.ascontiguousarray(W), np.ascontiguousarray(S), np.ascontiguousarray(B), scale_type,
                       np.ascontiguousarray(X_f16, np.uint16), y16, y32, T, N, K, _nt(nthreads))
    return y16, y32


def rel_error(actual, ref) -> float:
    """RelError.compute (RelError.swift:7-16): max|a-r| / max(max|r|, 1e-6)."""
    a = np.ascontiguousarray(actual, np.float32).reshape(-1)
    r = np.ascontiguousarray(ref, np.float32).reshape(-1)
    return float(lib().orc_rel_error(a, r, a.size))


# ------------------------------------------------------- decode stack ------
def _vp(a):
    return None if a is None else np.ascontiguousarray(a).ctypes.data_as(C.c_void_p)


def rmsnorm(x_f16, w_bf16, rows: int, d: int, eps: float = 1e-6) -> np.ndarray:
    """rmsnorm_bf16w (w given) / rmsnorm_no_scale (w None), fp16 bits out."""
    out = np.empty(rows * d, np.uint16)
    w = None if w_bf16 is None else np.ascontiguousarray(w_bf16, np.uint16)
    lib().orc_rmsnorm(np.ascontiguousarray(x_f16, np.uint16).reshape(-1), _vp(w), out, rows, d, eps)
    return out


def qkv_epilogue(q, k, v, qw, kw, hd, nq, nkv, position, theta, rotated_pairs, eps=1e-6):
    q, k, v = (np.ascontiguousarray(a, np.uint16).reshape(-1).copy() for a in (q, k, v))
    lib().orc_qkv_epilogue(q, k, v, np.ascontiguousarray(qw, np.uint16), np.ascontiguousarray(kw, np.uint16), hd,
                           nq, nkv, position, theta, rotated_pairs, eps)
    return q, k, v


def attention_decode(q, K, V, hd, nq, nkv, seq_len, kv_start=0, scale=1.0):
    """Returns (fp16 bits, fp32) [nq*hd]."""
    o16 = np.empty(nq * hd, np.uint16)
    o32 = np.empty(nq * hd, np.float32)
    keep = [np.ascontiguousarray(a, np.uint16).reshape(-1) for a in (q, K, V)]
    lib().orc_attention_decode(*keep, _vp(o16), _vp(o32), hd, nq, nkv, seq_len, kv_start, scale)
    return o16, o32


def post_attn_setup(hidden, attn, w_post_attn, w_pre_ffn, w_pre_ffn2, rows, d, eps=1e-6):
    h = np.ascontiguousarray(hidden, np.uint16).reshape(-1).copy()
    dx, rx, rt = (np.empty(rows * d, np.uint16) for _ in range(3))
    lib().orc_post_attn_setup(h, np.ascontiguousarray(attn, np.uint16).reshape(-1), dx, rx, rt,
                              *[np.ascontiguousarray(w, np.uint16) for w in (w_post_attn, w_pre_ffn, w_pre_ffn2)],
                              rows, d, eps)
    return h, dx, rx, rt


def layer_tail(h2, h1, hidden, w_postffn1, w_postffn2, w_postffn, layer_scalar, rows, d, eps=1e-6):
    h = np.ascontiguousarray(hidden, np.uint16).reshape(-1).copy()
    w1 = None if w_postffn1 is None else np.ascontiguousarray(w_postffn1, np.uint16)
    lib().orc_layer_tail(np.ascontiguousarray(h2, np.uint16).reshape(-1), np.ascontiguousarray(h1, np.uint16).reshape(-1),
                         h, _vp(w1), np.ascontiguousarray(w_postffn2, np.uint16),
                         np.ascontiguousarray(w_postffn, np.uint16), layer_scalar, rows, d, eps)
    return h


def embed_int4(table, S, B, tokens, d, out_scale=1.0, scale_type=0):
    t = np.ascontiguousarray(tokens, np.uint32)
    out = np.empty(t.size * d, np.uint16)
    lib().orc_embed_int4(np.ascontiguousarray(table), np.ascontiguousarray(S), np.ascontiguousarray(B), scale_type, t,
                         t.size, d, out_scale, out)
    return out


def lm_head_greedy(W, S, B, x_f16, vocab, d, scale_type=0, nthreads=0, want_logits=False):
    logits = np.empty(vocab, np.float32) if want_logits else None
    tok = lib().orc_lm_head_greedy(np.ascontiguousarray(W), np.ascontiguousarray(S), np.ascontiguousarray(B),
                                   scale_type, np.ascontiguousarray(x_f16, np.uint16), vocab, d, _vp(logits),
                                   _nt(nthreads))
    return (int(tok), logits) if want_logits else int(tok)


# ------------------------------------------------------------- sampling ----
def softcap_softmax(logits_f32, softcap: float = 30.0) -> np.ndarray:
    lg = np.ascontiguousarray(logits_f32, np.float32).reshape(-1)
    out = np.empty(lg.size, np.uint16)
    lib().orc_softcap_softmax(lg, out, lg.size, softcap)
    return out


def sample(probs_f16, temperature: float, top_k: int = 0, top_p: float = 1.0, seed: int = 0, position: int = 0):
    p = np.ascontiguousarray(probs_f16, np.uint16).reshape(-1)
    return int(lib().orc_sample(p, p.size, temperature, top_k, top_p, seed & 0xFFFFFFFFFFFFFFFF, position))


def sample_topk64(probs_f16, temperature: float, top_p: float = 1.0, seed: int = 0):
    p = np.ascontiguousarray(probs_f16, np.uint16).reshape(-1)
    return int(lib().orc_sample_topk64(p, p.size, temperature, top_p, seed & 0xFFFFFFFFFFFFFFFF))
