"""ctypes bindings of librocknpu.so: the reference C ABI (include/rocknpu.h)
and the B200 additions (include/rocknpu_b200.h).

``Context`` mirrors the reference interface one method per entry point, with
the same names, argument meaning and status codes; numpy arrays stand for the
caller's host buffers.  Nothing here computes: every call goes to the CUDA
library, and loading fails loudly when the library has not been built.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librocknpu.so")

STATUS_OK = 0
STATUS_INVALID_ARGUMENT = -1
STATUS_DEVICE_ERROR = -2
STATUS_EXECUTION_ERROR = -3

Q4_K, Q5_K, Q6_K = 4, 5, 6
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}

# ggml type ids understood by rocknpu_mul_mat_supported
GGML_F32, GGML_F16, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 0, 1, 12, 13, 14

_P = ctypes.c_void_p
_S = ctypes.c_size_t
_I = ctypes.c_int
_U32 = ctypes.c_uint32

# (name, restype, argtypes) of every exported entry point.
SIGNATURES = {
    # rocknpu.h
    "rocknpu_device_count": (_S, []),
    "rocknpu_context_create": (_P, []),
    "rocknpu_context_decode_cache_stats": (_I, [_P, _P]),
    "rocknpu_context_destroy": (None, [_P]),
    "rocknpu_context_set_overlap": (_I, [_P, _P, _P]),
    "rocknpu_matmul_q_concat_f32_f32_mtile": (_I, [_P, _S, _P, _P, _P, _P, _P, _P, _S, _S]),
    "rocknpu_mtile_release": (_I, [_P, _S, _P]),
    "rocknpu_prewarm_quantized_m16": (_I, [_P, _P, _S, _U32, _S, _S]),
    "rocknpu_matmul_f16_f32_f32": (_I, [_P, _P, _P, _P, _S, _S, _S]),
    "rocknpu_matmul_w8a8_f32_f32_m1": (_I, [_P, _P, _P, _P, _P, _S, _S]),
    "rocknpu_matmul_w8a8_f32_f32_m16": (_I, [_P, _P, _P, _P, _P, _S, _S]),
    "rocknpu_matmul_w8a8_f32_f32_m1_nsplit": (_I, [_P, _P, _P, _P, _P, _S, _S, _S]),
    "rocknpu_matmul_w8a8_swiglu_down_f32": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _S, _S, _S]),
    "rocknpu_matmul_w8a8_pair_f32_f32_m1": (_I, [_P, _P, _P, _S, _P, _P, _S, _P, _P, _P, _S]),
    "rocknpu_matmul_q_pair_f32_f32_mtile": (_I, [_P, _P, _S, _U32, _S, _P, _S, _U32, _S, _P, _P, _P, _S, _S]),
    "rocknpu_matmul_w8a8_triple_f32_f32_m1": (_I, [_P, _P, _P, _S, _P, _P, _S, _P, _P, _S, _P, _P, _P, _P, _S]),
    "rocknpu_matmul_q_pair_f32_f32_m1": (_I, [_P, _P, _S, _U32, _S, _P, _S, _U32, _S, _P, _P, _P, _S]),
    "rocknpu_matmul_q_triple_f32_f32_m1": (_I, [_P, _P, _S, _U32, _S, _P, _S, _U32, _S, _P, _S, _U32, _S,
                                               _P, _P, _P, _P, _S]),
    "rocknpu_matmul_q4_k_f32_f32": (_I, [_P, _P, _S, _P, _P, _S, _S, _S]),
    "rocknpu_matmul_q5_k_f32_f32": (_I, [_P, _P, _S, _P, _P, _S, _S, _S]),
    "rocknpu_matmul_q6_k_f32_f32": (_I, [_P, _P, _S, _P, _P, _S, _S, _S]),
    # rocknpu_b200.h
    "rocknpu_apply_default_env": (None, []),
    "rocknpu_mul_mat_supported": (_I, [_P]),
    "rocknpu_graph_state_create": (_P, [ctypes.c_int32]),
    "rocknpu_graph_state_destroy": (None, [_P]),
    "rocknpu_graph_plan": (_I, [_P, _P, _S, _P, _S]),
    "rocknpu_b200_context_stream": (_P, [_P]),
    "rocknpu_b200_context_check": (_I, [_P]),
    "rocknpu_b200_status_code": (_I, [_I]),
    "rocknpu_b200_context_prompt_cache_stats": (_I, [_P, _P]),
    "rocknpu_b200_host_mapped": (_I, [_P, _S]),
    "rocknpu_b200_host_alloc": (_P, [_S]),
    "rocknpu_b200_host_free": (_I, [_P]),
    "rocknpu_b200_prepare_w8": (_I, [_U32, _P, _S, _S, _P, _P, _P, _P]),
    "rocknpu_b200_quantize_rows": (_I, [_P, _S, _S, _P, _S, _P, _P, _P]),
    "rocknpu_b200_gemm_workspace_bytes": (_S, [_S, _S, _S]),
    "rocknpu_b200_gemm_w8a8": (_I, [_P, _S, _P, _P, _S, _P, _P, _S, _P, _S, _S, _S, _P, _S, _P, _P]),
    "rocknpu_b200_matmul_w8a8": (_I, [_P, _P, _P, _P, _P, _S, _S, _S, _P]),
    "rocknpu_b200_matmul_w8a8_noalloc": (_I, [_P, _P, _P, _P, _S, _S, _S, _P, _P]),
    "rocknpu_b200_convert_f16": (_I, [_P, _S, _S, _S, _P, _S, _P]),
    "rocknpu_b200_gemm_f16": (_I, [_P, _S, _P, _S, _P, _S, _S, _S, _S, _P, _P]),
    "rocknpu_b200_gemv_w8a8": (_I, [_P, _P, _P, _P, _P, _S, _S, _P]),
    "rocknpu_b200_kq_layout_bytes": (_S, [_U32, _S, _S]),
    "rocknpu_b200_kq_layout": (_I, [_U32, _P, _S, _S, _P, _P]),
    "rocknpu_b200_gemv_kq": (_I, [_U32, _P, _S, _S, _P, _P, _P, _P]),
    "rocknpu_b200_shard_rows": (_S, [_S, _S, _P, _P]),
    "rocknpu_b200_gather_shards": (_I, [_P, _S, _S, _S, _S, _P, _P, _P, _S, _P]),
    "rocknpu_b200_peer_buffer_create": (_I, [_S, _I, _I, _P, _P]),
    "rocknpu_b200_peer_buffer_open": (_I, [_P, _P]),
    "rocknpu_b200_peer_buffer_ptr": (_P, [_P, _I]),
    "rocknpu_b200_peer_barrier": (_I, [_P, _P, _P]),
    "rocknpu_b200_set_peer_wait_limit_ms": (_I, [_U32]),
    "rocknpu_b200_peer_buffer_destroy": (None, [_P]),
    "rocknpu_b200_gemm_w8a8_gather": (_I, [_P, _S, _P, _P, _S, _P, _P, _S, _S, _S, _S, _S, _S, _P, _P]),
    "rocknpu_b200_source_fingerprint": (ctypes.c_uint64, [_P, _S]),
    "rocknpu_b200_w8_sidecar_read": (_I, [ctypes.c_char_p, ctypes.c_char_p, _P, _S, _S, _S, _P, _P]),
    "rocknpu_b200_w8_sidecar_write": (_I, [ctypes.c_char_p, ctypes.c_char_p, _P, _S, _S, _S, _P, _P]),
    "rocknpu_synth_normal": (None, [ctypes.c_uint64, ctypes.c_uint64, _S, ctypes.c_float, _P]),
    "rocknpu_synth_encode": (_I, [_U32, _P, _S, _S, _P]),
}

_lib = None


class CacheStats(ctypes.Structure):
    """rocknpu_decode_cache_stats."""
    _fields_ = [("hits", _S), ("misses", _S), ("entries", _S), ("resident_bytes", _S),
                ("hit_ns", ctypes.c_uint64), ("miss_ns", ctypes.c_uint64), ("tuned_shapes", _S),
                ("worker1_calls", _S), ("worker2_calls", _S), ("worker3_calls", _S), ("ksplit_calls", _S)]


class PromptCacheStats(ctypes.Structure):
    """rocknpu_b200_prompt_cache_stats."""
    _fields_ = [("single_entries", _S), ("group_entries", _S), ("hits", _S), ("misses", _S),
                ("resident_bytes", _S)]


class MulMatDesc(ctypes.Structure):
    """rocknpu_mul_mat_desc."""
    _fields_ = [("is_mul_mat", ctypes.c_int32), ("weight_type", ctypes.c_int32), ("act_type", ctypes.c_int32),
                ("dst_type", ctypes.c_int32), ("weight_ne", ctypes.c_int64 * 4), ("act_ne", ctypes.c_int64 * 4),
                ("weight_contiguous", ctypes.c_int32), ("act_contiguous", ctypes.c_int32),
                ("dst_contiguous", ctypes.c_int32)]


OVERLAP_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p)


def lib():
    """The loaded library; raises if it was never built (no silent fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m rocknpu_b200.build` (there is no CPU path)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ptr(a):
    """Address of a numpy array's data (or None)."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "buffers must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


class _HostBlock:
    """Owner of one rocknpu_b200_host_alloc buffer, released with the object;
    numpy views of it keep it alive through their ``base``."""

    def __init__(self, nbytes: int):
        p = lib().rocknpu_b200_host_alloc(nbytes)
        if not p:
            raise RuntimeError(f"rocknpu_b200_host_alloc({nbytes}) failed (no GPU, or the memory cannot be locked)")
        self.ptr = p
        self.__array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (p, False), "version": 3}

    def __del__(self):
        p, self.ptr = getattr(self, "ptr", None), None
        if p and _lib is not None:
            _lib.rocknpu_b200_host_free(p)


def host_empty(shape, dtype=np.float32) -> np.ndarray:
    """Uninitialised host array in rocknpu_b200_host_alloc memory (page-locked,
    huge-page backed): the buffer type for the host-pointer entry points'
    activations and outputs."""
    dtype = np.dtype(dtype)
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    nbytes = int(np.prod(shape, dtype=np.int64)) * dtype.itemsize
    raw = np.asarray(_HostBlock(max(nbytes, 1)))
    return raw[:nbytes].view(dtype).reshape(shape)


def device_count() -> int:
    return int(lib().rocknpu_device_count())


def apply_default_env() -> None:
    lib().rocknpu_apply_default_env()


def mul_mat_supported(weight_type: int, k: int, n: int, m: int, act_type: int = GGML_F32,
                      dst_type: int = GGML_F32, contiguous=(True, True, True), batch=(1, 1, 1, 1),
                      is_mul_mat: bool = True) -> bool:
    d = MulMatDesc()
    d.is_mul_mat = int(is_mul_mat)
    d.weight_type, d.act_type, d.dst_type = weight_type, act_type, dst_type
    d.weight_ne[:] = [k, n, batch[0], batch[1]]
    d.act_ne[:] = [k, m, batch[2], batch[3]]
    d.weight_contiguous, d.act_contiguous, d.dst_contiguous = (int(c) for c in contiguous)
    return bool(lib().rocknpu_mul_mat_supported(ctypes.byref(d)))


def synth_normal(seed: int, count: int, sigma: float = 1.0, first: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib().rocknpu_synth_normal(seed, first, count, sigma, ptr(out))
    return out


def synth_encode(kind: int, values: np.ndarray) -> np.ndarray:
    values = np.ascontiguousarray(values, dtype=np.float32)
    n, k = values.shape
    out = np.empty(n * (k // 256) * BLOCK_BYTES[kind], dtype=np.uint8)
    if lib().rocknpu_synth_encode(kind, ptr(values), k, n, ptr(out)) != 0:
        raise ValueError("bad shape for synth_encode")
    return out


def synth_q_weights(kind: int, n: int, k: int, seed: int, sigma: float = 0.02) -> np.ndarray:
    """N(0, sigma^2) [n, k] weights encoded as K-quant blocks."""
    return synth_encode(kind, synth_normal(seed, n * k, sigma).reshape(n, k))


class Context:
    """One rocknpu_context (one GPU): the reference C ABI, method per entry."""

    def __init__(self):
        self._lib = lib()
        self.handle = self._lib.rocknpu_context_create()
        if not self.handle:
            raise RuntimeError("rocknpu_context_create returned NULL (no sm_100 GPU)")
        self._keep = []

    def close(self):
        if self.handle:
            self._lib.rocknpu_context_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- statistics / callbacks ------------------------------------------
    def decode_cache_stats(self) -> CacheStats:
        s = CacheStats()
        st = self._lib.rocknpu_context_decode_cache_stats(self.handle, ctypes.byref(s))
        if st != 0:
            raise RuntimeError(f"decode_cache_stats status {st}")
        return s

    def prompt_cache_stats(self) -> PromptCacheStats:
        s = PromptCacheStats()
        st = self._lib.rocknpu_b200_context_prompt_cache_stats(self.handle, ctypes.byref(s))
        if st != 0:
            raise RuntimeError(f"prompt_cache_stats status {st}")
        return s

    def set_overlap(self, fn) -> int:
        cb = OVERLAP_FN(lambda _u: fn()) if fn is not None else None
        self._keep.append(cb)
        return self._lib.rocknpu_context_set_overlap(self.handle, cb, None)

    def stream(self) -> int:
        return self._lib.rocknpu_b200_context_stream(self.handle)

    # -- quantized weights -------------------------------------------------
    def matmul_q(self, kind: int, weights: np.ndarray, a: np.ndarray, out: np.ndarray, m: int, k: int, n: int,
                 weights_bytes: int | None = None) -> int:
        fn = {Q4_K: self._lib.rocknpu_matmul_q4_k_f32_f32, Q5_K: self._lib.rocknpu_matmul_q5_k_f32_f32,
              Q6_K: self._lib.rocknpu_matmul_q6_k_f32_f32}[kind]
        nbytes = weights.nbytes if weights_bytes is None else weights_bytes
        return fn(self.handle, ptr(weights), nbytes, ptr(a), ptr(out), m, k, n)

    def matmul_q_concat(self, weights, kinds, ns, a, outs, m, k, bytes_=None) -> int:
        count = len(weights)
        W = (ctypes.c_void_p * count)(*[w.ctypes.data for w in weights])
        B = (ctypes.c_size_t * count)(*[(w.nbytes if bytes_ is None else bytes_[i]) for i, w in enumerate(weights)])
        K = (ctypes.c_uint32 * count)(*kinds)
        N = (ctypes.c_size_t * count)(*ns)
        O = (ctypes.c_void_p * count)(*[o.ctypes.data for o in outs])
        return self._lib.rocknpu_matmul_q_concat_f32_f32_mtile(self.handle, count, W, B, K, N, ptr(a), O, m, k)

    def mtile_release(self, weights) -> int:
        W = (ctypes.c_void_p * len(weights))(*[w.ctypes.data for w in weights])
        return self._lib.rocknpu_mtile_release(self.handle, len(weights), W)

    def prewarm_quantized_m16(self, weights, kind, k, n) -> int:
        return self._lib.rocknpu_prewarm_quantized_m16(self.handle, ptr(weights), weights.nbytes, kind, k, n)

    def matmul_q_pair_mtile(self, w1, kind1, n1, w2, kind2, n2, a, o1, o2, m, k) -> int:
        return self._lib.rocknpu_matmul_q_pair_f32_f32_mtile(self.handle, ptr(w1), w1.nbytes, kind1, n1, ptr(w2),
                                                             w2.nbytes, kind2, n2, ptr(a), ptr(o1), ptr(o2), m, k)

    def matmul_q_pair_m1(self, w1, kind1, n1, w2, kind2, n2, a, o1, o2, k) -> int:
        return self._lib.rocknpu_matmul_q_pair_f32_f32_m1(self.handle, ptr(w1), w1.nbytes, kind1, n1, ptr(w2),
                                                          w2.nbytes, kind2, n2, ptr(a), ptr(o1), ptr(o2), k)

    def matmul_q_triple_m1(self, w1, kind1, n1, w2, kind2, n2, w3, kind3, n3, a, o1, o2, o3, k) -> int:
        return self._lib.rocknpu_matmul_q_triple_f32_f32_m1(
            self.handle, ptr(w1), w1.nbytes, kind1, n1, ptr(w2), w2.nbytes, kind2, n2, ptr(w3), w3.nbytes, kind3,
            n3, ptr(a), ptr(o1), ptr(o2), ptr(o3), k)

    # -- FP16 / W8 weights ---------------------------------------------------
    def matmul_f16(self, w_bits, a, out, m, k, n) -> int:
        return self._lib.rocknpu_matmul_f16_f32_f32(self.handle, ptr(w_bits), ptr(a), ptr(out), m, k, n)

    def matmul_w8a8_m1(self, w, s, a, out, k, n) -> int:
        return self._lib.rocknpu_matmul_w8a8_f32_f32_m1(self.handle, ptr(w), ptr(s), ptr(a), ptr(out), k, n)

    def matmul_w8a8_m16(self, w, s, a, out, k, n) -> int:
        return self._lib.rocknpu_matmul_w8a8_f32_f32_m16(self.handle, ptr(w), ptr(s), ptr(a), ptr(out), k, n)

    def matmul_w8a8_m1_nsplit(self, w, s, a, out, k, n, chunk_n) -> int:
        return self._lib.rocknpu_matmul_w8a8_f32_f32_m1_nsplit(self.handle, ptr(w), ptr(s), ptr(a), ptr(out), k,
                                                               n, chunk_n)

    def matmul_w8a8_pair_m1(self, w1, s1, n1, w2, s2, n2, a, o1, o2, k) -> int:
        return self._lib.rocknpu_matmul_w8a8_pair_f32_f32_m1(self.handle, ptr(w1), ptr(s1), n1, ptr(w2), ptr(s2),
                                                             n2, ptr(a), ptr(o1), ptr(o2), k)

    def matmul_w8a8_triple_m1(self, w1, s1, n1, w2, s2, n2, w3, s3, n3, a, o1, o2, o3, k) -> int:
        return self._lib.rocknpu_matmul_w8a8_triple_f32_f32_m1(
            self.handle, ptr(w1), ptr(s1), n1, ptr(w2), ptr(s2), n2, ptr(w3), ptr(s3), n3, ptr(a), ptr(o1),
            ptr(o2), ptr(o3), k)

    def matmul_w8a8_swiglu_down(self, gw, gs, uw, us, dw, ds, a, out, projection_k, ffn_n, output_n) -> int:
        return self._lib.rocknpu_matmul_w8a8_swiglu_down_f32(self.handle, ptr(gw), ptr(gs), ptr(uw), ptr(us),
                                                             ptr(dw), ptr(ds), ptr(a), ptr(out), projection_k,
                                                             ffn_n, output_n)
