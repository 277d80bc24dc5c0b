"""ctypes view of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py`` -- as the checker and the timed CPU
reference -- and never by the ``rocknpu_b200`` package.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

Q4_K, Q5_K, Q6_K = 4, 5, 6
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc, OpenMP)."""
    srcs = [os.path.join(_HERE, f) for f in ("oracle.c", "synth.c", "oracle.h", "Makefile")]
    stale = (not os.path.exists(_LIB_PATH)
             or any(os.path.getmtime(_LIB_PATH) < os.path.getmtime(s) for s in srcs))
    if force or stale:
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "liboracle.so"],
                       check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        S = ctypes.c_size_t
        L.orc_block_bytes.restype = S
        L.orc_block_bytes.argtypes = [ctypes.c_uint32]
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        for name in ("orc_dequant_q4_k", "orc_dequant_q5_k", "orc_dequant_q6_k"):
            getattr(L, name).restype = None
            getattr(L, name).argtypes = [P, S, P]
        L.orc_quantize_symmetric_into.restype = ctypes.c_int
        L.orc_quantize_symmetric_into.argtypes = [P, S, P, P]
        L.orc_prepare_w8a8.restype = ctypes.c_int
        L.orc_prepare_w8a8.argtypes = [ctypes.c_uint32, P, S, S, S, P, P]
        L.orc_gemm_path.restype = ctypes.c_int
        L.orc_gemm_path.argtypes = [S, S, S]
        L.orc_gemm_i8_i32.restype = None
        L.orc_gemm_i8_i32.argtypes = [P, P, P, S, S, S]
        L.orc_rescale_i32_row.restype = None
        L.orc_rescale_i32_row.argtypes = [P, P, ctypes.c_float, P, S]
        L.orc_quantize_rows.restype = ctypes.c_int
        L.orc_quantize_rows.argtypes = [P, S, S, P, P]
        L.orc_matmul_w8a8.restype = ctypes.c_int
        L.orc_matmul_w8a8.argtypes = [P, P, P, P, P, S, S, S]
        L.orc_matmul_q.restype = ctypes.c_int
        L.orc_matmul_q.argtypes = [ctypes.c_uint32, P, S, P, P, P, S, S, S]
        L.orc_matmul_f16.restype = None
        L.orc_matmul_f16.argtypes = [P, P, P, S, S, S]
        L.orc_swiglu.restype = None
        L.orc_swiglu.argtypes = [P, P, P, S]
        L.orc_source_fingerprint.restype = ctypes.c_uint64
        L.orc_source_fingerprint.argtypes = [P, S]
        L.orc_hilo_stack.restype = ctypes.c_int
        L.orc_hilo_stack.argtypes = [P, S, S, P]
        L.orc_hilo_sum.restype = None
        L.orc_hilo_sum.argtypes = [P, S, P]
        L.orc_split_blocks.restype = S
        L.orc_split_blocks.argtypes = [S, S, S, P, P]
        L.orc_threads.restype = ctypes.c_int
        L.orc_threads.argtypes = []
        L.orc_set_threads.restype = None
        L.orc_set_threads.argtypes = [ctypes.c_int]
        L.orc_synth_normal.restype = None
        L.orc_synth_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, S, ctypes.c_float, P]
        L.orc_synth_encode.restype = ctypes.c_int
        L.orc_synth_encode.argtypes = [ctypes.c_uint32, P, S, S, P]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def threads() -> int:
    return int(lib().orc_threads())


def set_threads(n: int) -> None:
    """OpenMP threads of the oracle's parallel loops from now on."""
    lib().orc_set_threads(int(n))


def host_threads() -> int:
    """Every hardware thread this process may run on (its CPU affinity set),
    whatever OMP_NUM_THREADS the launcher exported."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def synth_normal(seed: int, count: int, sigma: float = 1.0, first: int = 0) -> np.ndarray:
    """Seeded N(0, sigma^2) f32 values, the same as the library's
    rocknpu_synth_normal."""
    out = np.empty(count, dtype=np.float32)
    lib().orc_synth_normal(seed, first, count, sigma, _p(out))
    return out


def synth_encode(kind: int, values: np.ndarray) -> np.ndarray:
    """Rows of f32 values [n, k] as K-quant superblocks (flat uint8), the same
    bytes as the library's rocknpu_synth_encode."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    n, k = values.shape
    out = np.empty(n * (k // 256) * BLOCK_BYTES[kind], dtype=np.uint8)
    if lib().orc_synth_encode(kind, _p(values), k, n, _p(out)) != 0:
        raise ValueError("synth_encode: k must be a multiple of 256")
    return out


def synth_q_weights(kind: int, n: int, k: int, seed: int, sigma: float = 0.02) -> np.ndarray:
    """Seeded N(0, sigma^2) weights [n, k] encoded as K-quant blocks, the same
    bytes as rocknpu_b200.synth_q_weights."""
    return synth_encode(kind, synth_normal(seed, n * k, sigma).reshape(n, k))


def dequant(kind: int, blocks: np.ndarray) -> np.ndarray:
    """Dequantise a flat byte array of K-quant superblocks to f32."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    nb = blocks.size // BLOCK_BYTES[kind]
    assert nb * BLOCK_BYTES[kind] == blocks.size
    out = np.empty(nb * 256, dtype=np.float32)
    fn = {Q4_K: lib().orc_dequant_q4_k, Q5_K: lib().orc_dequant_q5_k, Q6_K: lib().orc_dequant_q6_k}[kind]
    fn(_p(blocks), nb, _p(out))
    return out


def quantize_symmetric(values: np.ndarray):
    """(int8 row, scale) or None for a non-finite row."""
    values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    out = np.empty(values.size, dtype=np.int8)
    scale = np.zeros(1, dtype=np.float32)
    if lib().orc_quantize_symmetric_into(_p(values), values.size, _p(out), _p(scale)) != 0:
        return None
    return out, np.float32(scale[0])


def quantize_rows(a: np.ndarray):
    a = np.ascontiguousarray(a, dtype=np.float32)
    m, k = a.shape
    q = np.empty((m, k), dtype=np.int8)
    s = np.empty(m, dtype=np.float32)
    st = lib().orc_quantize_rows(_p(a), m, k, _p(q), _p(s))
    return st, q, s


def prepare_w8a8(kind: int, blocks: np.ndarray, k: int, n: int):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    w = np.empty((n, k), dtype=np.int8)
    s = np.empty(n, dtype=np.float32)
    st = lib().orc_prepare_w8a8(kind, _p(blocks), blocks.size, k, n, _p(w), _p(s))
    return st, w, s


def gemm_path(m: int, k: int, n: int) -> str:
    """The CPU path of the exact int8 GEMM for this shape: amx, vnni or scalar."""
    return {2: "amx", 1: "vnni", 0: "scalar"}[int(lib().orc_gemm_path(m, k, n))]


def gemm_i8_i32(a: np.ndarray, w: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.int8)
    w = np.ascontiguousarray(w, dtype=np.int8)
    m, k = a.shape
    n = w.shape[0]
    c = np.empty((m, n), dtype=np.int32)
    lib().orc_gemm_i8_i32(_p(a), _p(w), _p(c), m, k, n)
    return c


def matmul_w8a8(w: np.ndarray, w_scales: np.ndarray, a: np.ndarray, want_acc: bool = False):
    w = np.ascontiguousarray(w, dtype=np.int8)
    w_scales = np.ascontiguousarray(w_scales, dtype=np.float32)
    a = np.ascontiguousarray(a, dtype=np.float32)
    m, k = a.shape
    n = w.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    acc = np.empty((m, n), dtype=np.int32) if want_acc else None
    st = lib().orc_matmul_w8a8(_p(w), _p(w_scales), _p(a), _p(out),
                               _p(acc) if want_acc else None, m, k, n)
    return (st, out, acc) if want_acc else (st, out)


def matmul_q(kind: int, blocks: np.ndarray, a: np.ndarray, n: int, want_acc: bool = False):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    a = np.ascontiguousarray(a, dtype=np.float32)
    m, k = a.shape
    out = np.empty((m, n), dtype=np.float32)
    acc = np.empty((m, n), dtype=np.int32) if want_acc else None
    st = lib().orc_matmul_q(kind, _p(blocks), blocks.size, _p(a), _p(out),
                            _p(acc) if want_acc else None, m, k, n)
    return (st, out, acc) if want_acc else (st, out)


def matmul_f16(w_bits: np.ndarray, a: np.ndarray) -> np.ndarray:
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    a = np.ascontiguousarray(a, dtype=np.float32)
    m, k = a.shape
    n = w_bits.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    lib().orc_matmul_f16(_p(w_bits), _p(a), _p(out), m, k, n)
    return out


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    gate = np.ascontiguousarray(gate, dtype=np.float32)
    up = np.ascontiguousarray(up, dtype=np.float32)
    out = np.empty_like(gate)
    lib().orc_swiglu(_p(gate), _p(up), _p(out), gate.size)
    return out


def source_fingerprint(data: np.ndarray) -> int:
    data = np.ascontiguousarray(data, dtype=np.uint8).reshape(-1)
    return int(lib().orc_source_fingerprint(_p(data), data.size))


def hilo_stack(a: np.ndarray):
    """(status, stacked [2m, k]) of the two-part activation encoding."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    m, k = a.shape
    out = np.empty((2 * m, k), dtype=np.float32)
    st = lib().orc_hilo_stack(_p(a), m, k, _p(out))
    return st, out


def hilo_sum(stacked: np.ndarray) -> np.ndarray:
    stacked = np.ascontiguousarray(stacked, dtype=np.float32)
    half = stacked.shape[0] // 2
    out = np.empty((half,) + stacked.shape[1:], dtype=np.float32)
    lib().orc_hilo_sum(_p(stacked), out.size, _p(out))
    return out


def matmul_w8a8_hilo(w: np.ndarray, w_scales: np.ndarray, a: np.ndarray):
    """The reference's HILO prompt projection: W8A8 over [x; residual(x)],
    then the two output halves summed (capi/src/lib.rs:4981-5001)."""
    st, stacked = hilo_stack(a)
    if st != 0:
        return st, None
    st, y = matmul_w8a8(w, w_scales, stacked)
    if st != 0:
        return st, None
    return 0, hilo_sum(y)


def split_blocks(blocks: int, block_width: int, workers: int):
    starts = np.zeros(max(workers, 1), dtype=np.uint64)
    widths = np.zeros(max(workers, 1), dtype=np.uint64)
    n = lib().orc_split_blocks(blocks, block_width, workers, _p(starts), _p(widths))
    return [(int(starts[i]), int(widths[i])) for i in range(n)]


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    L = lib()
    flat = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    return np.array([L.orc_f32_to_f16(float(v)) for v in flat], dtype=np.uint16).reshape(np.shape(x))
