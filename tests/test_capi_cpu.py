"""Host-side checks of librocknpu.so that need no GPU: every declared symbol
is exported, the argument checks of the C ABI reject bad calls before any
device work, and the ggml plugin's supports_op rules."""
import ctypes
import os
import re

import pytest

import rocknpu_b200 as rk
from rocknpu_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = []
    for h in ("rocknpu.h", "rocknpu_b200.h"):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(rocknpu_\w+)\s*\(", text, flags=re.M)
    return sorted(set(n for n in names if not n.endswith("_fn")))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(capi.LIB_PATH)
    names = _declared_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding covers all of them
    assert set(names) <= set(capi.SIGNATURES), set(names) - set(capi.SIGNATURES)


def test_reference_header_entry_points_are_all_present():
    # the 22 exports of crates/rocknpu-capi/include/rocknpu.h
    expected = """rocknpu_device_count rocknpu_context_create rocknpu_context_decode_cache_stats
    rocknpu_context_destroy rocknpu_context_set_overlap rocknpu_matmul_q_concat_f32_f32_mtile rocknpu_mtile_release
    rocknpu_prewarm_quantized_m16 rocknpu_matmul_f16_f32_f32 rocknpu_matmul_w8a8_f32_f32_m1
    rocknpu_matmul_w8a8_f32_f32_m16 rocknpu_matmul_w8a8_f32_f32_m1_nsplit rocknpu_matmul_w8a8_swiglu_down_f32
    rocknpu_matmul_w8a8_pair_f32_f32_m1 rocknpu_matmul_q_pair_f32_f32_mtile rocknpu_matmul_w8a8_triple_f32_f32_m1
    rocknpu_matmul_q_pair_f32_f32_m1 rocknpu_matmul_q_triple_f32_f32_m1 rocknpu_matmul_q4_k_f32_f32
    rocknpu_matmul_q5_k_f32_f32 rocknpu_matmul_q6_k_f32_f32""".split()
    assert len(expected) == 21
    names = _declared_functions()
    assert all(e in names for e in expected)


def test_device_count_and_null_context():
    n = rk.device_count()
    assert n >= 0
    L = rk.lib()
    # null context is rejected before any pointer access (capi/src/lib.rs:5791-5806)
    assert L.rocknpu_matmul_f16_f32_f32(None, None, None, None, 4, 32, 16) == -1
    assert L.rocknpu_matmul_q4_k_f32_f32(None, None, 0, None, None, 1, 256, 32) == -1
    assert L.rocknpu_matmul_q6_k_f32_f32(None, None, 0, None, None, 1, 256, 32) == -1
    assert L.rocknpu_matmul_q5_k_f32_f32(None, None, 0, None, None, 2, 256, 32) == -1
    assert L.rocknpu_matmul_w8a8_f32_f32_m1(None, None, None, None, None, 512, 32) == -1
    assert L.rocknpu_matmul_w8a8_f32_f32_m16(None, None, None, None, None, 512, 32) == -1
    assert L.rocknpu_matmul_w8a8_f32_f32_m1_nsplit(None, None, None, None, None, 512, 32, 32) == -1
    assert L.rocknpu_matmul_q_concat_f32_f32_mtile(None, 1, None, None, None, None, None, None, 4, 512) == -1
    assert L.rocknpu_mtile_release(None, 1, None) == -1
    assert L.rocknpu_prewarm_quantized_m16(None, None, 0, 4, 2048, 256) == -1
    assert L.rocknpu_context_set_overlap(None, None, None) == -1
    assert L.rocknpu_context_decode_cache_stats(None, None) == -1
    L.rocknpu_context_destroy(None)  # no-op


def test_context_create_without_gpu_returns_null():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except Exception:
        pass
    assert rk.lib().rocknpu_context_create() is None
    assert rk.device_count() == 0


def test_device_entry_points_reject_bad_arguments():
    L = rk.lib()
    assert L.rocknpu_b200_prepare_w8(7, None, 256, 1, None, None, None, None) == -1
    assert L.rocknpu_b200_prepare_w8(4, 1, 100, 1, 1, 1, 1, None) == -1  # k % 256
    assert L.rocknpu_b200_prepare_w8(4, 4098, 256, 1, 16, 16, 16, None) == -1  # blocks not 4-byte aligned
    assert L.rocknpu_b200_quantize_rows(None, 1, 1, None, 1, None, None, None) == -1
    assert L.rocknpu_b200_gemm_w8a8(None, 0, None, None, 0, None, None, 0, None, 1, 1, 1, None, 0, None, None) == -1
    assert L.rocknpu_b200_gemv_w8a8(1, 1, 1, 1, 1, 100, 4, None) == -1  # k % 16
    assert L.rocknpu_b200_matmul_w8a8(None, None, None, None, None, 1, 1, 1, None) == -1
    assert L.rocknpu_b200_gemm_workspace_bytes(0, 1, 1) == 0


def test_host_buffer_entry_points_without_gpu():
    """rocknpu_b200_host_alloc / _free / _host_mapped on a machine with no
    GPU: nothing can be page-locked, so allocation returns NULL (and the
    Python helper raises), freeing NULL is a no-op, freeing any other pointer
    is rejected, and no host range counts as device-mapped."""
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except Exception:
        pass
    import numpy as np
    L = rk.lib()
    assert L.rocknpu_b200_host_alloc(1 << 20) is None
    assert L.rocknpu_b200_host_alloc(0) is None
    with pytest.raises(RuntimeError):
        rk.host_empty((16, 16))
    assert L.rocknpu_b200_host_free(None) == rk.STATUS_OK
    a = np.zeros(1024, dtype=np.float32)
    assert L.rocknpu_b200_host_free(a.ctypes.data) == rk.STATUS_INVALID_ARGUMENT
    assert L.rocknpu_b200_host_mapped(a.ctypes.data, a.nbytes) == 0
    assert L.rocknpu_b200_host_mapped(None, 16) == 0


# ---- ggml plugin supports_op rules (ggml-rocknpu.cpp:614-715) ---------------

ENV = ["ROCKNPU_W8_DIRECT_SUBMIT", "ROCKNPU_EXPERIMENT_DIRECT_SCRATCH", "ROCKNPU_PREFILL_CACHE",
       "ROCKNPU_NATIVE_MTILE", "ROCKNPU_W8_MTILE", "ROCKNPU_MTILE_PERSIST", "ROCKNPU_MTILE_MC",
       "ROCKNPU_NATIVE_MTILE_DOWN", "ROCKNPU_DECODE", "ROCKNPU_W8_MTILE_SCOPE", "ROCKNPU_M16_ONLY",
       "ROCKNPU_SCHED_FFN_ONLY", "ROCKNPU_NPU_OUTPUT_HEAD"]


@pytest.fixture
def clean_env(monkeypatch):
    for k in ENV:
        monkeypatch.delenv(k, raising=False)
    return monkeypatch


def _c_getenv(name):
    libc = ctypes.CDLL(None)
    libc.getenv.restype = ctypes.c_char_p
    v = libc.getenv(name.encode())
    return v.decode() if v is not None else None


def test_apply_default_env(clean_env):
    clean_env.setenv("ROCKNPU_MTILE_MC", "0")
    rk.apply_default_env()
    for k in ENV[:8]:
        if k != "ROCKNPU_MTILE_MC":
            assert _c_getenv(k) == "1"
    assert _c_getenv("ROCKNPU_MTILE_MC") == "0"  # never overwrites


def test_supports_op_defaults_tinyllama(clean_env):
    rk.apply_default_env()
    sup = rk.mul_mat_supported
    Q4, Q5, Q6, F16 = capi.GGML_Q4_K, capi.GGML_Q5_K, capi.GGML_Q6_K, capi.GGML_F16
    # prompt projections of TinyLlama at any batch size
    for m in (2, 5, 16, 100, 128, 512, 2048):
        assert sup(Q4, 2048, 2048, m) and sup(Q4, 2048, 256, m) and sup(Q6, 2048, 256, m)
        assert sup(Q4, 2048, 5632, m) and sup(Q6, 5632, 2048, m)
    # decode stays on the CPU by default (ROCKNPU_DECODE=cpu)
    assert not sup(Q4, 2048, 2048, 1)
    # vocabulary head is too wide (n > 3*8192)
    assert not sup(Q6, 2048, 32000, 512)
    # k must be a multiple of 256 with ceil512(k) <= 12288
    assert not sup(Q4, 2000, 2048, 16)
    assert not sup(Q4, 12544, 2048, 16)
    assert sup(Q4, 12288, 2048, 16)
    # n % 32
    assert not sup(Q4, 2048, 2000, 16)
    # Q5_K prompt needs k <= 4096, k % 512, n % 32, n <= 8192
    assert sup(Q5, 4096, 8192, 16) and not sup(Q5, 4608, 2048, 16) and not sup(Q5, 2048, 8224, 16)
    assert not sup(Q5, 2048, 2048, 1)
    # F16 weights: m % 4, k % 32, n % 16
    assert sup(F16, 64, 16, 4) and not sup(F16, 64, 16, 3) and not sup(F16, 48, 16, 4)
    # type / layout rejections
    assert not sup(Q4, 2048, 2048, 16, act_type=capi.GGML_F16)
    assert not sup(Q4, 2048, 2048, 16, dst_type=capi.GGML_F16)
    assert not sup(Q4, 2048, 2048, 16, contiguous=(True, False, True))
    assert not sup(Q4, 2048, 2048, 16, batch=(2, 1, 1, 1))
    assert not sup(capi.GGML_F32, 2048, 2048, 16)
    assert not sup(Q4, 2048, 2048, 16, is_mul_mat=False)


def test_supports_op_decode_and_env_switches(clean_env):
    rk.apply_default_env()
    sup = rk.mul_mat_supported
    Q4 = capi.GGML_Q4_K
    clean_env.setenv("ROCKNPU_DECODE", "npu")
    assert sup(Q4, 2048, 2048, 1) and sup(Q4, 5632, 2048, 1)
    assert not sup(Q4, 2304, 2048, 1)  # k % 512
    assert not sup(Q4, 2048, 32000, 1)  # output head off by default
    clean_env.setenv("ROCKNPU_NPU_OUTPUT_HEAD", "1")
    assert sup(Q4, 2048, 32000, 1) and not sup(Q4, 2048, 32800, 1)
    clean_env.setenv("ROCKNPU_M16_ONLY", "1")
    assert sup(Q4, 2048, 2048, 16) and not sup(Q4, 2048, 2048, 32)


def test_supports_op_without_native_routes(clean_env):
    # plugin loaded but its defaults switched off
    for k in ENV[:8]:
        clean_env.setenv(k, "0")
    sup = rk.mul_mat_supported
    Q4 = capi.GGML_Q4_K
    assert not sup(Q4, 2048, 2048, 129)  # m > 128 needs PREFILL_CACHE
    assert sup(Q4, 2048, 2048, 16)  # generic rule: m % 4, k % 256, n % 16
    assert not sup(Q4, 2048, 2048, 8)  # small M needs the native W8 path
    assert not sup(Q4, 2048, 9000, 16)  # n > 8192


def test_status_code_mapping():
    """Device status words map to the reference's status codes the way the
    host-pointer entry points report them (rocknpu.h:27-32)."""
    L = rk.lib()
    assert L.rocknpu_b200_status_code(0) == rk.STATUS_OK
    assert L.rocknpu_b200_status_code(1) == rk.STATUS_INVALID_ARGUMENT
    for code in range(2, 8):
        assert L.rocknpu_b200_status_code(code) == rk.STATUS_EXECUTION_ERROR
    assert L.rocknpu_b200_set_peer_wait_limit_ms(600001) == rk.STATUS_INVALID_ARGUMENT
    assert L.rocknpu_b200_set_peer_wait_limit_ms(0) == rk.STATUS_OK
