"""W8 sidecar: prepared int8 weights cached on disk next to a GGUF model.

``prepared_w8`` is the plugin's ``rocknpu_w8_sidecar_get``
(adapters/ggml-rocknpu/src/ggml-rocknpu.cpp:212-259): with
``ROCKNPU_W8_SIDECAR_DIR`` set it loads ``<dir>/<name>.w8`` / ``.scale.f32``
when ``<name>.source.fnv1a64`` matches the tensor's source bytes; otherwise,
unless ``ROCKNPU_W8_CONVERT=0``, it prepares the weight -- here with the K1
kernel on the GPU, bit-identical to the plugin's CPU conversion and to the
sidecar script -- and returns host arrays ready for the W8A8 entry points
(``rocknpu_matmul_w8a8_f32_f32_m1`` and friends take host int8 weights).
``write_sidecar`` produces the three files the reference script writes.
"""
from __future__ import annotations

import os

import numpy as np

from .capi import BLOCK_BYTES, STATUS_OK, lib, ptr


def source_fingerprint(source: np.ndarray) -> int:
    src = np.ascontiguousarray(source, dtype=np.uint8).reshape(-1)
    return int(lib().rocknpu_b200_source_fingerprint(ptr(src), src.size))


def read_sidecar(directory: str, name: str, source: np.ndarray, k: int, n: int):
    """(w8 [n, k] int8, scales [n] f32) from valid sidecar files, else None."""
    src = np.ascontiguousarray(source, dtype=np.uint8).reshape(-1)
    w8 = np.empty((n, k), dtype=np.int8)
    scales = np.empty(n, dtype=np.float32)
    st = lib().rocknpu_b200_w8_sidecar_read(directory.encode(), name.encode(), ptr(src), src.size, k, n, ptr(w8),
                                            ptr(scales))
    return (w8, scales) if st == STATUS_OK else None


def write_sidecar(directory: str, name: str, source: np.ndarray, w8: np.ndarray, scales: np.ndarray) -> None:
    src = np.ascontiguousarray(source, dtype=np.uint8).reshape(-1)
    w8 = np.ascontiguousarray(w8, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    n, k = w8.shape
    st = lib().rocknpu_b200_w8_sidecar_write(directory.encode(), name.encode(), ptr(src), src.size, k, n, ptr(w8),
                                             ptr(scales))
    if st != STATUS_OK:
        raise RuntimeError(f"rocknpu_b200_w8_sidecar_write({name}) failed with status {st}")


def prepare_on_gpu(kind: int, source: np.ndarray, k: int, n: int):
    """K1 on the current GPU, copied back to host arrays."""
    import torch

    from . import device
    src = np.ascontiguousarray(source, dtype=np.uint8).reshape(-1)
    if src.size != n * (k // 256) * BLOCK_BYTES[kind]:
        raise ValueError(f"{src.size} source bytes do not hold {n} rows of {k} kind-{kind} values")
    status = device.new_status()
    w8, scales = device.prepare_w8(kind, torch.from_numpy(src).cuda(), k, n, status)
    torch.cuda.synchronize()
    if status.item() != 0:
        return None  # non-finite dequantised values: the plugin rejects the tensor
    return w8.cpu().numpy(), scales.cpu().numpy()


def _convert_enabled() -> bool:
    # rocknpu_env_enabled_default("ROCKNPU_W8_CONVERT", true)
    # (ggml-rocknpu.cpp:266-272): unset or empty -> on, else first char != '0'
    v = os.environ.get("ROCKNPU_W8_CONVERT")
    return True if not v else v[0] != "0"


def prepared_w8(name: str, kind: int, source: np.ndarray, k: int, n: int, cache: dict | None = None):
    """The plugin's sidecar lookup for one weight tensor; None when neither a
    valid sidecar nor (allowed) conversion yields the weight."""
    if cache is not None and name in cache:
        hit = cache[name]
        return hit if hit is not None and hit[0].shape == (n, k) else None
    directory = os.environ.get("ROCKNPU_W8_SIDECAR_DIR", "")
    if not directory and not _convert_enabled():
        return None
    result = read_sidecar(directory, name, source, k, n) if directory else None
    if result is None and _convert_enabled():
        result = prepare_on_gpu(kind, source, k, n)
    if cache is not None:
        cache[name] = result
    return result
