"""Device-pointer entry points (include/rocknpu_b200.h) on torch CUDA tensors.

torch provides the device memory and the stream; the work is done by the
library's kernels.  Each function checks shapes and dtypes, queues the kernel
on the current torch stream (or the given one) and returns without waiting.
"""
from __future__ import annotations

import torch

from .capi import lib


def _stream(stream) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _check(st: int, what: str) -> None:
    if st != 0:
        raise RuntimeError(f"{what} failed with status {st}")


def new_status(device=None) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device or "cuda")


def prepare_w8(kind: int, blocks: torch.Tensor, k: int, n: int, status: torch.Tensor, stream=None):
    """K1: K-quant rows -> (int8 [n, k], f32 scales [n])."""
    assert blocks.is_cuda and blocks.dtype == torch.uint8 and blocks.is_contiguous()
    w = torch.empty((n, k), dtype=torch.int8, device=blocks.device)
    s = torch.empty(n, dtype=torch.float32, device=blocks.device)
    _check(lib().rocknpu_b200_prepare_w8(kind, blocks.data_ptr(), k, n, w.data_ptr(), s.data_ptr(),
                                         status.data_ptr(), _stream(stream)), "prepare_w8")
    return w, s


def quantize_rows(a: torch.Tensor, status: torch.Tensor, out: torch.Tensor | None = None,
                  scales: torch.Tensor | None = None, stream=None):
    """K2: f32 [m, k] -> (int8 [m, k], f32 scales [m])."""
    assert a.is_cuda and a.dtype == torch.float32 and a.is_contiguous() and a.dim() == 2
    m, k = a.shape
    out = torch.empty((m, k), dtype=torch.int8, device=a.device) if out is None else out
    scales = torch.empty(m, dtype=torch.float32, device=a.device) if scales is None else scales
    _check(lib().rocknpu_b200_quantize_rows(a.data_ptr(), m, k, out.data_ptr(), out.stride(0), scales.data_ptr(),
                                            status.data_ptr(), _stream(stream)), "quantize_rows")
    return out, scales


def workspace_bytes(m: int, n: int, k: int) -> int:
    return int(lib().rocknpu_b200_gemm_workspace_bytes(m, n, k))


def new_workspace(nbytes: int, device=None) -> torch.Tensor:
    """Zeroed split-K workspace (the GEMM keeps it zero between launches)."""
    return torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=device or "cuda")


def gemm_w8a8(a8: torch.Tensor, a_scales: torch.Tensor, w8: torch.Tensor, w_scales: torch.Tensor,
              status: torch.Tensor, out: torch.Tensor | None = None, acc: torch.Tensor | None = None,
              workspace: torch.Tensor | None = None, stream=None):
    """K3: (f32(acc) * a_s) * w_s with acc = a8 . w8^T exact int32."""
    m, k = a8.shape
    n = w8.shape[0]
    out = torch.empty((m, n), dtype=torch.float32, device=a8.device) if out is None else out
    ws_ptr = workspace.data_ptr() if workspace is not None else None
    ws_bytes = workspace.numel() if workspace is not None else 0
    _check(lib().rocknpu_b200_gemm_w8a8(a8.data_ptr(), a8.stride(0), a_scales.data_ptr(), w8.data_ptr(),
                                        w8.stride(0), w_scales.data_ptr(), out.data_ptr(), out.stride(0),
                                        acc.data_ptr() if acc is not None else None, m, k, n, ws_ptr, ws_bytes,
                                        status.data_ptr(), _stream(stream)), "gemm_w8a8")
    return out


def convert_f16(a: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """The FP16 executor's f32 -> f16 activation conversion (round to nearest even)."""
    assert a.is_cuda and a.dtype == torch.float32 and a.dim() == 2 and a.stride(1) == 1
    m, k = a.shape
    out = torch.empty((m, k), dtype=torch.float16, device=a.device) if out is None else out
    _check(lib().rocknpu_b200_convert_f16(a.data_ptr(), m, k, a.stride(0), out.data_ptr(), out.stride(0),
                                          _stream(stream)), "convert_f16")
    return out


def gemm_f16(a16: torch.Tensor, w16: torch.Tensor, status: torch.Tensor, out: torch.Tensor | None = None,
             stream=None):
    """K4: f16 [m, k] . f16 [n, k]^T accumulated in f32."""
    m, k = a16.shape
    n = w16.shape[0]
    out = torch.empty((m, n), dtype=torch.float32, device=a16.device) if out is None else out
    _check(lib().rocknpu_b200_gemm_f16(a16.data_ptr(), a16.stride(0), w16.data_ptr(), w16.stride(0), out.data_ptr(),
                                       out.stride(0), m, k, n, status.data_ptr(), _stream(stream)), "gemm_f16")
    return out


def gemv_w8a8(a8: torch.Tensor, a_scale: torch.Tensor, w8: torch.Tensor, w_scales: torch.Tensor,
              out: torch.Tensor | None = None, stream=None):
    """K5: M=1 W8A8 GEMV."""
    n, k = w8.shape
    out = torch.empty(n, dtype=torch.float32, device=w8.device) if out is None else out
    _check(lib().rocknpu_b200_gemv_w8a8(a8.data_ptr(), a_scale.data_ptr(), w8.data_ptr(), w_scales.data_ptr(),
                                        out.data_ptr(), k, n, _stream(stream)), "gemv_w8a8")
    return out


def kq_layout(kind: int, blocks: torch.Tensor, k: int, n: int, stream=None) -> torch.Tensor:
    """Decode layout of a K-quant weight (device uint8 blocks, n rows of k)."""
    nbytes = int(lib().rocknpu_b200_kq_layout_bytes(kind, k, n))
    if nbytes == 0:
        raise ValueError(f"no decode layout for kind {kind}, k={k}")
    out = torch.empty(nbytes, dtype=torch.uint8, device=blocks.device)
    _check(lib().rocknpu_b200_kq_layout(kind, blocks.data_ptr(), k, n, out.data_ptr(), _stream(stream)), "kq_layout")
    return out


def gemv_kq(kind: int, layout: torch.Tensor, x: torch.Tensor, n: int, status: torch.Tensor,
            out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """K5b: y[n] = dequant(W) . x straight from the K-quant decode layout."""
    k = x.numel()
    out = torch.empty(n, dtype=torch.float32, device=x.device) if out is None else out
    _check(lib().rocknpu_b200_gemv_kq(kind, layout.data_ptr(), k, n, x.data_ptr(), out.data_ptr(),
                                      status.data_ptr(), _stream(stream)), "gemv_kq")
    return out


def matmul_w8a8(ctx, a: torch.Tensor, w8: torch.Tensor, w_scales: torch.Tensor, out: torch.Tensor, stream=None):
    """K2 + K3 (K5 at m == 1) through a context's workspace.  On torch's
    default stream (handle 0, also what stream=None gives there) the work
    runs on the context's own stream: rocknpu_b200_context_check (or a device
    synchronisation) orders it before later reads of `out`."""
    m, k = a.shape
    n = w8.shape[0]
    _check(lib().rocknpu_b200_matmul_w8a8(ctx.handle, a.data_ptr(), w8.data_ptr(), w_scales.data_ptr(),
                                          out.data_ptr(), m, k, n, _stream(stream)), "matmul_w8a8")
    return out
