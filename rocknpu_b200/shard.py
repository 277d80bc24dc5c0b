"""N-sharded W8A8 MUL_MAT over the GPUs of one node, one process per GPU.

The reference splits a GEMM's weight rows (output columns) over its NPU
cores: n / 32 blocks of 32 rows, evenly, remainder blocks to the first
workers (rocknpu-matmul/src/int8_decode_pool.rs:1484-1522).  Here the
workers are GPUs: every rank keeps its rows' prepared int8 weights resident
(K1 on its own GPU), quantises the whole activation matrix (K2, replicated:
it is small next to the weights), runs the tcgen05 GEMM (K3) over its rows,
and the output columns are all-gathered so that every rank ends with ggml's
row-major [m][n] f32 result.  Columns are independent and K is never split
across ranks, so every int32 accumulator -- and every output value -- is
bit-identical to the single-GPU result.

Two exchange routes:

* ``"peer"`` (default): the GEMM epilogue stores each output tile straight
  into every rank's output buffer over NVLink (CUDA IPC mappings, plain
  stores), overlapping the exchange with the tensor-core work, then a
  device-side barrier orders those stores before the consumers.  Output
  buffers are double-buffered, so one barrier per call suffices.
* ``"allgather"``: each rank writes its block into a rank-major buffer,
  NCCL ``all_gather_into_tensor`` exchanges it, and a copy kernel lays it
  out row-major.

Requires ``torch.distributed`` initialised (NCCL for the all-gather route);
without it the module runs as a single rank.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import device as dev
from .capi import BLOCK_BYTES, lib

IPC_HANDLE_BYTES = 64
MAX_RANKS = 16


def shard_rows(n: int, world: int) -> list[tuple[int, int]]:
    """(start, width) of the weight rows of every rank (width 0: no rows)."""
    if world < 1 or world > MAX_RANKS:
        raise ValueError(f"world size {world} outside 1..{MAX_RANKS}")
    starts = (ctypes.c_size_t * world)()
    widths = (ctypes.c_size_t * world)()
    lib().rocknpu_b200_shard_rows(n, world, starts, widths)
    return [(int(starts[r]), int(widths[r])) for r in range(world)]


def _dist():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist
    return None


def exchange(payload: bytes, group=None) -> list[bytes]:
    """Every rank's `payload`, in rank order (host transport: the process
    group's object all-gather)."""
    dist = _dist()
    if dist is None:
        return [payload]
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, payload, group=group)
    return out


class _CudaArray:
    """A device pointer presented through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class PeerBuffer:
    """`nbytes` of device memory on this rank that every rank maps (IPC)."""

    def __init__(self, nbytes: int, group=None):
        dist = _dist()
        self.rank = dist.get_rank(group) if dist else 0
        self.world = dist.get_world_size(group) if dist else 1
        self.nbytes = nbytes
        handle = (ctypes.c_uint8 * IPC_HANDLE_BYTES)()
        h = ctypes.c_void_p()
        st = lib().rocknpu_b200_peer_buffer_create(nbytes, self.rank, self.world, handle, ctypes.byref(h))
        if st != 0:
            raise RuntimeError(f"rocknpu_b200_peer_buffer_create failed with status {st}")
        self.handle = h.value
        handles = exchange(bytes(handle), group)
        allh = (ctypes.c_uint8 * (IPC_HANDLE_BYTES * self.world)).from_buffer_copy(b"".join(handles))
        st = lib().rocknpu_b200_peer_buffer_open(self.handle, allh)
        if st != 0:
            self.close()
            raise RuntimeError(f"rocknpu_b200_peer_buffer_open failed with status {st}")
        self.ptrs = [int(lib().rocknpu_b200_peer_buffer_ptr(self.handle, r)) for r in range(self.world)]

    def tensor(self, shape, dtype=torch.float32) -> torch.Tensor:
        """This rank's data region as a tensor (no ownership: keep self alive)."""
        assert dtype == torch.float32
        assert int(np.prod(shape)) * 4 <= self.nbytes
        return torch.as_tensor(_CudaArray(self.ptrs[self.rank], shape), device=torch.device("cuda"))

    def barrier(self, status: torch.Tensor, stream=None) -> None:
        st = lib().rocknpu_b200_peer_barrier(self.handle, status.data_ptr(), dev._stream(stream))
        if st != 0:
            raise RuntimeError(f"rocknpu_b200_peer_barrier failed with status {st}")

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().rocknpu_b200_peer_buffer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ShardedMatmul:
    """One K-quant weight matrix [n rows x k] sharded over the ranks.

    ``blocks``: the whole weight's K-quant bytes (host numpy uint8, every
    rank holding the same file, as llama.cpp loads it) or only this rank's
    rows (``blocks_are_local=True``).  ``max_m``: the largest token count a
    call may use (sizes the peer buffers).
    """

    def __init__(self, kind: int, blocks, k: int, n: int, group=None, route: str = "peer", max_m: int = 512,
                 blocks_are_local: bool = False):
        if route not in ("peer", "allgather"):
            raise ValueError(f"unknown route {route!r}")
        if k % 256:
            raise ValueError("k must be a multiple of 256")
        dist = _dist()
        self.group = group
        self.rank = dist.get_rank(group) if dist else 0
        self.world = dist.get_world_size(group) if dist else 1
        self.kind, self.k, self.n, self.route, self.max_m = kind, k, n, route, max_m
        self.rows = shard_rows(n, self.world)
        self.start, self.width = self.rows[self.rank]
        self.shard_ld = max(w for _, w in self.rows)
        self.status = dev.new_status()
        row_bytes = k // 256 * BLOCK_BYTES[kind]
        self.w8 = self.w_scales = None
        if self.width:
            if blocks_are_local:
                mine = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
            else:
                flat = np.asarray(blocks, dtype=np.uint8).reshape(-1)
                mine = flat[self.start * row_bytes:(self.start + self.width) * row_bytes]
            if mine.size != self.width * row_bytes:
                raise ValueError(f"expected {self.width * row_bytes} weight bytes for rank {self.rank}")
            self.w8, self.w_scales = dev.prepare_w8(kind, torch.from_numpy(np.ascontiguousarray(mine)).cuda(), k,
                                                    self.width, self.status)
        self._a8 = self._as = None
        self._peer = None
        self._parity = 0
        self._gathered = None
        if route == "peer" and self.world > 1:
            # two output buffers, used alternately
            self._peer = [PeerBuffer(max_m * n * 4, group) for _ in range(2)]
        torch.cuda.synchronize()
        if self.status.item() != 0:
            raise RuntimeError("weight preparation reported non-finite values")

    # -- pieces of a call -------------------------------------------------
    def quantize(self, a: torch.Tensor):
        m = a.shape[0]
        if self._a8 is None or self._a8.shape[0] < m:
            self._a8 = torch.empty((max(m, 1), self.k), dtype=torch.int8, device=a.device)
            self._as = torch.empty(max(m, 1), dtype=torch.float32, device=a.device)
        a8, a_s = self._a8[:m], self._as[:m]
        dev.quantize_rows(a, self.status, out=a8, scales=a_s)
        return a8, a_s

    def __call__(self, a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Y[m, n] = W8A8(a, W) on every rank.  With the peer route and more
        than one rank the result lives in a library buffer that the call after
        next overwrites; pass ``out`` to have it copied."""
        m, k = a.shape
        if k != self.k or m > self.max_m:
            raise ValueError(f"activation shape {tuple(a.shape)} does not fit k={self.k}, max_m={self.max_m}")
        a8, a_s = self.quantize(a)
        return self.matmul_quantized(a8, a_s, out)

    def matmul_quantized(self, a8: torch.Tensor, a_s: torch.Tensor, out: torch.Tensor | None = None):
        m = a8.shape[0]
        if m == 1 and self.k % 16 == 0:
            return self._decode(a8, a_s, out)
        if self.world == 1:
            out = torch.empty((m, self.n), dtype=torch.float32, device=a8.device) if out is None else out
            dev.gemm_w8a8(a8, a_s, self.w8, self.w_scales, self.status, out=out)
            return out
        if self.route == "peer":
            buf = self._peer[self._parity]
            self._parity ^= 1
            if self.width:
                ptrs = (ctypes.c_void_p * self.world)(*buf.ptrs)
                st = lib().rocknpu_b200_gemm_w8a8_gather(a8.data_ptr(), a8.stride(0), a_s.data_ptr(),
                                                         self.w8.data_ptr(), self.w8.stride(0),
                                                         self.w_scales.data_ptr(), ptrs, self.world, self.start,
                                                         self.n, m, self.k, self.width, self.status.data_ptr(),
                                                         dev._stream(None))
                if st != 0:
                    raise RuntimeError(f"rocknpu_b200_gemm_w8a8_gather failed with status {st}")
            buf.barrier(self.status)
            y = buf.tensor((m, self.n))
            if out is not None:
                out.copy_(y)
                return out
            return y
        # all-gather route: rank-major blocks -> NCCL -> row-major
        dist = _dist()
        elems = m * self.shard_ld
        if self._gathered is None or self._gathered.numel() < self.world * elems:
            self._gathered = torch.empty(self.world * self.max_m * self.shard_ld, dtype=torch.float32,
                                         device=a8.device)
        gathered = self._gathered[:self.world * elems]
        mine = gathered[self.rank * elems:(self.rank + 1) * elems]
        if self.width:
            view = mine.view(m, self.shard_ld)[:, :self.width]
            dev.gemm_w8a8(a8, a_s, self.w8, self.w_scales, self.status, out=view)
        dist.all_gather_into_tensor(gathered, mine, group=self.group)
        out = torch.empty((m, self.n), dtype=torch.float32, device=a8.device) if out is None else out
        starts = (ctypes.c_size_t * self.world)(*[s for s, _ in self.rows])
        widths = (ctypes.c_size_t * self.world)(*[w for _, w in self.rows])
        st = lib().rocknpu_b200_gather_shards(gathered.data_ptr(), elems, self.shard_ld, m, self.world, starts,
                                              widths, out.data_ptr(), out.stride(0), dev._stream(None))
        if st != 0:
            raise RuntimeError(f"rocknpu_b200_gather_shards failed with status {st}")
        return out

    def _decode(self, a8: torch.Tensor, a_s: torch.Tensor, out: torch.Tensor | None):
        """M = 1: the K5 GEMV over this rank's rows, then an NCCL all-gather of
        the n floats (latency-bound at this size whichever route is chosen)."""
        if self.world == 1:
            out = torch.empty((1, self.n), dtype=torch.float32, device=a8.device) if out is None else out
            dev.gemv_w8a8(a8, a_s, self.w8, self.w_scales, out=out.view(-1))
            return out
        dist = _dist()
        gathered = torch.empty(self.world * self.shard_ld, dtype=torch.float32, device=a8.device)
        mine = gathered[self.rank * self.shard_ld:(self.rank + 1) * self.shard_ld]
        if self.width:
            dev.gemv_w8a8(a8, a_s, self.w8, self.w_scales, out=mine[:self.width])
        dist.all_gather_into_tensor(gathered, mine, group=self.group)
        out = torch.empty((1, self.n), dtype=torch.float32, device=a8.device) if out is None else out
        starts = (ctypes.c_size_t * self.world)(*[s for s, _ in self.rows])
        widths = (ctypes.c_size_t * self.world)(*[w for _, w in self.rows])
        st = lib().rocknpu_b200_gather_shards(gathered.data_ptr(), self.shard_ld, self.shard_ld, 1, self.world, starts,
                                              widths, out.data_ptr(), out.stride(0), dev._stream(None))
        if st != 0:
            raise RuntimeError(f"rocknpu_b200_gather_shards failed with status {st}")
        return out

    def check(self) -> None:
        """Wait for the GPU and raise if a kernel reported an error."""
        torch.cuda.synchronize()
        v = int(self.status.item())
        if v != 0:
            self.status.zero_()
            raise RuntimeError(f"device status {v} (1 = non-finite input, >1 = a bounded wait ran out)")

    def close(self) -> None:
        for b in self._peer or []:
            b.close()
        self._peer = None
