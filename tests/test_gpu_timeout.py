"""A bounded device wait that runs out, on one GPU, without a fault.

The reference bounds its NPU completion wait (2 s,
rocknpu-matmul/src/int8_decode.rs:13, :502) and reports a failed job instead
of hanging.  Here every device wait is bounded the same way.  This test makes
the peer barrier's flag wait run out on purpose: two peer buffers of one
world-2 group are created and opened in this process on the same GPU, and
only rank 0 ever enters the barrier, so rank 1's flag never arrives.  The
kernel must give up after the (shortened) limit, leave status 6
(kErrTimeoutPeer) -- which the C ABI maps to ROCKNPU_STATUS_EXECUTION_ERROR --
and the GPU context must stay usable: a W8A8 call afterwards is bit-exact
against the oracle, and rank 1's late barrier completes cleanly.
"""
import ctypes
import threading
import time

import numpy as np
import pytest

import oracle
import rocknpu_b200 as rk
from rocknpu_b200.capi import lib

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

HANDLE_BYTES = 64


def _create(rank: int, world: int, nbytes: int):
    handle = (ctypes.c_uint8 * HANDLE_BYTES)()
    h = ctypes.c_void_p()
    assert lib().rocknpu_b200_peer_buffer_create(nbytes, rank, world, handle, ctypes.byref(h)) == 0
    return h.value, bytes(handle)


def test_peer_barrier_wait_runs_out_and_context_stays_usable():
    torch.cuda.init()
    nbytes = 1 << 20
    b0, h0 = _create(0, 2, nbytes)
    b1, h1 = _create(1, 2, nbytes)
    allh = (ctypes.c_uint8 * (2 * HANDLE_BYTES)).from_buffer_copy(h0 + h1)
    results = {}

    def open_(name, b):
        results[name] = lib().rocknpu_b200_peer_buffer_open(b, allh)

    try:
        # each open sends its buffer to the other and waits for the other's,
        # so the two run on two host threads (ctypes releases the GIL)
        ts = [threading.Thread(target=open_, args=("r0", b0)), threading.Thread(target=open_, args=("r1", b1))]
        for t in ts:
            t.start()
        for t in ts:
            t.join(timeout=120)
        assert results == {"r0": 0, "r1": 0}

        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        assert lib().rocknpu_b200_set_peer_wait_limit_ms(20) == 0
        t0 = time.perf_counter()
        assert lib().rocknpu_b200_peer_barrier(b0, status.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        code = int(status.item())
        assert code == 6, f"expected the peer-barrier timeout code, got {code}"
        assert lib().rocknpu_b200_status_code(code) == rk.STATUS_EXECUTION_ERROR
        assert waited < 1.5, f"the 20 ms limit was not honoured ({waited:.3f} s)"

        # the context is still usable: rank 1 arrives late and its barrier
        # finds rank 0's flag already there
        assert lib().rocknpu_b200_set_peer_wait_limit_ms(0) == 0
        status.zero_()
        assert lib().rocknpu_b200_peer_barrier(b1, status.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        assert status.item() == 0
    finally:
        lib().rocknpu_b200_set_peer_wait_limit_ms(0)
        lib().rocknpu_b200_peer_buffer_destroy(b0)
        lib().rocknpu_b200_peer_buffer_destroy(b1)

    # and ordinary work on the same GPU context is bit-exact afterwards
    m, k, n = 64, 2048, 256
    w = rk.synth_q_weights(rk.Q4_K, n, k, seed=11)
    a = rk.synth_normal(12, m * k).reshape(m, k)
    out = np.empty((m, n), dtype=np.float32)
    with rk.Context() as ctx:
        assert ctx.matmul_q(rk.Q4_K, w, a, out, m, k, n) == 0
    st, ref = oracle.matmul_q(rk.Q4_K, w, a, n)
    assert st == 0
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))

