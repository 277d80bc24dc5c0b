"""The allocation-free W8A8 entry point (rocknpu_b200_matmul_w8a8_noalloc).

It serves callers that may not allocate GPU memory once running (a memory
plan fixed at start-up, or a framework allocator that must own every byte)
by keeping its scratch in a fixed array inside the library.  The test calls it through the C ABI and
checks it against the context entry point rocknpu_b200_matmul_w8a8 on two
calls in a row, bit-exact (the tolerance every W8A8 test here uses), so that
contents left in the shared scratch by the first call cannot leak into the
second.  The file name keeps it last in collection order.
"""
import numpy as np
import pytest

import rocknpu_b200 as rk

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _noalloc(a, w, s, out, status, stream):
    m, k = a.shape
    n = w.shape[0]
    return rk.lib().rocknpu_b200_matmul_w8a8_noalloc(a.data_ptr(), w.data_ptr(), s.data_ptr(), out.data_ptr(), m, k,
                                                     n, status.data_ptr(), stream)


def _with_context(ctx, a, w, s, out, stream):
    m, k = a.shape
    n = w.shape[0]
    return rk.lib().rocknpu_b200_matmul_w8a8(ctx.handle, a.data_ptr(), w.data_ptr(), s.data_ptr(), out.data_ptr(), m,
                                             k, n, stream)


@pytest.mark.parametrize("m,k,n", [(128, 2048, 5632), (77, 5632, 256), (1, 2048, 512), (512, 2048, 2048)])
def test_noalloc_matches_context_entry_point_twice(m, k, n):
    rng = np.random.default_rng(m * 7 + n)
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.ones(1, dtype=torch.int32, device="cuda")
    with rk.Context() as ctx:
        for call in range(2):
            a = torch.from_numpy((rng.standard_normal((m, k)) * (1 + call)).astype(np.float32)).cuda()
            w = torch.from_numpy(rng.integers(-127, 128, size=(n, k), dtype=np.int8)).cuda()
            s = torch.from_numpy(rng.uniform(1e-3, 1e-2, size=n).astype(np.float32)).cuda()
            ref = torch.full((m, n), float("nan"), device="cuda")
            got = torch.full((m, n), float("nan"), device="cuda")
            assert _with_context(ctx, a, w, s, ref, stream) == 0
            torch.cuda.synchronize()
            assert rk.lib().rocknpu_b200_context_check(ctx.handle) == 0
            assert _noalloc(a, w, s, got, status, stream) == 0
            torch.cuda.synchronize()
            assert status.item() == 0
            assert torch.equal(got.view(torch.int32), ref.view(torch.int32)), f"call {call} differs"


def test_noalloc_rejects_oversize_and_flags_non_finite():
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    k, n = 8192, 128
    w = torch.zeros((n, k), dtype=torch.int8, device="cuda")
    s = torch.ones(n, device="cuda")
    a = torch.zeros((2048, k), device="cuda")
    out = torch.empty((2048, n), device="cuda")
    assert _noalloc(a, w, s, out, status, stream) == rk.STATUS_INVALID_ARGUMENT  # beyond the fixed scratch
    a = torch.ones((4, 256), device="cuda")
    a[1, 5] = float("inf")
    w = torch.ones((64, 256), dtype=torch.int8, device="cuda")
    s = torch.ones(64, device="cuda")
    out = torch.empty((4, 64), device="cuda")
    assert _noalloc(a, w, s, out, status, stream) == 0
    torch.cuda.synchronize()
    assert status.item() == 1
