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


# (336, 49152, 256): the tile plan splits K (few output tiles, long K), but
# the int32 partial sums do not fit beside the 15.75 MiB of int8 activations
# in the 16 MiB array, so this call takes the branch that runs the GEMM
# without K splits.
@pytest.mark.parametrize("m,k,n", [(128, 2048, 5632), (77, 5632, 256), (1, 2048, 512), (512, 2048, 2048),
                                   (336, 49152, 256)])
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


def test_noalloc_no_split_branch_is_reached():
    """The shape above splits K in the context path (it has a workspace) and
    its partial sums would overflow the fixed array."""
    m, k, n = 336, 49152, 256
    ws = rk.lib().rocknpu_b200_gemm_workspace_bytes(m, n, k)
    assert ws > 0 and ws > (16 << 20) - (m * k + 4 * m)


def test_noalloc_rejects_oversize_and_flags_non_finite():
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # k not a multiple of 16: rejected before any work is queued, so the
    # status word keeps the value it had
    status.fill_(5)
    a = torch.ones((3, 200), device="cuda")
    w = torch.ones((64, 200), dtype=torch.int8, device="cuda")
    s = torch.ones(64, device="cuda")
    out = torch.empty((3, 64), device="cuda")
    assert _noalloc(a, w, s, out, status, stream) == rk.STATUS_INVALID_ARGUMENT
    torch.cuda.synchronize()
    assert status.item() == 5
    status.zero_()
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
