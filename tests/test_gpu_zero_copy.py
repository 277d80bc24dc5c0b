"""Host-pointer calls on page-locked, device-mapped buffers.

The C ABI reads such activations and writes such outputs in place (the
quantiser and the GEMM epilogue access host memory over PCIe) instead of
copying them through device buffers.  Every result must be the same bits as
the oracle's and as the copy route's, in every ROCKNPU_B200_ZERO_COPY mode,
and a rejected call must leave an in-place output untouched.
"""
import numpy as np
import pytest

import oracle
import rocknpu_b200 as rk

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

MODES = ["1", "in", "out", "0"]


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _pinned(shape, fill=np.nan):
    t = torch.empty(shape, dtype=torch.float32).pin_memory()
    a = t.numpy()
    a[...] = fill
    return t, a


def _mapped(a: np.ndarray) -> int:
    return rk.lib().rocknpu_b200_host_mapped(a.ctypes.data, a.nbytes)


@pytest.fixture
def ctx():
    # one context per test: its resident-weight caches are keyed by the host
    # address of the weight bytes (the reference's DecodeWeightKey), and a
    # freed test array's address can come back for the next test's weights
    rk.apply_default_env()
    c = rk.Context()
    yield c
    c.close()


def test_host_mapped_query():
    t, a = _pinned((64, 128))
    assert _mapped(a) == 1
    assert _mapped(a[8:]) == 1                      # an interior range
    assert rk.lib().rocknpu_b200_host_mapped(a.ctypes.data, 1 << 40) == 0  # runs past the allocation
    assert _mapped(np.zeros((64, 128), dtype=np.float32)) == 0  # pageable
    assert rk.lib().rocknpu_b200_host_mapped(None, 16) == 0
    assert rk.lib().rocknpu_b200_host_mapped(a.ctypes.data, 0) == 0
    dev_t = torch.empty(1024, device="cuda")
    assert rk.lib().rocknpu_b200_host_mapped(dev_t.data_ptr(), 4096) == 0  # device memory


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("kind,m,k,n", [(4, 512, 2048, 2048), (6, 300, 2048, 96), (4, 77, 5632, 256),
                                        (4, 1000, 2048, 640), (6, 16, 2048, 2048)])
def test_matmul_q_in_place_bit_exact(ctx, rng, monkeypatch, mode, kind, m, k, n):
    monkeypatch.setenv("ROCKNPU_B200_ZERO_COPY", mode)
    blocks = rk.synth_q_weights(kind, n, k, seed=31 + m)
    ta, a = _pinned((m, k))
    a[...] = rng.standard_normal((m, k)).astype(np.float32)
    to, out = _pinned((m, n))
    assert _mapped(a) == 1 and _mapped(out) == 1
    assert ctx.matmul_q(kind, blocks, a, out, m, k, n) == 0
    st, ref = oracle.matmul_q(kind, blocks, a, n)
    assert st == 0
    assert np.array_equal(_bits(out), _bits(ref))


@pytest.mark.parametrize("mode", MODES)
def test_concat_group_in_place(ctx, rng, monkeypatch, mode):
    monkeypatch.setenv("ROCKNPU_B200_ZERO_COPY", mode)
    m, k = 192, 2048
    ns, kinds = [2048, 256, 256], [4, 4, 6]
    ws = [rk.synth_q_weights(kd, n, k, seed=60 + i) for i, (kd, n) in enumerate(zip(kinds, ns))]
    ta, a = _pinned((m, k))
    a[...] = rng.standard_normal((m, k)).astype(np.float32)
    pinned = [_pinned((m, n)) for n in ns]
    outs = [o for _, o in pinned]
    assert ctx.matmul_q_concat(ws, kinds, ns, a, outs, m, k) == 0
    for w, kd, n, o in zip(ws, kinds, ns, outs):
        st, ref = oracle.matmul_q(kd, w, a, n)
        assert np.array_equal(_bits(o), _bits(ref))


def test_mixed_pinned_and_pageable_members(ctx, rng):
    # one pageable member output: the outputs go through the copy pipeline,
    # the pinned activations are still read in place
    m, k = 64, 2048
    ns, kinds = [2048, 256], [4, 6]
    ws = [rk.synth_q_weights(kd, n, k, seed=70 + i) for i, (kd, n) in enumerate(zip(kinds, ns))]
    ta, a = _pinned((m, k))
    a[...] = rng.standard_normal((m, k)).astype(np.float32)
    to, o0 = _pinned((m, ns[0]))
    o1 = np.full((m, ns[1]), np.nan, dtype=np.float32)
    assert ctx.matmul_q_concat(ws, kinds, ns, a, [o0, o1], m, k) == 0
    for w, kd, n, o in zip(ws, kinds, ns, [o0, o1]):
        st, ref = oracle.matmul_q(kd, w, a, n)
        assert np.array_equal(_bits(o), _bits(ref))


@pytest.mark.parametrize("mode", ["1", "out"])
@pytest.mark.parametrize("m", [4, 700])
def test_rejected_call_leaves_in_place_output_untouched(ctx, rng, monkeypatch, mode, m):
    # the epilogue's store guard: nothing reaches an in-place output once the
    # quantiser has flagged a non-finite row (with copies, rows of chunks
    # finished before the bad one are copied back, as the reference's
    # chunked prompt path leaves them)
    monkeypatch.setenv("ROCKNPU_B200_ZERO_COPY", mode)
    k, n = 2048, 256
    blocks = rk.synth_q_weights(4, n, k, seed=4)
    ta, a = _pinned((m, k))
    a[...] = rng.standard_normal((m, k)).astype(np.float32)
    a[m // 2, 3] = np.inf
    to, out = _pinned((m, n), fill=0.0)
    assert ctx.matmul_q(4, blocks, a, out, m, k, n) == -1
    if mode == "1":
        assert not out.any()  # one launch pair: nothing stored
    else:
        # activations still copied in row chunks: chunks before the bad
        # row's may be stored, nothing from its chunk on
        assert not out[m // 2:].any()
    a[m // 2, 3] = 0.0
    assert ctx.matmul_q(4, blocks, a, out, m, k, n) == 0  # status cleared, context usable
    st, ref = oracle.matmul_q(4, blocks, a, n)
    assert np.array_equal(_bits(out), _bits(ref))


@pytest.mark.parametrize("mode", MODES)
def test_f16_executor_in_place_equals_copied(ctx, rng, monkeypatch, mode):
    m, k, n = 96, 1024, 160
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float16)
    ta, a = _pinned((m, k))
    a[...] = rng.standard_normal((m, k)).astype(np.float32)
    copied = np.empty((m, n), dtype=np.float32)
    monkeypatch.setenv("ROCKNPU_B200_ZERO_COPY", "0")
    assert ctx.matmul_f16(w.view(np.uint16), a, copied, m, k, n) == 0
    monkeypatch.setenv("ROCKNPU_B200_ZERO_COPY", mode)
    to, out = _pinned((m, n))
    assert ctx.matmul_f16(w.view(np.uint16), a, out, m, k, n) == 0
    assert np.array_equal(_bits(out), _bits(copied))
    ref = oracle.matmul_f16(w.view(np.uint16), a)
    np.testing.assert_allclose(out, ref, rtol=1e-3, atol=1e-3 * np.abs(ref).max())


@pytest.mark.parametrize("mode", MODES)
def test_host_alloc_buffers(ctx, rng, monkeypatch, mode):
    monkeypatch.setenv("ROCKNPU_B200_ZERO_COPY", mode)
    m, k, n = 300, 2048, 640
    a = rk.host_empty((m, k))
    out = rk.host_empty((m, n))
    assert a.ctypes.data % (2 << 20) == 0
    assert _mapped(a) == 1 and _mapped(out) == 1
    a[...] = rng.standard_normal((m, k)).astype(np.float32)
    out[...] = np.nan
    blocks = rk.synth_q_weights(4, n, k, seed=90)
    assert ctx.matmul_q(4, blocks, a, out, m, k, n) == 0
    st, ref = oracle.matmul_q(4, blocks, a, n)
    assert np.array_equal(_bits(out), _bits(ref))
    # only block starts are released; the block goes with its last view
    assert rk.lib().rocknpu_b200_host_free(a.ctypes.data + 4096) == rk.STATUS_INVALID_ARGUMENT
