"""The C ABI's opt-in K5b decode route (ROCKNPU_B200_DECODE_KQ set when the
context is created): M=1 Q4_K / Q6_K calls -- single, pair and triple -- are
served by the K-quant decode GEMV from cached decode layouts instead of the
W8A8 route's int8 rows.

Numerics: f32 results against the f64 product of the oracle's dequantised
weights and x, |y - ref| <= 1e-3 * |ref| + 2e-5 * sum_k |w_k x_k| (north_star's
1e-3 relative bound; the second term covers cancelling dot products).  The
W8A8 route's bit-exact results stay the default and are tested elsewhere;
here the same entry points without the switch are checked to give those bits.
"""
import numpy as np
import pytest

import oracle
import rocknpu_b200 as rk

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _check(y, kind, blocks, x, n):
    w = oracle.dequant(kind, blocks).reshape(n, -1).astype(np.float64)
    ref = w @ x.astype(np.float64)
    mag = np.abs(w) @ np.abs(x).astype(np.float64)
    err = np.abs(y.astype(np.float64) - ref)
    bad = np.nonzero(err > 1e-3 * np.abs(ref) + 2e-5 * mag)[0]
    assert bad.size == 0, f"{bad.size} rows outside the bound, first {bad[:5]}"


def _layout_bytes(kind, k, n):
    nb = k // 256
    return n * nb * 144 if kind == 4 else n * nb * 210 + 16


@pytest.fixture
def kq_ctx(monkeypatch):
    monkeypatch.setenv("ROCKNPU_B200_DECODE_KQ", "1")
    rk.apply_default_env()
    c = rk.Context()
    yield c
    c.close()


@pytest.fixture
def ctx(monkeypatch):
    monkeypatch.delenv("ROCKNPU_B200_DECODE_KQ", raising=False)
    rk.apply_default_env()
    c = rk.Context()
    yield c
    c.close()


@pytest.mark.parametrize("kind,k,n", [(4, 2048, 5632), (6, 2048, 2048), (4, 5632, 2048), (6, 5632, 256),
                                      (4, 512, 32), (6, 24576, 64)])
def test_single_m1(kq_ctx, kind, k, n):
    w = rk.synth_q_weights(kind, n, k, seed=500 + kind + n)
    x = rk.synth_normal(501 + k, k)
    y = np.empty(n, np.float32)
    assert kq_ctx.matmul_q(kind, w, x, y, 1, k, n) == 0
    _check(y, kind, w, x, n)
    s = kq_ctx.decode_cache_stats()
    assert (s.misses, s.hits, s.entries) == (1, 0, 1)
    assert s.resident_bytes == _layout_bytes(kind, k, n)
    y2 = np.full(n, np.nan, np.float32)
    assert kq_ctx.matmul_q(kind, w, x, y2, 1, k, n) == 0
    assert np.array_equal(_bits(y2), _bits(y))  # deterministic reduction
    s = kq_ctx.decode_cache_stats()
    assert (s.misses, s.hits, s.entries, s.worker1_calls) == (1, 1, 1, 2)


def test_random_blocks_outlier_x(kq_ctx, rng):
    """Every code, scale, min and sign of d, with outlier channels in x."""
    from conftest import random_kquant_blocks
    k, n = 4096, 96
    for kind in (4, 6):
        w = random_kquant_blocks(kind, n * (k // 256), rng)
        x = rng.standard_normal(k).astype(np.float32)
        x[rng.choice(k, k // 100, replace=False)] *= 20.0
        y = np.empty(n, np.float32)
        assert kq_ctx.matmul_q(kind, w, x, y, 1, k, n) == 0
        _check(y, kind, w, x, n)


@pytest.mark.parametrize("kinds", [(4, 4), (4, 6), (6, 6)])
def test_pair_m1(kq_ctx, kinds):
    k, n = 2048, 5632
    w1 = rk.synth_q_weights(kinds[0], n, k, seed=521)
    w2 = rk.synth_q_weights(kinds[1], n, k, seed=522)
    x = rk.synth_normal(523, k)
    o1, o2 = np.empty(n, np.float32), np.empty(n, np.float32)
    assert kq_ctx.matmul_q_pair_m1(w1, kinds[0], n, w2, kinds[1], n, x, o1, o2, k) == 0
    _check(o1, kinds[0], w1, x, n)
    _check(o2, kinds[1], w2, x, n)
    s = kq_ctx.decode_cache_stats()
    # one layout (and one GEMV launch) per same-kind group of the members
    if kinds[0] == kinds[1]:
        assert s.misses == 1 and s.entries == 1
        assert s.resident_bytes == _layout_bytes(kinds[0], k, 2 * n)
    else:
        assert s.misses == 1 and s.entries == 2
        assert s.resident_bytes == _layout_bytes(kinds[0], k, n) + _layout_bytes(kinds[1], k, n)
    p1, p2 = o1.copy(), o2.copy()
    assert kq_ctx.matmul_q_pair_m1(w1, kinds[0], n, w2, kinds[1], n, x, o1, o2, k) == 0
    assert np.array_equal(_bits(o1), _bits(p1)) and np.array_equal(_bits(o2), _bits(p2))  # deterministic
    s2 = kq_ctx.decode_cache_stats()
    assert s2.hits == s.hits + 1 and s2.entries == s.entries
    # a single call on one member: its own group, which a mixed-kind pair
    # already holds (a hit) and a same-kind pair does not (a new layout)
    y = np.empty(n, np.float32)
    assert kq_ctx.matmul_q(kinds[0], w1, x, y, 1, k, n) == 0
    _check(y, kinds[0], w1, x, n)
    s3 = kq_ctx.decode_cache_stats()
    if kinds[0] == kinds[1]:
        assert s3.misses == s2.misses + 1 and s3.entries == s2.entries + 1
    else:
        assert s3.hits == s2.hits + 1 and s3.entries == s2.entries
        assert np.array_equal(_bits(y), _bits(o1))


def test_triple_m1(kq_ctx):
    k = 2048
    ns, kinds = (2048, 256, 256), (4, 6, 4)
    ws = [rk.synth_q_weights(kd, n, k, seed=540 + i) for i, (kd, n) in enumerate(zip(kinds, ns))]
    x = rk.synth_normal(544, k)
    outs = [np.empty(n, np.float32) for n in ns]
    assert kq_ctx.matmul_q_triple_m1(ws[0], kinds[0], ns[0], ws[1], kinds[1], ns[1], ws[2], kinds[2], ns[2], x,
                                     *outs, k) == 0
    for o, w, kd, n in zip(outs, ws, kinds, ns):
        _check(o, kd, w, x, n)
    # q and k (Q4_K) share a layout, v (Q6_K) has its own
    s = kq_ctx.decode_cache_stats()
    assert s.entries == 2 and s.resident_bytes == _layout_bytes(4, k, 2048 + 256) + _layout_bytes(6, k, 256)


def test_non_finite_x_is_invalid_and_context_recovers(kq_ctx):
    k, n = 2048, 256
    w = rk.synth_q_weights(4, n, k, seed=550)
    x = rk.synth_normal(551, k)
    bad = x.copy()
    bad[1000] = np.inf
    y = np.zeros(n, np.float32)
    assert kq_ctx.matmul_q(4, w, bad, y, 1, k, n) == rk.STATUS_INVALID_ARGUMENT
    assert np.all(y == 0)  # outputs untouched on the error
    assert kq_ctx.matmul_q(4, w, x, y, 1, k, n) == 0
    _check(y, 4, w, x, n)


def test_shape_checks_unchanged(kq_ctx):
    """The M=1 entry's shape checks (k % 512, n % 32, n <= 8192) hold on the
    route too, and a wrong byte count is rejected."""
    k, n = 2048, 256
    w = rk.synth_q_weights(6, n, k, seed=560)
    x = rk.synth_normal(561, k)
    y = np.empty(8224, np.float32)
    assert kq_ctx.matmul_q(6, w, x, y, 1, k, 250, weights_bytes=250 * 8 * 210) == rk.STATUS_INVALID_ARGUMENT
    assert kq_ctx.matmul_q(6, w, x, y, 1, k, n, weights_bytes=w.nbytes - 1) == rk.STATUS_INVALID_ARGUMENT
    assert kq_ctx.decode_cache_stats().entries == 0


def test_wide_k_keeps_w8a8_bits(kq_ctx):
    """K above the GEMV's 24576 stays on the W8A8 route: the reference's bits."""
    k, n = 25088, 32
    w = rk.synth_q_weights(4, n, k, seed=570)
    x = rk.synth_normal(571, k)
    y = np.empty(n, np.float32)
    assert kq_ctx.matmul_q(4, w, x, y, 1, k, n) == 0
    st, ref = oracle.matmul_q(4, w, x.reshape(1, k), n)
    assert st == 0 and np.array_equal(_bits(y), _bits(ref.reshape(-1)))


def test_overlap_callback_runs_once(kq_ctx):
    k, n = 2048, 256
    w = rk.synth_q_weights(4, n, k, seed=580)
    x = rk.synth_normal(581, k)
    y = np.empty(n, np.float32)
    calls = []
    assert kq_ctx.set_overlap(lambda: calls.append(1)) == 0
    assert kq_ctx.matmul_q(4, w, x, y, 1, k, n) == 0
    assert kq_ctx.matmul_q(4, w, x, y, 1, k, n) == 0
    assert calls == [1]


def test_off_by_default_gives_w8a8_bits(ctx):
    k, n = 2048, 256
    for kind in (4, 6):
        w = rk.synth_q_weights(kind, n, k, seed=590 + kind)
        x = rk.synth_normal(591, k)
        y = np.empty(n, np.float32)
        assert ctx.matmul_q(kind, w, x, y, 1, k, n) == 0
        st, ref = oracle.matmul_q(kind, w, x.reshape(1, k), n)
        assert st == 0 and np.array_equal(_bits(y), _bits(ref.reshape(-1)))
