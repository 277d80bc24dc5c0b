"""GPU parity of the C-ABI exports that only the ggml plugin's decode and cache
paths call, each against the CPU oracle through include/rocknpu.h:

* rocknpu_matmul_w8a8_swiglu_down_f32   capi/src/lib.rs:4308-4389
* rocknpu_matmul_w8a8_f32_f32_m1_nsplit  :4259-4300
* rocknpu_matmul_q_pair_f32_f32_m1       :4633-4717
* rocknpu_matmul_q_pair_f32_f32_mtile    :4719-4821
* rocknpu_matmul_q_triple_f32_f32_m1     :4823-4931
* rocknpu_mtile_release                  :2426-2445
* rocknpu_prewarm_quantized_m16          :4074-4121
* rocknpu_context_set_overlap            :3860-3878

W8A8 outputs are compared bit for bit: int8 quantisation and int32 sums are
exact and the rescale runs in the reference's operation order.  The SwiGLU
between the gate/up and down projections runs on the host with the C
library's expf, which is what Rust's f32::exp calls, so its activations --
and therefore the down projection -- are bit-exact too.
"""
import numpy as np
import pytest

import oracle
import rocknpu_b200 as rk

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.fixture
def ctx():
    rk.apply_default_env()
    c = rk.Context()
    yield c
    c.close()


def _w8(rng, n, k):
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    s = rng.uniform(1e-3, 1e-2, size=n).astype(np.float32)
    return w, s


def _m1(w, s, a):
    st, y = oracle.matmul_w8a8(w, s, a.reshape(1, -1))
    assert st == 0
    return y.reshape(-1)


@pytest.mark.parametrize("k,ffn,out_n", [(2048, 5632, 2048), (1024, 4096, 1024)])
def test_swiglu_down_bit_exact(ctx, rng, k, ffn, out_n):
    gw, gs = _w8(rng, ffn, k)
    uw, us = _w8(rng, ffn, k)
    dw, ds = _w8(rng, out_n, ffn)
    a = rng.standard_normal(k).astype(np.float32)
    out = np.empty(out_n, dtype=np.float32)
    assert ctx.matmul_w8a8_swiglu_down(gw, gs, uw, us, dw, ds, a, out, k, ffn, out_n) == 0
    gate, up = _m1(gw, gs, a), _m1(uw, us, a)
    act = oracle.swiglu(gate, up)
    ref = _m1(dw, ds, act)
    assert np.array_equal(_bits(out), _bits(ref))


def test_swiglu_down_rejects_non_finite(ctx, rng):
    k, ffn, out_n = 512, 512, 256
    gw, gs = _w8(rng, ffn, k)
    uw, us = _w8(rng, ffn, k)
    dw, ds = _w8(rng, out_n, ffn)
    a = rng.standard_normal(k).astype(np.float32)
    a[7] = np.nan
    out = np.full(out_n, 3.0, dtype=np.float32)
    assert ctx.matmul_w8a8_swiglu_down(gw, gs, uw, us, dw, ds, a, out, k, ffn, out_n) == rk.STATUS_INVALID_ARGUMENT


@pytest.mark.parametrize("n,chunk", [(32000, 8192), (20480, 4096), (2048, 8192)])
def test_m1_nsplit_bit_exact(ctx, rng, n, chunk):
    k = 2048
    w, s = _w8(rng, n, k)
    a = rng.standard_normal(k).astype(np.float32)
    out = np.empty(n, dtype=np.float32)
    assert ctx.matmul_w8a8_m1_nsplit(w, s, a, out, k, n, chunk) == 0
    assert np.array_equal(_bits(out), _bits(_m1(w, s, a)))
    # one decode-cache entry per chunk, like the reference's per-chunk calls
    assert ctx.decode_cache_stats().entries == (n + chunk - 1) // chunk
    assert ctx.matmul_w8a8_m1_nsplit(w, s, a, out, k, n, 100) == rk.STATUS_INVALID_ARGUMENT  # chunk % 32


@pytest.mark.parametrize("kinds", [(4, 4), (4, 6), (6, 6)])
def test_q_pair_m1_bit_exact(ctx, kinds):
    k, n = 2048, 5632
    w1 = rk.synth_q_weights(kinds[0], n, k, seed=21)
    w2 = rk.synth_q_weights(kinds[1], n, k, seed=22)
    a = rk.synth_normal(23, k)
    o1, o2 = np.empty(n, np.float32), np.empty(n, np.float32)
    assert ctx.matmul_q_pair_m1(w1, kinds[0], n, w2, kinds[1], n, a, o1, o2, k) == 0
    for o, w, kd in ((o1, w1, kinds[0]), (o2, w2, kinds[1])):
        st, ref = oracle.matmul_q(kd, w, a.reshape(1, k), n)
        assert st == 0
        assert np.array_equal(_bits(o), _bits(ref.reshape(-1)))
    st = ctx.decode_cache_stats()
    assert st.misses == 1 and st.entries == 1
    assert ctx.matmul_q_pair_m1(w1, kinds[0], n, w2, kinds[1], n, a, o1, o2, k) == 0
    assert ctx.decode_cache_stats().hits == st.hits + 1
    # a wrong byte count is rejected (prepare_q*_k_w8a8's check, L:713-717)
    assert ctx._lib.rocknpu_matmul_q_pair_f32_f32_m1(ctx.handle, w1.ctypes.data, w1.nbytes - 1, kinds[0], n,
                                                     w2.ctypes.data, w2.nbytes, kinds[1], n, a.ctypes.data,
                                                     o1.ctypes.data, o2.ctypes.data, k) == rk.STATUS_INVALID_ARGUMENT


@pytest.mark.parametrize("m", [4, 16, 64, 128])
def test_q_pair_mtile_bit_exact(ctx, m):
    k, n = 2048, 5632
    w1 = rk.synth_q_weights(4, n, k, seed=31)
    w2 = rk.synth_q_weights(6, n, k, seed=32)
    a = rk.synth_normal(33 + m, m * k).reshape(m, k)
    o1, o2 = np.empty((m, n), np.float32), np.empty((m, n), np.float32)
    assert ctx.matmul_q_pair_mtile(w1, 4, n, w2, 6, n, a, o1, o2, m, k) == 0
    for o, w, kd in ((o1, w1, 4), (o2, w2, 6)):
        st, ref = oracle.matmul_q(kd, w, a, n)
        assert st == 0
        assert np.array_equal(_bits(o), _bits(ref))
    # rows outside MTILE_ROWS are rejected (L:2628-2639)
    assert ctx.matmul_q_pair_mtile(w1, 4, n, w2, 6, n, a[:3].copy(), o1, o2, 3, k) == rk.STATUS_INVALID_ARGUMENT


def test_q_triple_m1_bit_exact(ctx):
    k = 2048
    ns, kinds = (2048, 256, 256), (4, 6, 4)
    ws = [rk.synth_q_weights(kd, n, k, seed=40 + i) for i, (kd, n) in enumerate(zip(kinds, ns))]
    a = rk.synth_normal(44, k)
    outs = [np.empty(n, np.float32) for n in ns]
    assert ctx.matmul_q_triple_m1(ws[0], kinds[0], ns[0], ws[1], kinds[1], ns[1], ws[2], kinds[2], ns[2], a,
                                  *outs, k) == 0
    for o, w, kd, n in zip(outs, ws, kinds, ns):
        st, ref = oracle.matmul_q(kd, w, a.reshape(1, k), n)
        assert st == 0
        assert np.array_equal(_bits(o), _bits(ref.reshape(-1)))


def test_mtile_release_drops_and_rebuilds(ctx):
    """Releasing Q/K/V drops their single-projection caches and every other
    group containing them, keeps the exact (Q, K, V) group and unrelated
    weights, and a released weight is rebuilt bit-exactly on its next call."""
    m, k = 64, 2048
    q = rk.synth_q_weights(4, 2048, k, seed=51)
    kk = rk.synth_q_weights(4, 256, k, seed=52)
    v = rk.synth_q_weights(6, 256, k, seed=53)
    other = rk.synth_q_weights(4, 2048, k, seed=54)
    a = rk.synth_normal(55, m * k).reshape(m, k)
    refs = {}
    for name, w, kd, n in (("q", q, 4, 2048), ("k", kk, 4, 256), ("v", v, 6, 256), ("o", other, 4, 2048)):
        st, refs[name] = oracle.matmul_q(kd, w, a, n)
        assert st == 0
    out = {name: np.empty((m, r.shape[1]), np.float32) for name, r in refs.items()}
    assert ctx.matmul_q(4, q, a, out["q"], m, k, 2048) == 0
    assert ctx.matmul_q(4, other, a, out["o"], m, k, 2048) == 0
    assert ctx.matmul_q_concat([q, kk, v], [4, 4, 6], [2048, 256, 256], a, [out["q"], out["k"], out["v"]], m, k) == 0
    assert ctx.matmul_q_concat([kk, v], [4, 6], [256, 256], a, [out["k"], out["v"]], m, k) == 0
    s0 = ctx.prompt_cache_stats()
    assert (s0.single_entries, s0.group_entries) == (2, 2)
    assert ctx.mtile_release([q, kk, v]) == 0
    s1 = ctx.prompt_cache_stats()
    # q's single entry and the (k, v) group are gone; the exact group and
    # the unrelated weight stay
    assert (s1.single_entries, s1.group_entries) == (1, 1)
    assert s1.resident_bytes < s0.resident_bytes
    # the kept group is a hit, the released single projection is rebuilt
    assert ctx.matmul_q_concat([q, kk, v], [4, 4, 6], [2048, 256, 256], a, [out["q"], out["k"], out["v"]], m, k) == 0
    assert ctx.prompt_cache_stats().hits == s1.hits + 1
    assert ctx.matmul_q(4, q, a, out["q"], m, k, 2048) == 0
    s2 = ctx.prompt_cache_stats()
    assert s2.misses == s1.misses + 1 and s2.single_entries == 2
    assert ctx.matmul_q(4, other, a, out["o"], m, k, 2048) == 0
    assert ctx.prompt_cache_stats().hits == s2.hits + 1
    for name in ("q", "k", "v", "o"):
        assert np.array_equal(_bits(out[name]), _bits(refs[name])), name
    assert ctx.mtile_release([]) == rk.STATUS_INVALID_ARGUMENT


@pytest.mark.parametrize("kind,k,n", [(4, 2048, 2048), (6, 2048, 256), (4, 5632, 2048)])
def test_prewarm_then_hit(ctx, kind, k, n):
    w = rk.synth_q_weights(kind, n, k, seed=60 + n)
    before = ctx.prompt_cache_stats()
    assert ctx.prewarm_quantized_m16(w, kind, k, n) == 0
    s = ctx.prompt_cache_stats()
    assert s.single_entries == before.single_entries + 1 and s.misses == before.misses
    assert ctx.prewarm_quantized_m16(w, kind, k, n) == 0  # already resident: no second copy
    assert ctx.prompt_cache_stats().single_entries == s.single_entries
    a = rk.synth_normal(61, 16 * k).reshape(16, k)
    out = np.empty((16, n), np.float32)
    assert ctx.matmul_q(kind, w, a, out, 16, k, n) == 0
    s2 = ctx.prompt_cache_stats()
    assert s2.hits == s.hits + 1 and s2.misses == s.misses
    st, ref = oracle.matmul_q(kind, w, a, n)
    assert st == 0 and np.array_equal(_bits(out), _bits(ref))


def test_prewarm_other_shapes_are_a_no_op(ctx):
    w = rk.synth_q_weights(4, 512, 1024, seed=70)
    assert ctx.prewarm_quantized_m16(w, 4, 1024, 512) == 0
    assert ctx.prompt_cache_stats().single_entries == 0


def test_overlap_callback_runs_once_per_m1_call(ctx, rng):
    k, n = 2048, 256
    w, s = _w8(rng, n, k)
    w2, s2 = _w8(rng, n, k)
    a = rng.standard_normal(k).astype(np.float32)
    calls = []
    o = np.empty(n, np.float32)
    assert ctx.set_overlap(lambda: calls.append("a")) == 0
    # a prompt (M > 1) call does not consume the one-shot callback
    a16 = rng.standard_normal((16, k)).astype(np.float32)
    o16 = np.empty((16, n), np.float32)
    assert ctx.matmul_w8a8_m16(w, s, a16, o16, k, n) == 0
    assert calls == []
    assert ctx.matmul_w8a8_m1(w, s, a, o, k, n) == 0
    assert calls == ["a"]
    assert ctx.matmul_w8a8_m1(w, s, a, o, k, n) == 0  # one-shot: cleared after running
    assert calls == ["a"]
    assert np.array_equal(_bits(o), _bits(_m1(w, s, a)))
    assert ctx.set_overlap(lambda: calls.append("b")) == 0
    o1, o2 = np.empty(n, np.float32), np.empty(n, np.float32)
    assert ctx.matmul_w8a8_pair_m1(w, s, n, w2, s2, n, a, o1, o2, k) == 0
    assert calls == ["a", "b"]
    assert ctx.set_overlap(lambda: calls.append("c")) == 0
    assert ctx.set_overlap(None) == 0  # cleared before any call
    assert ctx.matmul_w8a8_m1(w, s, a, o, k, n) == 0
    assert calls == ["a", "b"]
    assert np.array_equal(_bits(o1), _bits(_m1(w, s, a))) and np.array_equal(_bits(o2), _bits(_m1(w2, s2, a)))
