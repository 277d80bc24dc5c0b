"""The CPU oracle pinned against golden vectors and the reference's own tests.

Fixtures (tests/golden/, made by make_golden.py):
* kquant_dequant.npz -- gguf-py 0.19.0 dequantisation of random superblocks;
* w8_sidecar.npz -- the reference's own sidecar quantiser
  (scripts/make_tinyllama_w8_sidecar_gguf.py::quantize_rows);
* act_quant.npz -- the reference quantisation test vector
  (crates/rocknpu-capi/src/lib.rs:5680-5700).
"""
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("kind", [4, 5, 6])
def test_dequant_matches_gguf_py_golden(kind):
    g = np.load(os.path.join(GOLDEN, "kquant_dequant.npz"))
    got = oracle.dequant(kind, g[f"q{kind}_blocks"])
    assert np.array_equal(_bits(got), _bits(g[f"q{kind}_dequant"]))


@pytest.mark.parametrize("kind", [4, 5, 6])
def test_w8_prepare_matches_reference_sidecar(kind):
    g = np.load(os.path.join(GOLDEN, "w8_sidecar.npz"))
    n, k = (int(v) for v in g[f"q{kind}_shape"])
    st, w, s = oracle.prepare_w8a8(kind, g[f"q{kind}_blocks"], k, n)
    assert st == 0
    assert np.array_equal(w, g[f"q{kind}_w8"])
    assert np.array_equal(_bits(s), _bits(g[f"q{kind}_scale"]))


def test_activation_quant_tie_vector():
    g = np.load(os.path.join(GOLDEN, "act_quant.npz"))
    q, s = oracle.quantize_symmetric(g["ties"])
    assert np.array_equal(q, g["ties_q"])
    assert _bits(np.array([s]))[0] == _bits(g["ties_scale"])[0]
    st, qr, sr = oracle.quantize_rows(g["rows"])
    assert st == 0
    assert np.array_equal(qr, g["rows_q"])
    assert np.array_equal(_bits(sr), _bits(g["rows_scale"]))
    # all-zero row -> scale 1.0 (capi/src/lib.rs:645)
    assert sr[1] == 1.0 and not qr[1].any()


def test_quantize_rejects_non_finite():
    for bad in (np.nan, np.inf, -np.inf):
        v = np.linspace(-1, 1, 64, dtype=np.float32)
        v[17] = bad
        assert oracle.quantize_symmetric(v) is None
        st, _, _ = oracle.quantize_rows(v.reshape(1, -1))
        assert st == -1


def test_quantize_half_away_from_zero():
    # scale = 127/127 = 1: x/scale is x itself
    v = np.array([127.0, 0.5, -0.5, 1.5, -1.5, 2.5, 0.49999997, -0.49999997], dtype=np.float32)
    q, s = oracle.quantize_symmetric(v)
    assert s == 1.0
    assert q.tolist() == [127, 1, -1, 2, -2, 3, 0, 0]


def test_f16_conversions_round_trip_and_rne():
    bits = np.arange(0, 1 << 16, dtype=np.uint32)
    L = oracle.lib()
    finite = [b for b in range(0, 1 << 16, 37) if (b >> 10) & 0x1F != 0x1F]
    for b in finite:
        f = L.orc_f16_to_f32(b)
        assert np.float16(f).view(np.uint16) == b or (b & 0x7FFF) == 0
        assert L.orc_f32_to_f16(f) == b
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(4000).astype(np.float32) * 100,
                        rng.standard_normal(1000).astype(np.float32) * 1e-6,
                        np.array([65504, 65520, 1e9, -1e9, 6e-8, 3e-8], dtype=np.float32)])
    ours = oracle.f32_to_f16_bits(x)
    assert np.array_equal(ours, x.astype(np.float16).view(np.uint16))
    del bits


def test_prepare_rejects_bad_sizes():
    w = np.zeros(144 * 8, dtype=np.uint8)
    assert oracle.prepare_w8a8(4, w, 2048, 1)[0] == 0
    assert oracle.prepare_w8a8(4, w[:-1], 2048, 1)[0] == -1
    assert oracle.prepare_w8a8(4, w, 2000, 1)[0] == -1


def test_prepare_rejects_non_finite_weights():
    blk = np.zeros(144, dtype=np.uint8)
    blk[0:2] = np.array([np.inf], dtype=np.float16).view(np.uint8)
    blk[4] = 1  # sub-block 0 scale 1 -> d*sc = inf
    st, _, _ = oracle.prepare_w8a8(4, blk, 256, 1)
    assert st == -1


def test_int8_decode_m1_kat():
    # crates/rocket-smoke/src/bin/int8_decode_m1.rs:35-45
    k, n = 2048, 64
    a = (((np.arange(k) * 7 + 3) % 9) - 4).astype(np.int8).reshape(1, k)
    b = (((np.arange(n * k) * 5 + 1) % 11) - 5).astype(np.int8).reshape(n, k)
    c = oracle.gemm_i8_i32(a, b)
    assert np.array_equal(c, a.astype(np.int64) @ b.T.astype(np.int64))


@pytest.mark.parametrize("m", [4, 8, 12, 16, 32, 48, 64, 128])
def test_int8_mtile_kat(m):
    # crates/rocket-smoke/src/bin/int8_mtile.rs:28-86: row r = r%5+1, W = 1
    K, N = 2048, 64
    a = np.repeat(((np.arange(m) % 5) + 1).astype(np.int8)[:, None], K, axis=1)
    w = np.ones((N, K), dtype=np.int8)
    c = oracle.gemm_i8_i32(a, w)
    assert np.all(c == (K * ((np.arange(m) % 5) + 1))[:, None])


def test_int8_ksplit_kat():
    # crates/rocket-smoke/src/bin/int8_mtile_ksplit.rs:20-33
    M, K, n = 16, 5632, 96
    r, kk = np.meshgrid(np.arange(M), np.arange(K), indexing="ij")
    a = (((r * 7 + kk * 3 + 5) % 13) - 6).astype(np.int8)
    c_, kk2 = np.meshgrid(np.arange(n), np.arange(K), indexing="ij")
    b = (((c_ * 5 + kk2 * 11 + 3) % 17) - 8).astype(np.int8)
    c = oracle.gemm_i8_i32(a, b)
    assert np.array_equal(c, a.astype(np.int64) @ b.T.astype(np.int64))


def test_split_geometry_matches_reference_tests():
    # rocknpu-matmul/src/int8_decode_pool.rs:1528-1548
    assert oracle.split_blocks(5632 // 32, 32, 3) == [(0, 1888), (1888, 1888), (3776, 1856)]
    assert oracle.split_blocks(1, 32, 3) == [(0, 32)]
    assert oracle.split_blocks(2, 32, 3) == [(0, 32), (32, 32)]
    assert oracle.split_blocks(5632 // 512, 512, 3) == [(0, 2048), (2048, 2048), (4096, 1536)]


def test_matmul_q_pipeline_consistent(rng):
    from conftest import random_kquant_blocks
    m, k, n = 5, 512, 64
    blocks = random_kquant_blocks(4, n * k // 256, rng)
    a = rng.standard_normal((m, k)).astype(np.float32)
    st, out, acc = oracle.matmul_q(4, blocks, a, n, want_acc=True)
    assert st == 0
    st, w, ws = oracle.prepare_w8a8(4, blocks, k, n)
    st2, a8, as_ = oracle.quantize_rows(a)
    ref_acc = a8.astype(np.int64) @ w.T.astype(np.int64)
    assert np.array_equal(acc, ref_acc)
    exp = (acc.astype(np.float32) * as_[:, None]).astype(np.float32) * ws[None, :]
    assert np.array_equal(_bits(out), _bits(exp.astype(np.float32)))


def test_matmul_f16_oracle_is_f64_exact(rng):
    m, k, n = 3, 96, 7
    w = rng.standard_normal((n, k)).astype(np.float16)
    a = rng.standard_normal((m, k)).astype(np.float32)
    out = oracle.matmul_f16(w.view(np.uint16), a)
    ref = (a.astype(np.float16).astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)
    assert np.allclose(out, ref, rtol=0, atol=1e-6)


def test_hilo_stack_and_sum_restatement():
    """hilo_stack (capi/src/lib.rs:2045-2070): [x; x - f32(q) * scale] with
    q, scale from quantize_symmetric_into, in f32 without contraction; and
    hilo_sum (:2073-2083).  The reference has no test of its own for these,
    so the C oracle is checked against the same operations in numpy f32."""
    rng = np.random.default_rng(5)
    a = rng.standard_normal((9, 768)).astype(np.float32)
    a[:, rng.choice(768, 8, replace=False)] *= 30.0
    a[4] = 0.0
    st, stacked = oracle.hilo_stack(a)
    assert st == 0
    st, q, s = oracle.quantize_rows(a)
    back = (q.astype(np.float32) * s[:, None]).astype(np.float32)
    residual = (a - back).astype(np.float32)
    assert np.array_equal(stacked[:9].view(np.uint32), a.view(np.uint32))
    assert np.array_equal(stacked[9:].view(np.uint32), residual.view(np.uint32))
    halves = rng.standard_normal((2, 5, 7)).astype(np.float32)
    assert np.array_equal(oracle.hilo_sum(halves.reshape(10, 7)), (halves[0] + halves[1]).astype(np.float32))
    bad = a.copy()
    bad[2, 3] = np.inf
    assert oracle.hilo_stack(bad)[0] != 0


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (5, 100, 7), (64, 2048, 256), (17, 8192, 33), (3, 65, 130)])
@pytest.mark.parametrize("path", ["amx", "vnni"])
def test_gemm_fast_path_equals_scalar_loops(monkeypatch, path, m, k, n):
    """The CPU baseline's fast products -- AMX tiles (tdpbssd) and AVX-512 VNNI
    (vpdpbusd with the unsigned-offset trick), each where the CPU has it, else
    the next path down -- are the same exact int32 result as the plain loops
    and as int64 arithmetic."""
    rng = np.random.default_rng(m * 31 + k)
    a = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    monkeypatch.setenv("ORACLE_GEMM_PATH", path)
    fast = oracle.gemm_i8_i32(a, w)
    monkeypatch.setenv("ORACLE_GEMM_PATH", "scalar")
    assert oracle.gemm_path(m, k, n) == "scalar"
    slow = oracle.gemm_i8_i32(a, w)
    assert np.array_equal(fast, slow)
    assert np.array_equal(fast, (a.astype(np.int64) @ w.astype(np.int64).T).astype(np.int32))


@pytest.mark.parametrize("kind", [4, 5, 6])
def test_oracle_synth_equals_library_synth(kind):
    """The reference arm of bench.py builds its inputs with the oracle's own
    generator (so that its process never loads librocknpu.so); the values and
    K-quant block bytes must be the ones the library's generator gives the
    B200 arm.  Sizes span the parallel and the serial split of both."""
    import rocknpu_b200 as rk
    for seed, first, count in ((0, 0, 1), (7, 12345, 4097), (1000, 3 * 2048, 256 * 2048)):
        a = oracle.synth_normal(seed, count, 0.02, first=first)
        b = rk.synth_normal(seed, count, 0.02, first=first)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    for n, k in ((1, 256), (33, 512), (256, 2048)):
        vals = rk.synth_normal(kind * 100 + n, n * k, 0.02).reshape(n, k)
        assert np.array_equal(oracle.synth_encode(kind, vals), rk.synth_encode(kind, vals))
    # wide values (larger scales, clamped codes) and all-zero rows
    wide = rk.synth_normal(99, 64 * 256, 3.0).reshape(64, 256)
    wide[5] = 0.0
    assert np.array_equal(oracle.synth_encode(kind, wide), rk.synth_encode(kind, wide))
    assert np.array_equal(oracle.synth_q_weights(kind, 40, 1024, seed=3), rk.synth_q_weights(kind, 40, 1024, seed=3))
