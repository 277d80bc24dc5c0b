"""GPU parity: the sm_100a kernels and the C ABI against the CPU oracle.

Bit-exact for int8 weights/activations, int32 accumulators and (because the
rescale is evaluated in the reference's order with the same IEEE operations)
the f32 W8A8 outputs; the FP16 executor within rtol 1e-3 of the f64 oracle.
"""
import numpy as np
import pytest

import oracle
import rocknpu_b200 as rk
from conftest import random_kquant_blocks

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def dev():
    from rocknpu_b200 import device
    return device


@pytest.fixture
def ctx():
    # one context per test: resident weights are cached by the host address
    # of their bytes (the reference's DecodeWeightKey contract: weights stay
    # alive and unchanged for the context's lifetime), and a test's freed
    # arrays can hand their addresses to the next test's weights
    rk.apply_default_env()
    c = rk.Context()
    yield c
    c.close()


# ---- K1: weight preparation ---------------------------------------------------

@pytest.mark.parametrize("kind", [4, 5, 6])
@pytest.mark.parametrize("k,n", [(256, 8), (2048, 64), (5632, 33), (12288, 4)])
def test_prepare_w8_bit_exact(dev, rng, kind, k, n):
    blocks = random_kquant_blocks(kind, n * k // 256, rng)
    st, w_ref, s_ref = oracle.prepare_w8a8(kind, blocks, k, n)
    assert st == 0
    status = dev.new_status()
    w, s = dev.prepare_w8(kind, torch.from_numpy(blocks).cuda(), k, n, status)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert np.array_equal(w.cpu().numpy(), w_ref)
    assert np.array_equal(_bits(s.cpu().numpy()), _bits(s_ref))


def test_prepare_golden_sidecar(dev):
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "w8_sidecar.npz"))
    for kind in (4, 5, 6):
        n, k = (int(v) for v in g[f"q{kind}_shape"])
        status = dev.new_status()
        w, s = dev.prepare_w8(kind, torch.from_numpy(g[f"q{kind}_blocks"]).cuda(), k, n, status)
        torch.cuda.synchronize()
        assert status.item() == 0
        assert np.array_equal(w.cpu().numpy(), g[f"q{kind}_w8"])
        assert np.array_equal(_bits(s.cpu().numpy()), _bits(g[f"q{kind}_scale"]))


@pytest.mark.parametrize("k,n", [(2048, 24), (24576, 6)])
def test_prepare_q4k_edge_blocks_bit_exact(dev, rng, k, n):
    """Q4_K preparation (one thread per sub-block, a 16-entry table per
    sub-block, absmax from the smallest and largest code) against the oracle
    on blocks where that could go wrong: one code repeated over a sub-block,
    only codes 0 and 15, negative d and dmin, all-zero rows; k = 24576 takes
    three passes per row.  The same blocks 4 bytes past a 16-byte boundary
    take the other kernel (which needs 4-byte alignment only) and must give
    the same bytes."""
    nb = k // 256
    blocks = random_kquant_blocks(4, n * nb, rng).reshape(n, nb, 144)
    half = lambda v: np.array([v], dtype=np.float16).view(np.uint8)
    for r in range(n):
        for b in range(nb):
            mode = (r + b) % 4
            if mode == 0:  # every sub-block one repeated code
                for c in range(4):
                    blocks[r, b, 16 + 32 * c:48 + 32 * c] = rng.integers(0, 16) * 17
            elif mode == 1:  # only the extreme codes
                blocks[r, b, 16:] = rng.choice([0x00, 0x0F, 0xF0, 0xFF], size=128)
            elif mode == 2:  # negative scales
                blocks[r, b, 0:2] = half(-rng.uniform(1e-3, 2e-2))
                blocks[r, b, 2:4] = half(-rng.uniform(1e-3, 2e-2))
    blocks[n - 1] = 0  # an all-zero row: scale 1.0
    blocks = np.ascontiguousarray(blocks.reshape(-1))
    st, w_ref, s_ref = oracle.prepare_w8a8(4, blocks, k, n)
    assert st == 0
    status = dev.new_status()
    w, s = dev.prepare_w8(4, torch.from_numpy(blocks).cuda(), k, n, status)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert np.array_equal(w.cpu().numpy(), w_ref)
    assert np.array_equal(_bits(s.cpu().numpy()), _bits(s_ref))
    shifted = torch.zeros(blocks.size + 16, dtype=torch.uint8, device="cuda")
    shifted[4:4 + blocks.size] = torch.from_numpy(blocks).cuda()
    assert shifted[4:].data_ptr() % 16 == 4
    w2, s2 = dev.prepare_w8(4, shifted[4:4 + blocks.size], k, n, status)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert np.array_equal(w2.cpu().numpy(), w_ref) and np.array_equal(_bits(s2.cpu().numpy()), _bits(s_ref))


def test_prepare_flags_non_finite(dev):
    blk = np.zeros(144, dtype=np.uint8)
    blk[0:2] = np.array([np.inf], dtype=np.float16).view(np.uint8)
    blk[4] = 1
    status = dev.new_status()
    dev.prepare_w8(4, torch.from_numpy(blk).cuda(), 256, 1, status)
    torch.cuda.synchronize()
    assert status.item() == 1


# ---- K2: activation quantisation ----------------------------------------------

@pytest.mark.parametrize("m,k", [(1, 2048), (7, 512), (128, 2048), (33, 5632), (3, 8192), (2, 100)])
def test_quantize_rows_bit_exact(dev, rng, m, k):
    a = (rng.standard_normal((m, k)) * rng.uniform(0.01, 50, size=(m, 1))).astype(np.float32)
    if m > 2:
        a[1] = 0.0
    st, q_ref, s_ref = oracle.quantize_rows(a)
    status = dev.new_status()
    q, s = dev.quantize_rows(torch.from_numpy(a).cuda(), status)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(_bits(s.cpu().numpy()), _bits(s_ref))


def test_quantize_tie_vector(dev):
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "act_quant.npz"))
    v = g["ties"]
    v = np.concatenate([v, np.zeros((-v.size) % 16, dtype=np.float32)]).reshape(1, -1)
    status = dev.new_status()
    q, s = dev.quantize_rows(torch.from_numpy(v).cuda(), status)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy()[0, :g["ties"].size], g["ties_q"])
    assert _bits(s.cpu().numpy())[0] == _bits(g["ties_scale"])[0]


def test_quantize_flags_non_finite(dev):
    a = np.ones((4, 256), dtype=np.float32)
    a[2, 100] = np.nan
    status = dev.new_status()
    dev.quantize_rows(torch.from_numpy(a).cuda(), status)
    torch.cuda.synchronize()
    assert status.item() == 1


# ---- K3: W8A8 GEMM (int32 exact) ------------------------------------------------

GEMM_SHAPES = [
    (128, 2048, 5632),
    (1, 512, 128), (5, 256, 96), (16, 2048, 256), (17, 1024, 200), (64, 768, 384),
    (100, 4096, 128), (129, 512, 160), (300, 1024, 640), (512, 2048, 2560), (256, 5632, 2048),
]


@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("m,k,n", GEMM_SHAPES)
def test_gemm_w8a8_int32_exact(dev, rng, m, k, n, split):
    a8 = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    w8 = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    a_s = rng.uniform(0.001, 0.1, size=m).astype(np.float32)
    w_s = rng.uniform(0.001, 0.1, size=n).astype(np.float32)
    acc_ref = oracle.gemm_i8_i32(a8, w8)
    exp = np.empty((m, n), dtype=np.float32)
    for r in range(m):
        oracle.lib().orc_rescale_i32_row(oracle._p(np.ascontiguousarray(acc_ref[r])), oracle._p(w_s),
                                         float(a_s[r]), oracle._p(exp[r]), n)
    ws = dev.new_workspace(dev.workspace_bytes(m, n, k)) if split else None
    ta8, tas, tw8, tws = (torch.from_numpy(x).cuda() for x in (a8, a_s, w8, w_s))
    for _ in range(2 if split else 1):  # a split-K workspace is left zero for the next launch
        status = dev.new_status()
        acc = torch.empty((m, n), dtype=torch.int32, device="cuda")
        out = dev.gemm_w8a8(ta8, tas, tw8, tws, status, acc=acc, workspace=ws)
        torch.cuda.synchronize()
        assert status.item() == 0
        assert np.array_equal(acc.cpu().numpy(), acc_ref)
        assert np.array_equal(_bits(out.cpu().numpy()), _bits(exp))
    if split:
        assert not ws.any().item()


@pytest.mark.parametrize("wt,bt", [(128, 256), (256, 128), (128, 128), (256, 64), (128, 16), (256, 16)])
@pytest.mark.parametrize("m,k,n", [(300, 1024, 640), (512, 2048, 2560), (257, 384, 300), (1000, 640, 1024)])
def test_gemm_every_tile_configuration_exact(dev, rng, monkeypatch, wt, bt, m, k, n):
    """The tile plan is a heuristic; every instantiated configuration (forced
    through the tuning overrides) must give the same bits, with ragged M, N
    and K edges."""
    monkeypatch.setenv("ROCKNPU_B200_GEMM_WT", str(wt))
    monkeypatch.setenv("ROCKNPU_B200_GEMM_BT", str(bt))
    a8 = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    w8 = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    a_s = rng.uniform(0.001, 0.1, size=m).astype(np.float32)
    w_s = rng.uniform(0.001, 0.1, size=n).astype(np.float32)
    acc_ref = oracle.gemm_i8_i32(a8, w8)
    status = dev.new_status()
    ta8, tas, tw8, tws = (torch.from_numpy(x).cuda() for x in (a8, a_s, w8, w_s))
    for _ in range(2):  # two launches: units reuse the accumulator buffers
        acc = torch.full((m, n), -7, dtype=torch.int32, device="cuda")
        out = dev.gemm_w8a8(ta8, tas, tw8, tws, status, acc=acc)
        torch.cuda.synchronize()
        assert status.item() == 0
        assert np.array_equal(acc.cpu().numpy(), acc_ref)
    exp = np.empty((m, n), dtype=np.float32)
    for r in range(m):
        oracle.lib().orc_rescale_i32_row(oracle._p(np.ascontiguousarray(acc_ref[r])), oracle._p(w_s),
                                         float(a_s[r]), oracle._p(exp[r]), n)
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(exp))


PAIR_SHAPES = [(300, 1024, 640), (512, 2048, 2560), (257, 384, 300), (1000, 640, 1024), (64, 2048, 256),
               (33, 256, 2304), (2048, 512, 4096), (200, 112, 1000)]


@pytest.mark.parametrize("bt", [128, 256])
@pytest.mark.parametrize("m,k,n", PAIR_SHAPES)
def test_gemm_pair_tiles_exact(dev, rng, monkeypatch, bt, m, k, n):
    """Two-SM (cta_group::2) 256 x bt tiles, forced: the same bits as the
    oracle with ragged M, N and K edges, token halves that fall past M, and
    several units per pair (accumulator buffers reused across units and
    launches)."""
    monkeypatch.setenv("ROCKNPU_B200_GEMM_PAIR", "1")
    monkeypatch.setenv("ROCKNPU_B200_GEMM_BT", str(bt))
    a8 = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    w8 = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    a_s = rng.uniform(0.001, 0.1, size=m).astype(np.float32)
    w_s = rng.uniform(0.001, 0.1, size=n).astype(np.float32)
    acc_ref = oracle.gemm_i8_i32(a8, w8)
    status = dev.new_status()
    ta8, tas, tw8, tws = (torch.from_numpy(x).cuda() for x in (a8, a_s, w8, w_s))
    for _ in range(2):
        acc = torch.full((m, n), -7, dtype=torch.int32, device="cuda")
        out = dev.gemm_w8a8(ta8, tas, tw8, tws, status, acc=acc)
        torch.cuda.synchronize()
        assert status.item() == 0
        assert np.array_equal(acc.cpu().numpy(), acc_ref)
    exp = np.empty((m, n), dtype=np.float32)
    for r in range(m):
        oracle.lib().orc_rescale_i32_row(oracle._p(np.ascontiguousarray(acc_ref[r])), oracle._p(w_s),
                                         float(a_s[r]), oracle._p(exp[r]), n)
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(exp))


@pytest.mark.parametrize("bt", [128, 256])
@pytest.mark.parametrize("m,k,n", [(300, 1024, 640), (1000, 2048, 1536), (77, 512, 300)])
def test_gemm_f16_pair_tiles(dev, rng, monkeypatch, bt, m, k, n):
    a = rng.standard_normal((m, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float16)
    ta, tw = torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda()
    status = dev.new_status()
    monkeypatch.setenv("ROCKNPU_B200_GEMM_PAIR", "0")
    one_sm = dev.gemm_f16(ta, tw, status)
    monkeypatch.setenv("ROCKNPU_B200_GEMM_PAIR", "1")
    monkeypatch.setenv("ROCKNPU_B200_GEMM_BT", str(bt))
    pair = dev.gemm_f16(ta, tw, status)
    torch.cuda.synchronize()
    assert status.item() == 0
    ref = oracle.matmul_f16(w.view(np.uint16), a.astype(np.float32))
    got = pair.cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-3, atol=1e-3 * np.abs(ref).max())
    # the same f32 tensor-core accumulation as the one-SM tiles
    assert np.array_equal(_bits(got), _bits(one_sm.cpu().numpy()))


def test_pair_tiles_concat_group(ctx, rng, monkeypatch):
    monkeypatch.setenv("ROCKNPU_B200_GEMM_PAIR", "1")
    m, k = 320, 2048
    ns, kinds = [2048, 256, 256], [4, 4, 6]
    ws = [rk.synth_q_weights(kd, n, k, seed=80 + i) for i, (kd, n) in enumerate(zip(kinds, ns))]
    a = rng.standard_normal((m, k)).astype(np.float32)
    outs = [np.full((m, n), np.nan, dtype=np.float32) for n in ns]
    c = rk.Context()  # its own weight cache
    try:
        assert c.matmul_q_concat(ws, kinds, ns, a, outs, m, k) == 0
    finally:
        c.close()
    for w, kd, n, o in zip(ws, kinds, ns, outs):
        st, ref = oracle.matmul_q(kd, w, a, n)
        assert np.array_equal(_bits(o), _bits(ref))


@pytest.mark.parametrize("m", [4, 8, 12, 16, 32, 48, 64, 128])
def test_gemm_mtile_kat(dev, m):
    # crates/rocket-smoke/src/bin/int8_mtile.rs:28-86
    K, N = 2048, 2048
    a8 = np.repeat(((np.arange(m) % 5) + 1).astype(np.int8)[:, None], K, axis=1)
    w8 = np.ones((N, K), dtype=np.int8)
    status = dev.new_status()
    acc = torch.empty((m, N), dtype=torch.int32, device="cuda")
    dev.gemm_w8a8(torch.from_numpy(a8).cuda(), torch.ones(m, device="cuda"), torch.from_numpy(w8).cuda(),
                  torch.ones(N, device="cuda"), status, acc=acc)
    torch.cuda.synchronize()
    assert np.all(acc.cpu().numpy() == (K * ((np.arange(m) % 5) + 1))[:, None])


def test_gemm_ksplit_kat(dev):
    # crates/rocket-smoke/src/bin/int8_mtile_ksplit.rs:20-33
    M, K, n = 16, 5632, 2048
    r, kk = np.meshgrid(np.arange(M), np.arange(K), indexing="ij")
    a8 = (((r * 7 + kk * 3 + 5) % 13) - 6).astype(np.int8)
    c_, kk2 = np.meshgrid(np.arange(n), np.arange(K), indexing="ij")
    w8 = (((c_ * 5 + kk2 * 11 + 3) % 17) - 8).astype(np.int8)
    status = dev.new_status()
    acc = torch.empty((M, n), dtype=torch.int32, device="cuda")
    dev.gemm_w8a8(torch.from_numpy(a8).cuda(), torch.ones(M, device="cuda"), torch.from_numpy(w8).cuda(),
                  torch.ones(n, device="cuda"), status, acc=acc)
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), oracle.gemm_i8_i32(a8, w8))


# ---- K5: M=1 GEMV ---------------------------------------------------------------

def test_gemv_decode_m1_kat(dev):
    # crates/rocket-smoke/src/bin/int8_decode_m1.rs:35-45
    k, n = 2048, 2048
    a8 = (((np.arange(k) * 7 + 3) % 9) - 4).astype(np.int8)
    w8 = (((np.arange(n * k) * 5 + 1) % 11) - 5).astype(np.int8).reshape(n, k)
    out = dev.gemv_w8a8(torch.from_numpy(a8).cuda(), torch.ones(1, device="cuda"), torch.from_numpy(w8).cuda(),
                        torch.ones(n, device="cuda"))
    torch.cuda.synchronize()
    ref = (w8.astype(np.int64) @ a8.astype(np.int64)).astype(np.float32)
    assert np.array_equal(out.cpu().numpy(), ref)


# ---- C ABI end to end --------------------------------------------------------------

@pytest.mark.parametrize("kind", [4, 6])
@pytest.mark.parametrize("m,k,n", [(128, 2048, 5632), (1, 2048, 256), (5, 512, 64), (16, 2048, 2048),
                                   (300, 2048, 96), (77, 5632, 256), (8, 2304, 128), (1000, 2048, 640)])
def test_capi_matmul_q_bit_exact(ctx, rng, kind, m, k, n):
    blocks = rk.synth_q_weights(kind, n, k, seed=11 + m)
    a = rng.standard_normal((m, k)).astype(np.float32)
    out = np.full((m, n), np.nan, dtype=np.float32)
    assert ctx.matmul_q(kind, blocks, a, out, m, k, n) == 0
    st, ref = oracle.matmul_q(kind, blocks, a, n)
    assert st == 0
    assert np.array_equal(_bits(out), _bits(ref))
    # second call hits the resident weight cache
    out2 = np.zeros_like(out)
    assert ctx.matmul_q(kind, blocks, a, out2, m, k, n) == 0
    assert np.array_equal(_bits(out2), _bits(ref))


def test_capi_q5_prompt(ctx, rng):
    m, k, n = 32, 1024, 96
    blocks = rk.synth_q_weights(5, n, k, seed=5)
    a = rng.standard_normal((m, k)).astype(np.float32)
    out = np.empty((m, n), dtype=np.float32)
    assert ctx.matmul_q(5, blocks, a, out, m, k, n) == 0
    st, ref = oracle.matmul_q(5, blocks, a, n)
    assert np.array_equal(_bits(out), _bits(ref))
    assert ctx.matmul_q(5, blocks, a[:1], out[:1], 1, k, n) == -1  # Q5_K has no M=1 route


def test_capi_fp16_route_for_unaligned_n(ctx, rng):
    # n % 32 != 0: no W8A8 branch accepts it, the FP16 route runs
    m, k, n = 8, 512, 48
    blocks = rk.synth_q_weights(4, n, k, seed=3)
    a = rng.standard_normal((m, k)).astype(np.float32)
    out = np.empty((m, n), dtype=np.float32)
    assert ctx.matmul_q(4, blocks, a, out, m, k, n) == 0
    w16 = oracle.dequant(4, blocks).astype(np.float16).reshape(n, k)
    ref = oracle.matmul_f16(w16.view(np.uint16), a)
    np.testing.assert_allclose(out, ref, rtol=1e-3, atol=1e-3 * np.abs(ref).max())


def test_capi_rejects_non_finite(ctx, rng):
    m, k, n = 4, 512, 64
    blocks = rk.synth_q_weights(4, n, k, seed=4)
    a = rng.standard_normal((m, k)).astype(np.float32)
    a[2, 3] = np.inf
    out = np.zeros((m, n), dtype=np.float32)
    assert ctx.matmul_q(4, blocks, a, out, m, k, n) == -1
    assert not out.any()  # output untouched on error
    a[2, 3] = 0.0
    assert ctx.matmul_q(4, blocks, a, out, m, k, n) == 0  # context still usable


def test_capi_rejects_bad_sizes(ctx, rng):
    blocks = rk.synth_q_weights(4, 64, 512, seed=4)
    a = np.zeros((4, 512), dtype=np.float32)
    out = np.zeros((4, 64), dtype=np.float32)
    assert ctx.matmul_q(4, blocks, a, out, 4, 512, 64, weights_bytes=blocks.nbytes - 1) == -1
    assert ctx.matmul_q(4, blocks, a, out, 4, 500, 64) == -1
    assert ctx.matmul_q(4, blocks, a, out, 0, 512, 64) == -1
    # M=1 limits of execute_cached_w8a8_m1
    assert ctx.matmul_q(4, rk.synth_q_weights(4, 64, 256, 1), a[:1, :256].copy(), out[:1], 1, 256, 64) == -1


def test_capi_concat_group_equals_separate(ctx, rng):
    m, k = 64, 2048
    ns, kinds = [2048, 256, 256], [4, 4, 6]
    ws = [rk.synth_q_weights(kd, n, k, seed=20 + i) for i, (kd, n) in enumerate(zip(kinds, ns))]
    a = rng.standard_normal((m, k)).astype(np.float32)
    outs = [np.empty((m, n), dtype=np.float32) for n in ns]
    assert ctx.matmul_q_concat(ws, kinds, ns, a, outs, m, k) == 0
    for w, kd, n, o in zip(ws, kinds, ns, outs):
        st, ref = oracle.matmul_q(kd, w, a, n)
        assert np.array_equal(_bits(o), _bits(ref))


def test_capi_f16_executor(ctx, rng):
    m, k, n = 33, 1000, 80
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float16)
    a = rng.standard_normal((m, k)).astype(np.float32)
    out = np.empty((m, n), dtype=np.float32)
    assert ctx.matmul_f16(w.view(np.uint16), a, out, m, k, n) == 0
    ref = oracle.matmul_f16(w.view(np.uint16), a)
    np.testing.assert_allclose(out, ref, rtol=1e-3, atol=1e-3 * np.abs(ref).max())


def test_capi_w8a8_m1_pair_triple(ctx, rng):
    k = 2048
    ns = [2048, 256, 256]
    ws = [rng.integers(-127, 128, size=(n, k), dtype=np.int8) for n in ns]
    ss = [rng.uniform(0.001, 0.01, size=n).astype(np.float32) for n in ns]
    a = rng.standard_normal(k).astype(np.float32)
    refs = [oracle.matmul_w8a8(w, s, a.reshape(1, k))[1].reshape(-1) for w, s in zip(ws, ss)]
    before = ctx.decode_cache_stats()
    o = np.empty(ns[0], dtype=np.float32)
    assert ctx.matmul_w8a8_m1(ws[0], ss[0], a, o, k, ns[0]) == 0
    assert np.array_equal(_bits(o), _bits(refs[0]))
    o1, o2 = np.empty(ns[0], np.float32), np.empty(ns[1], np.float32)
    assert ctx.matmul_w8a8_pair_m1(ws[0], ss[0], ns[0], ws[1], ss[1], ns[1], a, o1, o2, k) == 0
    assert np.array_equal(_bits(o1), _bits(refs[0])) and np.array_equal(_bits(o2), _bits(refs[1]))
    t = [np.empty(n, np.float32) for n in ns]
    assert ctx.matmul_w8a8_triple_m1(ws[0], ss[0], ns[0], ws[1], ss[1], ns[1], ws[2], ss[2], ns[2], a, *t, k) == 0
    for x, r in zip(t, refs):
        assert np.array_equal(_bits(x), _bits(r))
    st = ctx.decode_cache_stats()
    assert st.entries - before.entries == 3 and st.misses - before.misses == 3
    assert ctx.matmul_w8a8_m1(ws[0], ss[0], a, o, k, ns[0]) == 0
    assert ctx.decode_cache_stats().hits == st.hits + 1


def test_capi_w8a8_m16(ctx, rng):
    k, n = 2048, 512
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    s = rng.uniform(0.001, 0.01, size=n).astype(np.float32)
    a = rng.standard_normal((16, k)).astype(np.float32)
    out = np.empty((16, n), dtype=np.float32)
    assert ctx.matmul_w8a8_m16(w, s, a, out, k, n) == 0
    assert np.array_equal(_bits(out), _bits(oracle.matmul_w8a8(w, s, a)[1]))


# ---- K2 fused into K3's prologue --------------------------------------------------

@pytest.mark.parametrize("m,k,n", [(2, 112, 64), (77, 304, 200), (128, 2048, 5632), (512, 2048, 2560),
                                   (600, 5632, 128), (1000, 1024, 1024), (16, 12288, 256)])
def test_fused_quantiser_matches_oracle_and_unfused(ctx, rng, monkeypatch, m, k, n):
    from rocknpu_b200 import device
    a = rng.standard_normal((m, k)).astype(np.float32)
    a[:, rng.choice(k, max(1, k // 100), replace=False)] *= 20.0  # outlier channels
    a[m // 2] = 0.0  # an all-zero token: scale 1.0
    w8 = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    ws = rng.uniform(1e-3, 1e-2, size=n).astype(np.float32)
    st, ref = oracle.matmul_w8a8(w8, ws, a)
    assert st == 0
    da, dw, dws = torch.from_numpy(a).cuda(), torch.from_numpy(w8).cuda(), torch.from_numpy(ws).cuda()
    outs = {}
    for fused in ("1", "0"):
        monkeypatch.setenv("ROCKNPU_B200_FUSED_QUANT", fused)
        for rep in range(2):  # the second launch reuses the self-cleared counters
            out = torch.full((m, n), float("nan"), device="cuda")
            device.matmul_w8a8(ctx, da, dw, dws, out)
            assert rk.lib().rocknpu_b200_context_check(ctx.handle) == 0
            outs[(fused, rep)] = out.cpu().numpy()
    for key, got in outs.items():
        assert np.array_equal(_bits(got), _bits(ref)), f"fused={key[0]} launch {key[1]} differs from the oracle"


def test_fused_quantiser_flags_non_finite(ctx, rng, monkeypatch):
    from rocknpu_b200 import device
    monkeypatch.setenv("ROCKNPU_B200_FUSED_QUANT", "1")
    m, k, n = 40, 512, 128
    a = rng.standard_normal((m, k)).astype(np.float32)
    a[17, 300] = np.nan
    w8 = torch.ones((n, k), dtype=torch.int8, device="cuda")
    ws = torch.ones(n, device="cuda")
    out = torch.empty((m, n), device="cuda")
    device.matmul_w8a8(ctx, torch.from_numpy(a).cuda(), w8, ws, out)
    assert rk.lib().rocknpu_b200_context_check(ctx.handle) == rk.STATUS_INVALID_ARGUMENT
    a[17, 300] = 1.0
    device.matmul_w8a8(ctx, torch.from_numpy(a).cuda(), w8, ws, out)  # counters were left clean
    assert rk.lib().rocknpu_b200_context_check(ctx.handle) == 0


def _near_half_rows(rng, m, k):
    """Rows whose quotients x / scale sit within a few ulps of half-integers
    (and on them), where a reciprocal multiply would round differently from
    the IEEE quotient: scale = 127-multiple absmax / 127 fixed by one entry."""
    rows = []
    for i in range(m):
        s0 = np.float32(rng.uniform(0.01, 3.0))
        row = np.empty(k, dtype=np.float32)
        row[0] = np.float32(127.0) * s0
        j = rng.integers(-127, 127, size=k - 1).astype(np.float32) + np.float32(0.5)
        x = (j * s0).astype(np.float32)
        steps = rng.integers(-3, 4, size=k - 1)
        for d in range(1, 4):  # nudge by up to 3 ulps either way
            x = np.where(steps >= d, np.nextafter(x, np.float32(np.inf)), x)
            x = np.where(steps <= -d, np.nextafter(x, np.float32(-np.inf)), x)
        row[1:] = x
        rows.append(row)
    return np.stack(rows)


def test_quantisers_round_like_the_ieee_quotient_near_half_integers(ctx, rng, monkeypatch, dev):
    m, k, n = 64, 2048, 128
    a = _near_half_rows(rng, m, k)
    st, q_ref, s_ref = oracle.quantize_rows(a)
    assert st == 0
    status = dev.new_status()
    q, s = dev.quantize_rows(torch.from_numpy(a).cuda(), status)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert np.array_equal(q.cpu().numpy(), q_ref) and np.array_equal(_bits(s.cpu().numpy()), _bits(s_ref))
    # the fused prologue quantiser: checked through the W8A8 output
    w8 = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    ws = rng.uniform(1e-3, 1e-2, size=n).astype(np.float32)
    st, ref = oracle.matmul_w8a8(w8, ws, a)
    monkeypatch.setenv("ROCKNPU_B200_FUSED_QUANT", "1")
    out = torch.empty((m, n), device="cuda")
    dev.matmul_w8a8(ctx, torch.from_numpy(a).cuda(), torch.from_numpy(w8).cuda(), torch.from_numpy(ws).cuda(), out)
    assert rk.lib().rocknpu_b200_context_check(ctx.handle) == 0
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(ref))


@pytest.mark.parametrize("case", ["normal", "outliers", "zero", "near_half", "subnormal"])
@pytest.mark.parametrize("k,n", [(2048, 2048), (5632, 256), (512, 32), (16384, 72)])
def test_gemv_fused_quant_m1_bit_exact(ctx, dev, rng, case, k, n):
    """M=1 through the context's device entry: the quantiser runs inside the
    GEMV (one launch), with the row quantiser's bits."""
    if case == "near_half":
        x = _near_half_rows(rng, 1, k)[0]
    elif case == "zero":
        x = np.zeros(k, np.float32)
    elif case == "subnormal":
        x = (rng.standard_normal(k) * 1e-39).astype(np.float32)
    else:
        x = rng.standard_normal(k).astype(np.float32)
        if case == "outliers":
            x[rng.choice(k, max(1, k // 100), replace=False)] *= 20.0
    w8 = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    ws = rng.uniform(1e-3, 1e-2, size=n).astype(np.float32)
    st, ref = oracle.matmul_w8a8(w8, ws, x.reshape(1, k))
    assert st == 0
    out = torch.full((1, n), float("nan"), device="cuda")
    dev.matmul_w8a8(ctx, torch.from_numpy(x.reshape(1, k)).cuda(), torch.from_numpy(w8).cuda(),
                    torch.from_numpy(ws).cuda(), out)
    assert rk.lib().rocknpu_b200_context_check(ctx.handle) == 0
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(ref))


def test_gemv_fused_quant_m1_flags_non_finite(ctx, dev, rng):
    k, n = 2048, 64
    w8 = torch.from_numpy(rng.integers(-127, 128, size=(n, k), dtype=np.int8)).cuda()
    ws = torch.from_numpy(rng.uniform(1e-3, 1e-2, size=n).astype(np.float32)).cuda()
    x = rng.standard_normal((1, k)).astype(np.float32)
    x[0, 1234] = np.nan
    out = torch.empty((1, n), device="cuda")
    dev.matmul_w8a8(ctx, torch.from_numpy(x).cuda(), w8, ws, out)
    assert rk.lib().rocknpu_b200_context_check(ctx.handle) == rk.STATUS_INVALID_ARGUMENT
    x[0, 1234] = 0.5
    dev.matmul_w8a8(ctx, torch.from_numpy(x).cuda(), w8, ws, out)
    assert rk.lib().rocknpu_b200_context_check(ctx.handle) == 0


# ---- HILO two-part activations (ROCKNPU_PREFILL_HILO) -------------------------

def _prepared(kind, blocks, k, n):
    st, w8, ws = oracle.prepare_w8a8(kind, blocks, k, n)
    assert st == 0
    return w8, ws


@pytest.mark.parametrize("mode,kind,m,k,n", [("1", 4, 64, 2048, 512), ("all", 6, 33, 2048, 256),
                                             ("down", 4, 16, 5632, 256), ("1", 4, 200, 2048, 2048)])
def test_hilo_prompt_matches_oracle(ctx, rng, monkeypatch, mode, kind, m, k, n):
    monkeypatch.setenv("ROCKNPU_PREFILL_HILO", mode)
    blocks = rk.synth_q_weights(kind, n, k, seed=m + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    a[:, rng.choice(k, 20, replace=False)] *= 25.0
    out = np.full((m, n), np.nan, dtype=np.float32)
    assert ctx.matmul_q(kind, blocks, a, out, m, k, n) == 0
    w8, ws = _prepared(kind, blocks, k, n)
    st, ref = oracle.matmul_w8a8_hilo(w8, ws, a)
    assert st == 0
    assert np.array_equal(_bits(out), _bits(ref))
    # it differs from the one-part encoding and is closer to the f32 product
    st, plain = oracle.matmul_w8a8(w8, ws, a)
    exact = a.astype(np.float64) @ (w8.astype(np.float64) * ws[:, None].astype(np.float64)).T
    assert np.abs(ref - exact).max() < np.abs(plain - exact).max()


def test_hilo_down_mode_leaves_narrow_k_alone(ctx, rng, monkeypatch):
    m, k, n = 32, 2048, 256
    blocks = rk.synth_q_weights(4, n, k, seed=9)
    a = rng.standard_normal((m, k)).astype(np.float32)
    monkeypatch.setenv("ROCKNPU_PREFILL_HILO", "down")
    out = np.empty((m, n), dtype=np.float32)
    assert ctx.matmul_q(4, blocks, a, out, m, k, n) == 0
    w8, ws = _prepared(4, blocks, k, n)
    st, ref = oracle.matmul_w8a8(w8, ws, a)
    assert np.array_equal(_bits(out), _bits(ref))


def test_hilo_concat_group_matches_oracle(ctx, rng, monkeypatch):
    monkeypatch.setenv("ROCKNPU_PREFILL_HILO", "1")
    m, k = 48, 2048
    ns, kinds = [2048, 256, 256], [4, 4, 6]
    ws = [rk.synth_q_weights(kd, n, k, seed=40 + i) for i, (kd, n) in enumerate(zip(kinds, ns))]
    a = rng.standard_normal((m, k)).astype(np.float32)
    outs = [np.full((m, n), np.nan, dtype=np.float32) for n in ns]
    assert ctx.matmul_q_concat(ws, kinds, ns, a, outs, m, k) == 0
    for (kd, n, b, o) in zip(kinds, ns, ws, outs):
        w8, s8 = _prepared(kd, b, k, n)
        st, ref = oracle.matmul_w8a8_hilo(w8, s8, a)
        assert np.array_equal(_bits(o), _bits(ref))


def test_hilo_non_finite_takes_the_normal_path(ctx, rng, monkeypatch):
    monkeypatch.setenv("ROCKNPU_PREFILL_HILO", "1")
    m, k, n = 8, 512, 64
    blocks = rk.synth_q_weights(4, n, k, seed=4)
    a = rng.standard_normal((m, k)).astype(np.float32)
    a[3, 7] = np.nan
    out = np.zeros((m, n), dtype=np.float32)
    assert ctx.matmul_q(4, blocks, a, out, m, k, n) == -1
    assert not out.any()


@pytest.mark.parametrize("m,k,lda", [(3, 100, 100), (64, 2048, 2048), (7, 96, 128)])
def test_convert_f16_rounds_to_nearest_even(dev, rng, m, k, lda):
    a = (rng.standard_normal((m, lda)) * 1000).astype(np.float32)
    a[0, :4] = [65520.0, -65519.0, 5.96e-8, 2.0 ** -25]  # overflow to inf, near-max, subnormal, tie to zero
    ta = torch.from_numpy(a).cuda()[:, :k]
    out = dev.convert_f16(ta)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint16), a[:, :k].astype(np.float16).view(np.uint16))
