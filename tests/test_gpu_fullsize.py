"""Parity at the BASELINE.json sizes.

Full-size shapes are too large for the oracle to recompute whole, so each
test checks what the domain makes size-independent:

* cfg5 weight (Q4_K, N=28672 x K=8192): the whole matrix is prepared on the
  GPU; sampled rows are compared with the oracle bit for bit.
* cfg5 GEMM at M=1024: the int32 accumulators of sampled token rows against
  the oracle's exact int32 products, and the whole accumulator matrix through
  the exact linearity of integer dot products: acc(A1) + acc(A2) = acc(A1 + A2)
  for int8 A1, A2 whose sum stays in int8.
* TinyLlama pp512 through the C ABI: the QKV group and the FFN down call of a
  layer at their full shapes against the oracle, bit for bit.
"""
import numpy as np
import pytest

import oracle
import rocknpu_b200 as rk

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

N5, K5 = 28672, 8192


@pytest.fixture(scope="module")
def cfg5_weight():
    from rocknpu_b200 import device as dev
    blocks = rk.synth_q_weights(4, N5, K5, seed=0, sigma=0.02)
    status = dev.new_status()
    w8, ws = dev.prepare_w8(4, torch.from_numpy(blocks).cuda(), K5, N5, status)
    torch.cuda.synchronize()
    assert status.item() == 0
    return blocks, w8, ws


def test_cfg5_preparation_sampled_rows(cfg5_weight):
    blocks, w8, ws = cfg5_weight
    rows = np.random.default_rng(0).choice(N5, 64, replace=False)
    row_bytes = K5 // 256 * 144
    src = blocks.reshape(N5, row_bytes)[rows]
    st, ref_w, ref_s = oracle.prepare_w8a8(4, src.reshape(-1), K5, len(rows))
    assert st == 0
    got_w = w8[torch.from_numpy(rows).cuda()].cpu().numpy()
    got_s = ws[torch.from_numpy(rows).cuda()].cpu().numpy()
    assert np.array_equal(got_w, ref_w)
    assert np.array_equal(got_s.view(np.uint32), ref_s.view(np.uint32))


def test_cfg5_gemm_int32_sampled_rows_and_linearity(cfg5_weight):
    from rocknpu_b200 import device as dev
    _, w8, ws = cfg5_weight
    m = 1024
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    a1 = torch.randint(-63, 64, (m, K5), dtype=torch.int8, device="cuda", generator=g)
    a2 = torch.randint(-63, 64, (m, K5), dtype=torch.int8, device="cuda", generator=g)
    a12 = (a1.to(torch.int16) + a2.to(torch.int16)).to(torch.int8)
    ones = torch.ones(m, device="cuda")
    status = dev.new_status()
    accs = []
    for a in (a1, a2, a12):
        acc = torch.empty((m, N5), dtype=torch.int32, device="cuda")
        dev.gemm_w8a8(a, ones, w8, ws, status, acc=acc)
        accs.append(acc)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert torch.equal(accs[0] + accs[1], accs[2]), "int32 accumulators are not exactly linear"
    rows = [0, 1, 255, 256, 511, 777, 1022, 1023]
    ref = np.empty((len(rows), N5), dtype=np.int32)
    oracle.lib().orc_gemm_i8_i32(oracle._p(np.ascontiguousarray(a1[rows].cpu().numpy())),
                                 oracle._p(np.ascontiguousarray(w8.cpu().numpy())), oracle._p(ref), len(rows), K5, N5)
    assert np.array_equal(accs[0][rows].cpu().numpy(), ref)


@pytest.fixture(scope="module")
def ctx():
    rk.apply_default_env()
    c = rk.Context()
    yield c
    c.close()


def test_tinyllama_pp512_layer_calls_through_the_c_abi(ctx):
    m, k = 512, 2048
    ns, kinds = [2048, 256, 256], [4, 4, 6]
    ws = [rk.synth_q_weights(kd, n, k, seed=60 + i) for i, (kd, n) in enumerate(zip(kinds, ns))]
    a = rk.synth_normal(61, m * k).reshape(m, k)
    outs = [np.full((m, n), np.nan, dtype=np.float32) for n in ns]
    assert ctx.matmul_q_concat(ws, kinds, ns, a, outs, m, k) == 0
    for kd, n, b, o in zip(kinds, ns, ws, outs):
        st, ref = oracle.matmul_q(kd, b, a, n)
        assert st == 0
        assert np.array_equal(o.view(np.uint32), ref.view(np.uint32))
    # ffn_down: k = 5632, Q6_K
    kd, k2, n2 = 6, 5632, 2048
    w = rk.synth_q_weights(kd, n2, k2, seed=62)
    a2 = rk.synth_normal(63, m * k2).reshape(m, k2)
    out = np.full((m, n2), np.nan, dtype=np.float32)
    assert ctx.matmul_q(kd, w, a2, out, m, k2, n2) == 0
    st, ref = oracle.matmul_q(kd, w, a2, n2)
    assert st == 0
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))
