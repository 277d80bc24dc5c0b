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


@pytest.mark.parametrize("kind", [4, 6])
def test_largest_plugin_shape_through_the_c_abi(ctx, kind):
    """The largest MUL_MAT the plugin offloads on the prompt path
    (ggml-rocknpu.cpp:614-715: k % 256 == 0 with ceil512(k) <= 12288, n % 32 == 0
    with n <= 24576): k = 12288, n = 24576 -- the reference splits such a call
    into <= 8192-column chunks (split_wide_mtile, capi/src/lib.rs:2136-2160),
    which leaves every element's value unchanged -- at m = 320, bit for bit
    against the oracle."""
    m, k, n = 320, 12288, 24576
    w = rk.synth_q_weights(kind, n, k, seed=70 + kind)
    a = rk.synth_normal(71, m * k).reshape(m, k)
    out = np.full((m, n), np.nan, dtype=np.float32)
    assert rk.mul_mat_supported(rk.capi.GGML_Q4_K if kind == 4 else rk.capi.GGML_Q6_K, k, n, m)
    assert ctx.matmul_q(kind, w, a, out, m, k, n) == 0
    st, ref = oracle.matmul_q(kind, w, a, n)
    assert st == 0
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_tinyllama_pp512_whole_step_through_the_c_abi():
    """Every MUL_MAT call of the default bench step (22 layers x {QKV group,
    O, gate/up group, down} of the TinyLlama-shaped Q4_K_M prefill at 512
    tokens, built by bench.py's own workload constructors) through the
    reference C ABI, each member's output bit for bit against the oracle."""
    import os
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    bench.set_model("tinyllama")
    m = 512
    weights = bench.make_weights()
    acts = bench.make_activations(m, seed=5000)
    c = rk.Context()
    try:
        for key, blocks in weights.items():
            _, members, k = bench.layer_plan(key[0])[["qkv", "o", "gate_up", "down"].index(key[1])]
            a = acts[key]
            outs = [np.full((m, n), np.nan, dtype=np.float32) for _, n in members]
            if len(members) > 1:
                st = c.matmul_q_concat(blocks, [kd for kd, _ in members], [n for _, n in members], a, outs, m, k)
            else:
                st = c.matmul_q(members[0][0], blocks[0], a, outs[0], m, k, members[0][1])
            assert st == 0, key
            for (kd, n), b, o in zip(members, blocks, outs):
                st, ref = oracle.matmul_q(kd, b, a, n)
                assert st == 0
                assert np.array_equal(o.view(np.uint32), ref.view(np.uint32)), (key, kd, n)
    finally:
        c.close()
