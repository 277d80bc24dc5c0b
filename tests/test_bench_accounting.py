"""The byte and op accounting behind bench.py's roofline and e2e fields.

The roofline fraction the bench reports is only as good as the algorithmic
bytes and int8 ops it divides by, so they are recomputed here from the
TinyLlama-1.1B MUL_MAT shapes (22 layers; per layer a Q/K/V group of
n = 2048 + 256 + 256 and an O projection of n = 2048 at k = 2048, a gate/up
group of n = 5632 + 5632 at k = 2048, and a down projection of n = 2048 at
k = 5632), with the per-launch formulas of the GEMM kernel: int8 weights n*k,
int8 activations m*k, f32 outputs 4*m*n, scales 4*(m+n), and 2*m*n*k ops.
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402

CALLS = [(2048 + 256 + 256, 2048), (2048, 2048), (5632 + 5632, 2048), (2048, 5632)]


def test_tinyllama_step_accounting():
    bench.set_model("tinyllama")
    for m in (128, 512):
        b = ops = h2d = d2h = 0
        for n, k in CALLS:
            b += n * k + m * k + 4 * m * n + 4 * (m + n)
            ops += 2 * m * n * k
            h2d += 4 * m * k
            d2h += 4 * m * n
        assert bench.algorithmic(m) == (22 * b, 22 * ops)
        assert bench.h2d_d2h_bytes(m) == (22 * h2d, 22 * d2h)
    # the published per-step figures of the default workload
    assert bench.algorithmic(512) == (1910689792, 992137445376)
    assert bench.h2d_d2h_bytes(512) == (530579456, 807403520)


def test_layer_plan_follows_the_q4_k_m_mix():
    bench.set_model("tinyllama")
    for layer in range(22):
        plan = bench.layer_plan(layer)
        assert [name for name, _, _ in plan] == ["qkv", "o", "gate_up", "down"]
        qkv = plan[0][1]
        assert [kind for kind, _ in qkv] == [4, 4, 6]  # attn_v in Q6_K
        assert plan[3][1][0][0] == (6 if layer % 2 == 0 else 4)  # every other ffn_down in Q6_K
