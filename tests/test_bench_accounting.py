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


def test_decode_plan_is_the_planner_m1_calls_on_the_prefill_weights():
    """The bench's decode key replays rocknpu_graph_plan's M=1 calls with the
    plugin's decode switch on: per layer the QKV triple (q, v, k), o, the
    gate/up pair and down -- 88 calls per token -- and every member is a
    prefill weight of the same kind and shape (the same resident bytes)."""
    bench.set_model("tinyllama")
    before = os.environ.get("ROCKNPU_DECODE")
    plan = bench.decode_plan()
    assert os.environ.get("ROCKNPU_DECODE") == before  # the switch is restored
    assert len(plan) == 22 and sum(len(calls) for calls in plan) == 88
    group = {"attn_q": ("qkv", 0), "attn_k": ("qkv", 1), "attn_v": ("qkv", 2), "attn_output": ("o", 0),
             "ffn_gate": ("gate_up", 0), "ffn_up": ("gate_up", 1), "ffn_down": ("down", 0)}
    for layer, calls in enumerate(plan):
        assert [c for c, _, _ in calls] == ["triple_m1", "single", "pair_m1", "single"]
        assert [name.split(".")[2] for name, _, _ in calls[0][1]] == ["attn_q", "attn_v", "attn_k"]
        prefill = {name: (members, k) for name, members, k in bench.layer_plan(layer)}
        for _, members, k in calls:
            for name, kind, n in members:
                call, slot = group[name.split(".")[2]]
                assert prefill[call][0][slot] == (kind, n) and prefill[call][1] == k
