"""The plugin's graph_compute decisions (rocknpu_graph_plan) on CPU, over the
node lists llama.cpp hands the plugin for TinyLlama-, Llama-3.2- and
Qwen2.5-shaped layers (ggml-rocknpu.cpp:838-976, 978-1650)."""
import pytest

import bench
import rocknpu_b200 as rk
from rocknpu_b200 import plugin
from rocknpu_b200.plugin import GGML_Q6_K, Node, OP_OTHER, OP_VIEW

TINY = dict(hidden=2048, ffn=5632, kv=256)
LLAMA = dict(hidden=2048, ffn=8192, kv=512)
QWEN = dict(hidden=1536, ffn=8960, kv=256)

ENV = ["ROCKNPU_DECODE", "ROCKNPU_FFN_COMPOSITE", "ROCKNPU_NPU_OUTPUT_HEAD", "ROCKNPU_MTILE_GROUP", "ROCKNPU_MTILE_QKV",
       "ROCKNPU_QKV_TRIPLE", "ROCKNPU_VK_PAIR", "ROCKNPU_FFN_PAIR", "ROCKNPU_M16_CHUNK_BATCH", "ROCKNPU_M32_AS_2X16",
       "ROCKNPU_RUNTIME_M16_PREWARM", "ROCKNPU_RUNTIME_M16_W8_ONLY"]


@pytest.fixture(autouse=True)
def env(monkeypatch):
    rk.apply_default_env()
    for name in ENV:
        monkeypatch.delenv(name, raising=False)
    return monkeypatch


def calls(planner, split):
    return [(a["call"], a["members"]) for a in planner.plan(split)]


def short(names):
    return [n.split(".", 2)[2].replace(".weight", "") for n in names]


def test_prompt_qkv_stash_across_splits_and_evaluations():
    """Q, K and V sit in separate splits.  The first evaluation runs them one
    by one (the plugin learns the layer's K and V weights); from the second on
    the Q node runs Q, K and V as one concatenated call, releases the three
    single-projection caches once, and the K and V nodes copy their outputs
    from the stash (:868-928, :948-960)."""
    p = plugin.GraphPlanner()
    first = [calls(p, s) for s in plugin.model_splits(TINY, 5, 512)]
    assert [c[0][0] for c in first] == ["single", "single", "single", "single", "concat", "single"]
    assert short(first[4][0][1]) == ["ffn_gate", "ffn_up"]
    second = [calls(p, s) for s in plugin.model_splits(TINY, 5, 512)]
    assert second[0][0][0] == "concat" and short(second[0][0][1]) == ["attn_q", "attn_k", "attn_v"]
    assert second[0][1][0] == "release"
    assert second[1] == [("stash", ["blk.5.attn_k.weight"])]
    assert second[2] == [("stash", ["blk.5.attn_v.weight"])]
    third = [calls(p, s) for s in plugin.model_splits(TINY, 5, 512)]
    assert len(third[0]) == 1 and third[0][0][0] == "concat"  # released only once


def test_stash_needs_the_same_activation_and_rows():
    p = plugin.GraphPlanner()
    for _ in range(2):
        for s in plugin.model_splits(TINY, 1, 256):
            p.plan(s)
    q, k, _ = plugin.model_splits(TINY, 1, 256)[:3]
    p.plan(q)
    k[0].m = 128  # a different batch: no stash, the node runs itself
    assert calls(p, k)[0][0] == "single"


@pytest.mark.parametrize("name,spec,m", [("tinyllama", TINY, 512), ("tinyllama", TINY, 128),
                                         ("llama32-1b", LLAMA, 512), ("qwen25-1.5b", QWEN, 2048)])
def test_bench_layer_plan_is_the_plugins(name, spec, m):
    """bench.py's per-layer MUL_MAT calls are the plugin's steady-state calls
    for these models (the reference arm replays the same list)."""
    bench.set_model(name)
    try:
        planned = plugin.layer_calls(spec, m, layers=4)
        for layer in range(4):
            got = [(c, [(plugin.TYPE_TO_KIND[t], n) for (_, t, n) in members], k) for c, members, k in planned[layer]]
            want = [("concat" if len(mem) > 1 else "single", mem, k) for _, mem, k in bench.layer_plan(layer)]
            assert got == want, (layer, got, want)
    finally:
        bench.set_model("tinyllama")


def test_same_input_group_limits():
    """At most 4 same-input projections form a group (:867-875); a group wider
    than 3 x 8192 columns keeps the lead on the per-node path (:935), and the
    next node leads a group of its own; k above 4096 or m below 32 never
    groups (:846-859)."""
    p = plugin.GraphPlanner()
    five = [Node(name=f"x{i}", k=2048, n=512, m=64, act=7) for i in range(5)]
    c = calls(p, five)
    assert c[0] == ("concat", ["x0", "x1", "x2", "x3"]) and c[1] == ("single", ["x4"])
    wide = [Node(name=f"w{i}", k=2048, n=8192, m=64, act=8) for i in range(4)]
    assert calls(p, wide) == [("single", ["w0"]), ("concat", ["w1", "w2", "w3"])]
    deep = [Node(name="a", k=5632, n=256, m=64, act=9), Node(name="b", k=5632, n=256, m=64, act=9)]
    assert [x[0] for x in calls(p, deep)] == ["single", "single"]
    short_m = [Node(name="c", k=2048, n=256, m=16, act=10), Node(name="d", k=2048, n=256, m=16, act=10)]
    assert [x[0] for x in calls(p, short_m)] == ["single", "single"]


@pytest.mark.parametrize("has_w8", [True, False])
def test_decode_triple_after_two_stable_observations(env, has_w8):
    """M=1: V and K (two nodes apart) run as a pair until the layer's Q, V
    and K weights have been seen unchanged twice; then the Q node runs the
    triple and the V/K node copies from its stash (:1185-1258, :1385-1445).
    Without W8 sidecars the calls are the K-quant forms."""
    env.setenv("ROCKNPU_DECODE", "npu")
    p = plugin.GraphPlanner()
    seen = []
    for _ in range(3):
        seen.append([(a["call"], a["w8"]) for s in plugin.model_splits(TINY, 2, 1, has_w8=has_w8)
                     for a in p.plan(s)])
    assert seen[0] == [("single", has_w8), ("pair_m1", has_w8), ("single", has_w8), ("pair_m1", has_w8),
                       ("single", has_w8)]
    assert seen[1] == seen[0]
    assert seen[2][:2] == [("triple_m1", has_w8), ("stash", False)]
    assert seen[2][2:] == seen[0][2:]


def test_decode_triple_resets_when_the_weights_change(env):
    env.setenv("ROCKNPU_DECODE", "npu")
    p = plugin.GraphPlanner()
    for _ in range(3):
        for s in plugin.model_splits(TINY, 2, 1):
            p.plan(s)
    splits = plugin.model_splits(TINY, 2, 1)
    splits[0][0].weight_id = 0xABC000  # another Q tensor (a reloaded model)
    assert calls(p, splits[0])[0][0] == "single"


def test_ffn_composite_defers_gate_up_to_down(env):
    """ROCKNPU_FFN_COMPOSITE with W8 sidecars: the M=1 gate/up pair waits for
    the down node, which runs gate, up, SwiGLU and down in one call
    (:1132-1183, :1300-1318); without sidecars the usual pair runs."""
    env.setenv("ROCKNPU_DECODE", "npu")
    env.setenv("ROCKNPU_FFN_COMPOSITE", "1")
    p = plugin.GraphPlanner()
    splits = plugin.model_splits(TINY, 0, 1, has_w8=True)
    assert calls(p, splits[3])[0][0] == "ffn_defer"
    c = calls(p, splits[4])
    assert c[0][0] == "swiglu_down" and short(c[0][1]) == ["ffn_gate", "ffn_up", "ffn_down"]
    p2 = plugin.GraphPlanner()
    splits = plugin.model_splits(TINY, 0, 1, has_w8=False)
    assert calls(p2, splits[3])[0][0] == "pair_m1"
    assert calls(p2, splits[4])[0][0] == "single"


def test_output_head_split(env):
    env.setenv("ROCKNPU_DECODE", "npu")
    env.setenv("ROCKNPU_NPU_OUTPUT_HEAD", "1")
    p = plugin.GraphPlanner()
    head = Node(name="output.weight", wtype=GGML_Q6_K, k=2048, n=32000, m=1, act=3, has_w8=True)
    a = p.plan([head])
    assert a[0]["call"] == "output_head_nsplit" and a[0]["n"] == 32000
    head.has_w8 = False  # no sidecar: graph_compute fails
    assert p.plan([head])[0]["call"] == "failed"


def test_view_nodes_and_failures():
    p = plugin.GraphPlanner()
    nodes = [Node(op=OP_VIEW), Node(name="a", k=2048, n=512, m=64, act=1, compute=False),
             Node(name="b", k=2048, n=512, m=64, act=2), Node(op=OP_OTHER), Node(name="c", k=2048, n=512, m=64, act=3)]
    assert calls(p, nodes) == [("single", ["b"]), ("failed", [])]
    # a MUL_MAT supports_op rejects fails the split too
    assert calls(p, [Node(name="d", k=100, n=512, m=64, act=4)])[0][0] == "failed"


def test_m16_router_sends_other_batches_to_the_cpu(env):
    """With the CPU fallback backend (ROCKNPU_RUNTIME_M16_ROUTER), splits that
    are not all M=16-routable run on the CPU, after pre-warming the TinyLlama
    shapes' prompt caches when ROCKNPU_RUNTIME_M16_PREWARM is set; M=16
    splits stay on the device (:980-1068)."""
    env.setenv("ROCKNPU_RUNTIME_M16_PREWARM", "1")
    p = plugin.GraphPlanner(cpu_fallback=True)
    c = calls(p, plugin.model_splits(TINY, 0, 512)[4])
    assert [x[0] for x in c] == ["prewarm", "prewarm", "cpu_fallback"]
    c = calls(p, plugin.model_splits(TINY, 0, 16)[4])
    assert "cpu_fallback" not in [x[0] for x in c]


def test_chunked_m16_batches(env):
    env.setenv("ROCKNPU_M16_CHUNK_BATCH", "1")
    env.setenv("ROCKNPU_NATIVE_MTILE", "0")
    p = plugin.GraphPlanner()
    c = p.plan([Node(name="x", k=2048, n=2048, m=64, act=1)])
    assert c[0]["call"] == "chunked_m16" and c[0]["m"] == 64


def test_plan_rejects_null_and_small_capacity():
    import ctypes
    L = plugin._lib()
    st = L.rocknpu_graph_state_create(0)
    try:
        nodes = (plugin.GraphNode * 1)()
        assert L.rocknpu_graph_plan(None, nodes, 1, None, 0) == -1
        out = (plugin.GraphAction * 1)()
        n = plugin.GraphNode()
        n.op = OP_VIEW
        n.compute = 1
        assert L.rocknpu_graph_plan(st, ctypes.byref(n), 1, out, 1) == 0
    finally:
        L.rocknpu_graph_state_destroy(st)
