"""The ggml plugin's graph_compute decisions (rocknpu_graph_plan in the
library) from Python: node lists for a model's splits, and the calls the
plugin makes for them.

``rocknpu_graph_plan`` restates rocknpu_backend_graph_compute
(adapters/ggml-rocknpu/src/ggml-rocknpu.cpp:978-1650) and
rocknpu_mtile_group (:838-976): which MUL_MAT nodes become one concatenated
call, which prompt-batch K/V outputs come from the Q node's stash, which
decode projections run as a triple or pair.  ``model_splits`` describes one
transformer layer's MUL_MATs the way llama.cpp hands them to the plugin:
Q, K and V in separate splits (RoPE, bias adds and the KV-cache copies are CPU
ops between them), V and K of a decode step two nodes apart, gate and up
adjacent, then down.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from .capi import MulMatDesc, lib

OP_MUL_MAT, OP_VIEW, OP_OTHER = 1, 2, 3
GGML_F32, GGML_F16, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 0, 1, 12, 13, 14

CALLS = {1: "concat", 2: "stash", 3: "release", 4: "output_head_nsplit", 5: "ffn_defer", 6: "swiglu_down",
         7: "triple_m1", 8: "pair_m1", 9: "pair_mtile", 10: "chunked_m16", 11: "single", 12: "prewarm",
         13: "cpu_fallback", 14: "failed"}
KIND_TO_TYPE = {4: GGML_Q4_K, 5: GGML_Q5_K, 6: GGML_Q6_K}
TYPE_TO_KIND = {v: k for k, v in KIND_TO_TYPE.items()}


class GraphNode(ctypes.Structure):
    """rocknpu_graph_node."""
    _fields_ = [("op", ctypes.c_int32), ("compute", ctypes.c_int32), ("desc", MulMatDesc),
                ("weight_name", ctypes.c_char_p), ("weight", ctypes.c_void_p), ("weight_bytes", ctypes.c_size_t),
                ("activation", ctypes.c_void_p), ("activation_data", ctypes.c_void_p), ("has_w8", ctypes.c_int32)]


class GraphAction(ctypes.Structure):
    """rocknpu_graph_action."""
    _fields_ = [("call", ctypes.c_int32), ("node", ctypes.c_int32), ("count", ctypes.c_int32),
                ("members", ctypes.c_int32 * 4), ("weights", ctypes.c_void_p * 4), ("w8", ctypes.c_int32),
                ("layer", ctypes.c_int32), ("m", ctypes.c_int64), ("k", ctypes.c_int64), ("n", ctypes.c_int64)]


def _lib():
    return lib()


@dataclass
class Node:
    """One node of a split: a MUL_MAT (weight name, ggml type, k, n, m and
    the activation it reads) or a view op."""
    name: str = ""
    wtype: int = GGML_Q4_K
    k: int = 0
    n: int = 0
    m: int = 0
    act: int = 0          # activation identity (same value = same src1 tensor)
    op: int = OP_MUL_MAT
    compute: bool = True
    has_w8: bool = False
    weight_id: int = 0    # weight identity (0: derived from the name)


def _weight_bytes(wtype: int, k: int, n: int) -> int:
    per = {GGML_Q4_K: 144, GGML_Q5_K: 176, GGML_Q6_K: 210}.get(wtype)
    return n * (k // 256) * per if per else n * k * 2


class GraphPlanner:
    """A rocknpu_graph_state: plan split after split, graph after graph."""

    def __init__(self, cpu_fallback: bool = False):
        self._L = _lib()
        self.handle = self._L.rocknpu_graph_state_create(1 if cpu_fallback else 0)
        if not self.handle:
            raise RuntimeError("rocknpu_graph_state_create failed")
        self._names = {}

    def close(self):
        if self.handle:
            self._L.rocknpu_graph_state_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _wid(self, node: Node) -> int:
        if node.weight_id:
            return node.weight_id
        return self._names.setdefault(node.name, 0x10000 + 0x1000 * len(self._names))

    def plan(self, nodes: list[Node]) -> list[dict]:
        """The plugin's calls for one split, in order."""
        arr = (GraphNode * max(1, len(nodes)))()
        keep = []
        names = {}
        for i, nd in enumerate(nodes):
            g = arr[i]
            g.op = nd.op
            g.compute = 1 if nd.compute else 0
            if nd.op == OP_MUL_MAT:
                d = g.desc
                d.is_mul_mat = 1
                d.weight_type, d.act_type, d.dst_type = nd.wtype, GGML_F32, GGML_F32
                d.weight_ne[:] = [nd.k, nd.n, 1, 1]
                d.act_ne[:] = [nd.k, nd.m, 1, 1]
                d.weight_contiguous = d.act_contiguous = d.dst_contiguous = 1
                name = nd.name.encode()
                keep.append(name)
                g.weight_name = name
                wid = self._wid(nd)
                names[wid] = nd.name
                g.weight = wid
                g.weight_bytes = _weight_bytes(nd.wtype, nd.k, nd.n)
                g.activation = 0x100 + nd.act
                g.activation_data = 0x100000 + nd.act
                g.has_w8 = 1 if nd.has_w8 else 0
        cap = 4 * len(nodes) + 4
        out = (GraphAction * cap)()
        cnt = self._L.rocknpu_graph_plan(self.handle, arr, len(nodes), out, cap)
        if cnt < 0:
            raise RuntimeError("rocknpu_graph_plan failed")
        for name, wid in self._names.items():
            names.setdefault(wid, name)
        res = []
        for a in out[:cnt]:
            members = [names.get(a.weights[j] or 0) for j in range(a.count)]
            res.append({"call": CALLS[a.call], "node": a.node, "members": members, "w8": bool(a.w8),
                        "layer": a.layer, "m": a.m, "k": a.k, "n": a.n})
        return res


def model_splits(spec: dict, layer: int, m: int, *, has_w8: bool = False, q6_down=None) -> list[list[Node]]:
    """One layer's MUL_MAT splits as llama.cpp hands them to the plugin.

    spec: hidden, ffn, kv (K/V projection width) of the model.  Q4_K_M's mix:
    Q4_K everywhere except attn_v and every other ffn_down (Q6_K).  Prompt
    batches (m > 1): Q, K and V each in their own split.  Decode (m == 1):
    Q, then V and K two nodes apart in one split (a view between them)."""
    h, f, kv = spec["hidden"], spec["ffn"], spec["kv"]
    down_q6 = (layer % 2 == 0) if q6_down is None else q6_down
    p = f"blk.{layer}."
    a_norm, a_attn, a_ffn, a_mid = 4 * layer + 1, 4 * layer + 2, 4 * layer + 3, 4 * layer + 4

    def mm(name, wtype, k, n, act):
        return Node(name=p + name, wtype=wtype, k=k, n=n, m=m, act=act, has_w8=has_w8)

    q = mm("attn_q.weight", GGML_Q4_K, h, h, a_norm)
    k = mm("attn_k.weight", GGML_Q4_K, h, kv, a_norm)
    v = mm("attn_v.weight", GGML_Q6_K, h, kv, a_norm)
    o = mm("attn_output.weight", GGML_Q4_K, h, h, a_attn)
    gate = mm("ffn_gate.weight", GGML_Q4_K, h, f, a_ffn)
    up = mm("ffn_up.weight", GGML_Q4_K, h, f, a_ffn)
    down = mm("ffn_down.weight", GGML_Q6_K if down_q6 else GGML_Q4_K, f, h, a_mid)
    if m == 1:
        return [[q], [v, Node(op=OP_VIEW), k], [o], [gate, up], [down]]
    return [[q], [k], [v], [o], [gate, up], [down]]


def layer_calls(spec: dict, m: int, layers: int, evaluations: int = 3) -> list[list[tuple]]:
    """The plugin's calls per layer in steady state (the last of
    `evaluations` graph evaluations, once the QKV stash is set up): per layer
    a list of (call, [(member name, ggml type, n)], k) for the calls that run
    a GEMM (stash copies and cache releases left out)."""
    planner = GraphPlanner()
    types = {}
    out = []
    for _ in range(evaluations):
        out = []
        for layer in range(layers):
            calls = []
            for split in model_splits(spec, layer, m):
                for nd in split:
                    if nd.op == OP_MUL_MAT:
                        types[nd.name] = (nd.wtype, nd.n)
                for a in planner.plan(split):
                    if a["call"] in ("stash", "release"):
                        continue
                    calls.append((a["call"], [(name, *types[name]) for name in a["members"]], a["k"]))
            out.append(calls)
    planner.close()
    return out
