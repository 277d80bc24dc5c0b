"""Benchmark of the RockNPU MUL_MAT offload on B200.

Default workload (the reference's headline metric):
every MUL_MAT the ggml plugin offloads in one TinyLlama-1.1B-shaped Q4_K_M
prefill of 512 tokens -- 22 layers x {QKV group (Q4_K 2048 + Q4_K 256 + Q6_K
256), O (Q4_K 2048), gate+up group (2 x Q4_K 5632), down (k 5632 -> 2048,
Q6_K in every other layer)}.  The vocabulary head (n = 32000) is not
offloaded by the reference (n > 24576, ggml-rocknpu.cpp:648) and the
attention / norm / RoPE work stays on llama.cpp's CPU backend, so neither is
in a step.  Weights are random-init (N(0, 0.02^2) encoded to Q4_K/Q6_K),
activations N(0, 1); prepared int8 weights are resident (the reference's
weight cache), 1.0 GB per step > L2, so no extra L2 flush is needed.

* pp128: the same step at 128 tokens (the headline metric is quoted at
  pp128 and pp512), device path.
* value: tok/s with activations already in HBM (device entry point
  rocknpu_b200_matmul_w8a8 per MUL_MAT: K2 per-token quantisation + the K3
  tcgen05 W8A8 GEMM, launched programmatically after it).
* e2e:   tok/s through the reference C ABI with page-locked host buffers
  (rocknpu_b200_host_alloc), as the plugin calls it
  (rocknpu_matmul_q_concat_f32_f32_mtile for the groups,
  rocknpu_matmul_q{4,6}_k_f32_f32 for O and down): H2D of every activation
  and D2H of every output inside the timed region.
* cpu_baseline / --impl reference: the reference's CPU path restated in C
  (oracle/, OpenMP, all host threads): per-token quantisation, exact int32
  GEMM (AMX tiles where the CPU has them, else AVX-512 VNNI; the line's
  "sample" names the path), rescale -- timed on a bounded sample of the same
  workload.

* pp128.roofline / roofline: the step's GEMM launches alone (one graph),
  algorithmic bytes and int8 ops against the measured peaks.
* cfg5 (N = 1): BASELINE.json configs[4] beside the headline step -- the
  W8A8 GEMM of the Q4_K weight N=28672 x K=8192 at M in {128, 1024, 4096,
  16384} (whole job and the GEMM kernel alone, against the int8 tensor or
  HBM roofline) and the M = 1 decode GEMVs on the same weight.
* shard (N > 1): the same GEMMs N-sharded over the ranks, the output columns
  all-gathered over NVLink by the GEMM epilogue's peer stores (strong
  scaling), with the per-rank receive bound and an in-run bit check of
  sampled rows against a single-GPU GEMM on rank 0.

Other configs: --workload llama32-1b (configs[2], pp512) and qwen25-1.5b
(configs[3], pp2048) replay those models' MUL_MAT calls the same way;
--workload cfg5 is the large-GEMM sharding sweep as its own line.

Multi-GPU (torchrun): the per-layer GEMMs do not shard at this size, so each
rank runs its own replica of the headline step on its own prompt batch (weak
scaling, no collective); value = all ranks' tokens / max-over-ranks time.
The large cfg5 GEMMs do shard (the `shard` key above).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# Shapes of the offloaded MUL_MATs of BASELINE.json configs[1..3] (the
# query projection is hidden wide; kv = kv heads x head dim).
MODELS = {
    "tinyllama": dict(name="tinyllama-1.1b", layers=22, hidden=2048, ffn=5632, kv=256, tokens=512),
    "llama32-1b": dict(name="llama-3.2-1b", layers=16, hidden=2048, ffn=8192, kv=512, tokens=512),
    "qwen25-1.5b": dict(name="qwen2.5-1.5b", layers=28, hidden=1536, ffn=8960, kv=256, tokens=2048),
}
MODEL = "tinyllama"
LAYERS = 22
HIDDEN, FFN, KV = 2048, 5632, 256


def set_model(name: str) -> None:
    global MODEL, LAYERS, HIDDEN, FFN, KV
    spec = MODELS[name]
    MODEL = name
    LAYERS, HIDDEN, FFN, KV = spec["layers"], spec["hidden"], spec["ffn"], spec["kv"]


def workload_name(m: int) -> str:
    return f"{MODELS[MODEL]['name']}-q4_k_m-prefill-pp{m}-mul_mat"


def metric_name(m: int) -> str:
    label = {"tinyllama": "TinyLlama", "llama32-1b": "Llama-3.2-1B", "qwen25-1.5b": "Qwen2.5-1.5B"}[MODEL]
    return f"prefill tok/s pp{m} {label}-shape Q4_K_M (ggml MUL_MAT offload)"


def layer_plan(layer: int):
    """(name, [(kind, n)], k) of the four offloaded MUL_MAT calls of a layer:
    Q4_K everywhere except attn_v and every other ffn_down (Q6_K), as
    llama.cpp's Q4_K_M mix places them."""
    down_kind = 6 if layer % 2 == 0 else 4
    return [("qkv", [(4, HIDDEN), (4, KV), (6, KV)], HIDDEN),
            ("o", [(4, HIDDEN)], HIDDEN),
            ("gate_up", [(4, FFN), (4, FFN)], HIDDEN),
            ("down", [(down_kind, HIDDEN)], FFN)]


def planned_layer_calls(m: int):
    """The plugin's own decisions for this model's layers in steady state
    (rocknpu_graph_plan over the splits llama.cpp hands the plugin), in the
    form of layer_plan(): [(call, [(kind, n)], k)] per layer.  Our arm checks
    that layer_plan() -- which the reference arm replays without loading the
    library -- is exactly this list."""
    from rocknpu_b200 import plugin
    spec = {"hidden": HIDDEN, "ffn": FFN, "kv": KV}
    out = []
    for calls in plugin.layer_calls(spec, m, LAYERS):
        out.append([(c, [(plugin.TYPE_TO_KIND[t], n) for (_, t, n) in members], k) for c, members, k in calls])
    return out


def check_layer_plan(m: int) -> str:
    planned = planned_layer_calls(m)
    for layer in range(LAYERS):
        want = [("concat" if len(members) > 1 else "single", members, k) for _, members, k in layer_plan(layer)]
        if planned[layer] != want:
            raise RuntimeError(f"layer {layer}: the plugin plans {planned[layer]}, the bench replays {want}")
    return "rocknpu_graph_plan (the plugin's graph_compute decisions, steady state)"


def algorithmic(m: int):
    """Bytes and int8 ops of the GEMM launches of one step (K3 only): int8
    weights + int8 activations + f32 output + scales, and 2*m*n*k."""
    b = ops = 0
    for layer in range(LAYERS):
        for _, members, k in layer_plan(layer):
            n = sum(nn for _, nn in members)
            b += n * k + m * k + 4 * m * n + 4 * n + 4 * m
            ops += 2 * m * n * k
    return b, ops


def h2d_d2h_bytes(m: int):
    h2d = d2h = 0
    for layer in range(LAYERS):
        for _, members, k in layer_plan(layer):
            h2d += 4 * m * k
            d2h += 4 * m * sum(nn for _, nn in members)
    return h2d, d2h


def new_graph():
    import torch
    try:
        return torch.cuda.CUDAGraph(keep_graph=True)
    except TypeError:
        return torch.cuda.CUDAGraph()


def graph_kernel_nodes(graph):
    """Kernel nodes of a captured CUDA graph (counted, not assumed), or None
    when the graph cannot be inspected."""
    try:
        from cuda.bindings import runtime as rt
        g = graph.raw_cuda_graph()
        err, _, count = rt.cudaGraphGetNodes(g, 0)
        err, nodes, count = rt.cudaGraphGetNodes(g, count)
        kernels = 0
        for node in nodes[:count]:
            err, kind = rt.cudaGraphNodeGetType(node)
            if kind == rt.cudaGraphNodeType.cudaGraphNodeTypeKernel:
                kernels += 1
        return kernels
    except Exception:
        return None


def profiled_traffic(m: int):
    """DRAM bytes per step of the GEMM launches, from the committed ncu
    summary of this workload (profiles/gemm_tc_tinyllama_pp512_dram.md);
    None for token counts that were not captured."""
    path = os.path.join(ROOT, "profiles", f"gemm_tc_{MODEL}_pp{m}_dram.md")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            if line.startswith("traffic_bytes_per_step:"):
                return int(line.split(":")[1])
    return None


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


_SAMPLER_SRC = r"""
import sys, time
import pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[1]))
getr = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
out = open(sys.argv[2], "w")
out.write("max %d\n" % pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
out.flush()
while True:
    t = time.monotonic()
    out.write("%.6f %d %d\n" % (t, pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), getr(h)))
    out.flush()
    time.sleep(0.002)
"""


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled through NVML every
    2 ms during the timed region, by a separate process (a sampling thread
    here could starve while the timed loop holds the interpreter lock);
    timestamps are CLOCK_MONOTONIC, shared by both processes."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples = []  # (time, sm MHz, reason bits)
        self.max_mhz = None

    def _read(self):
        try:
            with open(self.path) as f:
                lines = f.read().splitlines()
        except OSError:
            return
        samples = []
        for line in lines:
            parts = line.split()
            if len(parts) == 2 and parts[0] == "max":
                self.max_mhz = int(parts[1])
            elif len(parts) == 3:
                samples.append((float(parts[0]), int(parts[1]), int(parts[2])))
        self.samples = samples

    def __enter__(self):
        import subprocess
        import tempfile
        import torch
        try:
            idx = torch.cuda._get_nvml_device_index(self.cuda_index)
        except Exception:
            idx = self.cuda_index
        fd, self.path = tempfile.mkstemp(prefix="rocknpu_clocks_", suffix=".txt")
        os.close(fd)
        self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER_SRC, str(idx), self.path],
                                     stdout=subprocess.DEVNULL, stderr=subprocess.PIPE)
        # wait for the first samples (the sampler imports NVML first)
        deadline = time.monotonic() + 20.0
        while time.monotonic() < deadline and self.proc.poll() is None:
            self._read()
            if len(self.samples) >= 2:
                break
            time.sleep(0.01)
        if self.proc.poll() is not None:
            self.error = self.proc.stderr.read().decode(errors="replace").strip()[-300:] or "sampler exited"
        return self

    def __exit__(self, *exc):
        time.sleep(0.005)  # one more sample after the region
        if self.proc.poll() is None:
            self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except Exception:
            self.proc.kill()
        self._read()
        try:
            os.remove(self.path)
        except OSError:
            pass

    def mark(self, name):
        setattr(self, name, time.monotonic())

    def summary(self):
        t0, t1 = getattr(self, "t_start", None), getattr(self, "t_end", None)
        win = [x for x in self.samples if (t0 is None or x[0] >= t0) and (t1 is None or x[0] <= t1)]
        if not win and t0 is not None and t1 is not None:
            # a region shorter than the sampling period: the samples just
            # before and after it
            before = [x for x in self.samples if x[0] < t0][-1:]
            after = [x for x in self.samples if x[0] > t1][:1]
            win = before + after
        reasons = set()
        for _, _, r in win:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        out = {"sm_mhz": statistics.median([x[1] for x in win]) if win else None, "sm_max_mhz": self.max_mhz,
               "reasons": sorted(reasons), "samples": len(win)}
        if getattr(self, "error", None):
            out["error"] = self.error
        return out


# ---------------------------------------------------------------------------
# workload construction
# ---------------------------------------------------------------------------

def make_weights(seed: int = 1000, gen=None):
    """Host K-quant blocks per layer and call: {(layer, call): [blocks...]}.
    `gen` supplies synth_q_weights: the library (our arm) or the oracle's
    byte-identical generator (the reference arm, whose process must not load
    the library)."""
    if gen is None:
        import rocknpu_b200 as gen
    rk = gen
    weights = {}
    s = seed
    for layer in range(LAYERS):
        for name, members, k in layer_plan(layer):
            blocks = []
            for kind, n in members:
                blocks.append(rk.synth_q_weights(kind, n, k, seed=s, sigma=0.02))
                s += 1
            weights[(layer, name)] = blocks
    return weights


def make_activations(m: int, seed: int, gen=None):
    if gen is None:
        import rocknpu_b200 as gen
    rk = gen
    acts = {}
    s = seed
    for layer in range(LAYERS):
        for name, _, k in layer_plan(layer):
            acts[(layer, name)] = rk.synth_normal(s, m * k).reshape(m, k)
            s += 1
    return acts


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, rank: int, world: int):
    import torch
    import rocknpu_b200 as rk
    from rocknpu_b200 import device as dev

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    rk.apply_default_env()
    m = args.tokens
    hbm_peak, bf16_peak, peak_src = load_peaks()
    int8_peak_tops = 2.0 * bf16_peak  # dense int8 = 2x dense bf16 on B200

    t0 = time.time()
    plan_source = check_layer_plan(m)
    weights = make_weights()
    acts = make_activations(m, seed=5000 + 97 * rank)
    gen_s = time.time() - t0

    ctx = rk.Context()
    stream = torch.cuda.current_stream()
    status = dev.new_status()

    # resident prepared weights (K1 on the GPU), concatenated per call
    prepared = {}
    for key, blocks in weights.items():
        _, members, k = layer_plan(key[0])[["qkv", "o", "gate_up", "down"].index(key[1])]
        ws, ss = [], []
        for (kind, n), b in zip(members, blocks):
            w8, s8 = dev.prepare_w8(kind, torch.from_numpy(b).cuda(), k, n, status)
            ws.append(w8)
            ss.append(s8)
        prepared[key] = (torch.cat(ws).contiguous(), torch.cat(ss).contiguous(), k)
    torch.cuda.synchronize()
    assert status.item() == 0, "weight preparation failed"

    d_acts = {key: torch.from_numpy(a).cuda() for key, a in acts.items()}
    outs = {}
    for key, (w8, s8, k) in prepared.items():
        outs[key[1]] = torch.empty((m, w8.shape[0]), dtype=torch.float32, device="cuda")

    def step():
        for key, (w8, s8, k) in prepared.items():
            dev.matmul_w8a8(ctx, d_acts[key], w8, s8, outs[key[1]])


    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        dist = dist_mod

    def barrier():
        if dist is not None:
            dist.barrier()

    # eager warm-up sizes the context workspaces, then the step is captured
    # once as a CUDA graph (88 x {K2, K3}, each GEMM a programmatic dependent
    # launch of its quantiser) and replayed
    step()
    torch.cuda.synchronize()
    graph = new_graph()
    with torch.cuda.graph(graph):
        step()
    launches_per_step = graph_kernel_nodes(graph)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if rk.lib().rocknpu_b200_context_check(ctx.handle) != 0:
        raise RuntimeError("device status error during warm-up")

    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        clocks.mark("t_start")
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize()
        clocks.mark("t_end")
    barrier()
    ms = start.elapsed_time(end) / args.steps
    if rk.lib().rocknpu_b200_context_check(ctx.handle) != 0:
        raise RuntimeError("device status error during timing")

    # roofline of the dominant kernel (K3): the step's GEMM launches alone,
    # on pre-quantised activations, as one graph
    def gemm_roofline(mm, acts_src, outs_src, step_ms):
        a8 = {key: dev.quantize_rows(acts_src[key], status) for key in prepared}
        ws_bytes = max(dev.workspace_bytes(mm, w8.shape[0], k) for (w8, s8, k) in prepared.values())
        gemm_ws = dev.new_workspace(ws_bytes)

        def gemm_step():
            for key, (w8, s8, k) in prepared.items():
                dev.gemm_w8a8(a8[key][0], a8[key][1], w8, s8, status, out=outs_src[key[1]], workspace=gemm_ws)

        gemm_step()
        torch.cuda.synchronize()
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2):
            gemm_step()
        for _ in range(3):
            g2.replay()
        reps = max(5, args.steps)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            g2.replay()
        e1.record()
        torch.cuda.synchronize()
        assert status.item() == 0, "GEMM status error"
        gemm_ms = e0.elapsed_time(e1) / reps
        if dist is not None:
            t = torch.tensor([gemm_ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            gemm_ms = float(t.item())
        alg_bytes, alg_ops = algorithmic(mm)
        gb_s = alg_bytes / (gemm_ms * 1e-3) / 1e9
        tops = alg_ops / (gemm_ms * 1e-3) / 1e12
        t_hbm = alg_bytes / (hbm_peak * 1e9)
        t_tc = alg_ops / (int8_peak_tops * 1e12)
        if t_hbm >= t_tc:
            r = {"bound": "hbm", "achieved": round(gb_s, 1), "peak": hbm_peak, "unit": "GB/s",
                 "frac": round(gb_s / hbm_peak, 4)}
        else:
            r = {"bound": "tensor", "achieved": round(tops, 1), "peak": int8_peak_tops, "unit": "TOP/s",
                 "frac": round(tops / int8_peak_tops, 4)}
        traffic = profiled_traffic(mm)
        r.update({"kernel": "gemm_tc_kernel (K3, tcgen05 kind::i8)", "traffic": traffic,
                  "traffic_unit": f"DRAM bytes per step ({len(prepared)} launches), ncu capture" if traffic else None,
                  "peak_source": f"{peak_src} (int8 = 2 x bf16_tflops)" if r["bound"] == "tensor"
                  else f"{peak_src} hbm_gbs",
                  "hbm_frac": round(gb_s / hbm_peak, 4), "tensor_frac": round(tops / int8_peak_tops, 4),
                  "gemm_ms_per_step": round(gemm_ms, 4), "gemm_share_of_step": round(gemm_ms / step_ms, 3),
                  "gemm_launches_per_step": len(prepared),
                  "algorithmic_bytes_per_step": alg_bytes, "int8_ops_per_step": alg_ops})
        del g2
        return r

    # the other prompt length of the headline metric (pp128 beside pp512):
    # the same calls on the first 128 tokens of every activation
    short = None
    if m > 128 and not args.no_short:
        ms_short = 128
        s_acts = {key: d_acts[key][:ms_short] for key in prepared}
        s_outs = {name: torch.empty((ms_short, t.shape[1]), dtype=torch.float32, device="cuda")
                  for name, t in outs.items()}

        def short_step():
            for key, (w8, s8, k) in prepared.items():
                dev.matmul_w8a8(ctx, s_acts[key], w8, s8, s_outs[key[1]])
        short_step()
        torch.cuda.synchronize()
        gs = new_graph()
        with torch.cuda.graph(gs):
            short_step()
        for _ in range(args.warmup):
            gs.replay()
        torch.cuda.synchronize()
        e0s, e1s = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0s.record()
        for _ in range(args.steps):
            gs.replay()
        e1s.record()
        torch.cuda.synchronize()
        if rk.lib().rocknpu_b200_context_check(ctx.handle) != 0:
            raise RuntimeError("device status error during the pp128 timing")
        t_short = e0s.elapsed_time(e1s) / args.steps
        if dist is not None:
            t = torch.tensor([t_short], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_short = float(t.item())
        del gs
        short = {"tokens_per_step": ms_short, "value": round(world * ms_short / (t_short * 1e-3), 1), "unit": "tok/s",
                 "ms_per_step": round(t_short, 4), "roofline": gemm_roofline(ms_short, s_acts, s_outs, t_short)}

    roof = gemm_roofline(m, d_acts, outs, ms)

    # e2e through the reference C ABI with page-locked host buffers
    e2e = None
    if not args.no_e2e:
        # page-locked host buffers from the library's allocator (huge-page
        # backed: steady host-to-device copy rate)
        h_acts = {}
        for key, a in acts.items():
            h_acts[key] = rk.host_empty(a.shape)
            h_acts[key][...] = a
        h_outs = {}
        for key in prepared:
            members = layer_plan(key[0])[["qkv", "o", "gate_up", "down"].index(key[1])][1]
            h_outs[key] = [rk.host_empty((m, n)) for _, n in members]

        # each call as (C-ABI function, arguments) with the buffers' addresses
        # taken once (the arrays stay alive in weights / h_acts / h_outs), so
        # the timed loop costs what a C caller's would plus one ctypes call
        L = rk.lib()
        qfn = {4: L.rocknpu_matmul_q4_k_f32_f32, 6: L.rocknpu_matmul_q6_k_f32_f32}
        bound = []
        for key, blocks in weights.items():
            _, members, k = layer_plan(key[0])[["qkv", "o", "gate_up", "down"].index(key[1])]
            a, os_ = h_acts[key], h_outs[key]
            if len(members) > 1:
                cnt = len(members)
                arrs = ((ctypes.c_void_p * cnt)(*[b.ctypes.data for b in blocks]),
                        (ctypes.c_size_t * cnt)(*[b.nbytes for b in blocks]),
                        (ctypes.c_uint32 * cnt)(*[kd for kd, _ in members]),
                        (ctypes.c_size_t * cnt)(*[n for _, n in members]),
                        (ctypes.c_void_p * cnt)(*[o.ctypes.data for o in os_]))
                bound.append((key, L.rocknpu_matmul_q_concat_f32_f32_mtile,
                              (ctx.handle, cnt, arrs[0], arrs[1], arrs[2], arrs[3], a.ctypes.data, arrs[4], m, k),
                              arrs))
            else:
                kd, n = members[0]
                bound.append((key, qfn[kd], (ctx.handle, blocks[0].ctypes.data, blocks[0].nbytes, a.ctypes.data,
                                             os_[0].ctypes.data, m, k, n), None))

        def e2e_step():
            for key, fn, args, _ in bound:
                st = fn(*args)
                if st != 0:
                    raise RuntimeError(f"C ABI call {key} failed: {st}")

        for _ in range(max(1, args.warmup)):
            e2e_step()  # first pass also builds the resident weight caches
        barrier()
        e_steps = max(1, min(args.steps, 10))
        t_start = time.perf_counter()
        for _ in range(e_steps):
            e2e_step()
        e2e_s = (time.perf_counter() - t_start) / e_steps
        if dist is not None:
            t = torch.tensor([e2e_s], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        h2d, d2h = h2d_d2h_bytes(m)
        e2e = {"value": round(world * m / e2e_s, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_s * 1e3, 3),
               "path": "rocknpu_matmul_q_concat_f32_f32_mtile + rocknpu_matmul_q{4,6}_k_f32_f32, "
                       "rocknpu_b200_host_alloc host buffers"}

    # configs[1]'s decode steps: every rank decodes on its own GPU (M = 1
    # calls do not shard), rank 0 reports
    dec = None
    if not args.no_decode and MODEL == "tinyllama":
        dec = decode_block(weights, DECODE_TOKENS, args.warmup)

    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # BASELINE.json configs[4] beside the headline step: at N = 1 the large
    # W8A8 GEMM (M in {128, 1024, 4096, 16384}) and the M = 1 decode GEMVs on
    # the N=28672 x K=8192 Q4_K weight, against their rooflines; at N > 1 the
    # same GEMMs N-sharded over the ranks with the output all-gathered over
    # NVLink, checked bit for bit against one GPU in the run
    big = big_clocks = None
    if not args.no_cfg5 and MODEL == "tinyllama":
        big, big_clocks = cfg5_block(list(CFG5_M), min(args.steps, 10), max(args.warmup, 3), rank, world,
                                     route=args.route)
        if big is not None:
            big["clocks"] = big_clocks

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(weights, acts, m, budget_s=args.cpu_seconds)

    ctx.close()
    if rank != 0:
        return None
    line = {
        "metric": metric_name(m),
        "value": round(world * m / (ms * 1e-3), 1),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8 (W8A8, int32 accumulate, f32 out)",
        "data": "synthetic (random-init N(0,0.02^2) -> Q4_K/Q6_K weights, N(0,1) activations)",
        "config": step_config(m, world, len(prepared)),
        "roofline": roof,
        "pp128": short,
        "e2e": e2e,
        "decode": dec,
        "cpu_baseline": cpu,
        "gpu_launches": launches_per_step * args.steps if launches_per_step is not None else None,
        "launches_per_step": launches_per_step,
        "calls_planned_by": plan_source,
        "clocks": clocks.summary(),
        "setup_s": round(gen_s, 1),
    }
    if big is not None:
        line["cfg5" if world == 1 else "shard"] = big
    return line


DECODE_TOKENS = 128  # configs[1]: 128 decode steps after the prompt


def decode_plan():
    """The plugin's M=1 calls per layer with its decode switch on
    (ROCKNPU_DECODE=npu, ggml-rocknpu.cpp:313-322): [(call, [(kind, n)], k)]
    -- the QKV triple (q, v, k), o, the gate/up pair, down."""
    from rocknpu_b200 import plugin
    old = os.environ.get("ROCKNPU_DECODE")
    os.environ["ROCKNPU_DECODE"] = "npu"
    try:
        spec = {"hidden": HIDDEN, "ffn": FFN, "kv": KV}
        out = []
        for calls in plugin.layer_calls(spec, 1, LAYERS):
            out.append([(c, [(name, plugin.TYPE_TO_KIND[t], n) for (name, t, n) in members], k)
                        for c, members, k in calls])
        return out
    finally:
        if old is None:
            os.environ.pop("ROCKNPU_DECODE", None)
        else:
            os.environ["ROCKNPU_DECODE"] = old


def decode_block(weights, tokens, warmup):
    """TinyLlama-shape decode (configs[1]'s decode steps): per token the
    plugin's 88 M=1 calls (decode_plan) through the reference's M=1 entry
    points from page-locked host buffers, on the default W8A8 route and on
    the opt-in K5b route (ROCKNPU_B200_DECODE_KQ); wall time per token (each
    call is synchronous).  Weights as in the prefill step; x per call N(0,1)."""
    import rocknpu_b200 as rk
    plan = decode_plan()
    slot = {"attn_q": 0, "attn_k": 1, "attn_v": 2, "attn_output": 0, "ffn_gate": 0, "ffn_up": 1, "ffn_down": 0}
    group = {"attn_q": "qkv", "attn_k": "qkv", "attn_v": "qkv", "attn_output": "o", "ffn_gate": "gate_up",
             "ffn_up": "gate_up", "ffn_down": "down"}
    calls = []  # (entry, [(blocks, kind, n)], k, x, outs)
    s = 7000
    for layer, lcalls in enumerate(plan):
        for call, members, k in lcalls:
            ms = []
            for name, kind, n in members:
                short = name.split(".")[2]
                blocks = weights[(layer, group[short])][slot[short]]
                if blocks.size != n * (k // 256) * rk.BLOCK_BYTES[kind]:
                    raise RuntimeError(f"decode plan member {name} does not match the prefill weights")
                ms.append((blocks, kind, n))
            x = rk.host_empty((k,))
            x[...] = rk.synth_normal(s, k)
            s += 1
            calls.append((call, ms, k, x, [rk.host_empty((n,)) for _, _, n in ms]))
    weight_bytes = sum(b.nbytes for _, ms, _, _, _ in calls for b, _, _ in ms)
    int8_bytes = sum(n * k for _, ms, k, _, _ in calls for _, _, n in ms)
    rows = sum(n for _, ms, _, _, _ in calls for _, _, n in ms)
    hbm_gbs = load_peaks()[0]

    def bind(ctx):
        # each call as (C-ABI function, its arguments) with the buffers'
        # addresses taken once (the arrays stay alive in `calls`): the loop
        # then costs what a C caller's would plus one ctypes call
        L, h = rk.lib(), ctx.handle
        fns = {4: L.rocknpu_matmul_q4_k_f32_f32, 6: L.rocknpu_matmul_q6_k_f32_f32}
        bound = []
        for call, ms, k, x, outs in calls:
            xa, oa = x.ctypes.data, [o.ctypes.data for o in outs]
            if call == "triple_m1":
                args = [h]
                for w, kd, n in ms:
                    args += [w.ctypes.data, w.nbytes, kd, n]
                bound.append((call, L.rocknpu_matmul_q_triple_f32_f32_m1, tuple(args + [xa] + oa + [k])))
            elif call == "pair_m1":
                args = [h]
                for w, kd, n in ms:
                    args += [w.ctypes.data, w.nbytes, kd, n]
                bound.append((call, L.rocknpu_matmul_q_pair_f32_f32_m1, tuple(args + [xa] + oa + [k])))
            else:
                w, kd, n = ms[0]
                bound.append((call, fns[kd], (h, w.ctypes.data, w.nbytes, xa, oa[0], 1, k, n)))
        return bound

    def token(bound):
        for call, fn, args in bound:
            st = fn(*args)
            if st != 0:
                raise RuntimeError(f"decode call {call} failed: {st}")

    res = {"tokens": tokens, "calls_per_token": len(calls), "planned_by": "rocknpu_graph_plan, ROCKNPU_DECODE=npu",
           "path": "rocknpu_matmul_q_triple/pair_f32_f32_m1 + rocknpu_matmul_q{4,6}_k_f32_f32 at m = 1, "
                   "rocknpu_b200_host_alloc host buffers"}
    for route, env in (("w8a8", None), ("kq", "1")):
        old = os.environ.pop("ROCKNPU_B200_DECODE_KQ", None)
        if env is not None:
            os.environ["ROCKNPU_B200_DECODE_KQ"] = env
        try:
            ctx = rk.Context()  # the route is read when the context is created
        finally:
            os.environ.pop("ROCKNPU_B200_DECODE_KQ", None)
            if old is not None:
                os.environ["ROCKNPU_B200_DECODE_KQ"] = old
        try:
            bound = bind(ctx)
            for _ in range(max(1, warmup)):
                token(bound)  # the first token also builds the resident decode weights
            t0 = time.perf_counter()
            for _ in range(tokens):
                token(bound)
            dt = (time.perf_counter() - t0) / tokens
            resident = ctx.decode_cache_stats().resident_bytes
        finally:
            ctx.close()
        # weight bytes one token streams on this route, and their time at the
        # measured copy rate (the calls are host-round-trip bound well above it)
        streamed = int8_bytes + 4 * rows if route == "w8a8" else weight_bytes
        res[route] = {"tok_s": round(1.0 / dt, 1), "ms_per_token": round(dt * 1e3, 3),
                      "us_per_call": round(dt * 1e6 / len(calls), 1), "resident_weight_bytes": int(resident),
                      "weight_bytes_per_token": int(streamed),
                      "hbm_floor_ms": round(streamed / (hbm_gbs * 1e9) * 1e3, 4)}
    res["numerics"] = "w8a8: the reference's W8A8 bits; kq: f32 within 1e-3 of the exact product"
    return res


# Token rows of the CPU samples: the CPU path's cost is linear in the rows,
# so long prompts are timed on their first rows and scaled.
CPU_SAMPLE_ROWS = 512


def cpu_baseline(weights, acts, m, budget_s=10.0):
    """The reference's CPU path (oracle C port, OpenMP) on MUL_MAT calls of the
    workload (the first CPU_SAMPLE_ROWS tokens of each) until the time budget
    is spent; scaled by int8 ops to tok/s of a whole step."""
    import oracle
    oracle.set_threads(oracle.host_threads())
    prepared = []
    for key, blocks in list(weights.items())[:8]:  # two layers' worth of calls
        _, members, k = layer_plan(key[0])[["qkv", "o", "gate_up", "down"].index(key[1])]
        ws, ss = [], []
        for (kind, n), b in zip(members, blocks):
            st, w, s = oracle.prepare_w8a8(kind, b, k, n)
            ws.append(w)
            ss.append(s)
        prepared.append((key, np.concatenate(ws), np.concatenate(ss), k))
    calls = 0
    ops_done = 0
    t0 = time.perf_counter()
    rows = min(m, CPU_SAMPLE_ROWS)
    while True:
        for key, w, s, k in prepared:
            st, _ = oracle.matmul_w8a8(w, s, np.ascontiguousarray(acts[key][:rows]))
            calls += 1
            ops_done += 2 * rows * w.shape[0] * k
            if time.perf_counter() - t0 > budget_s:
                break
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    _, step_ops = algorithmic(m)
    step_s = dt * step_ops / ops_done
    return {"value": round(m / step_s, 2), "unit": "tok/s", "cores": oracle.threads(), "kind": "port",
            "sample": f"{calls} MUL_MAT calls of layers 0-1 on {rows} of {m} tokens (quantize + int32 GEMM on "
                      f"{oracle.gemm_path(rows, HIDDEN, HIDDEN)} + rescale, prepared weights), {dt:.1f} s, scaled by "
                      f"int8 ops to one {LAYERS}-layer step"}


def step_config(m: int, world: int, calls: int) -> dict:
    """The `config` of a model-workload line, the same dict in both arms: N
    replicas of one m-token prompt (N = world)."""
    wbytes = sum(sum(n for _, n in members) * k for layer in range(LAYERS) for _, members, k in layer_plan(layer))
    return {"workload": workload_name(m), "tokens_per_step": m, "global_batch": world * m, "seq_len": m,
            "layers": LAYERS, "calls_per_step": calls, "parallelism": f"replicas{world}",
            "l2": f"inputs > L2: {wbytes / 1e9:.2f} GB resident int8 weights streamed per step"}


def run_reference(args, rank: int, world: int):
    """--impl reference: the reference's CPU implementation of the path (the
    oracle port; the Rust reference has no toolchain here) on every host
    thread this process may use (the OMP_NUM_THREADS=1 that torchrun exports
    is overridden).  Its inputs come from the oracle's own generator, byte for
    byte those of our arm, so this process never loads librocknpu.so.  A step
    is the same job as our arm's step at this world size: `world` replicas of
    the whole workload (every layer's MUL_MAT calls over all m tokens); on N
    GPUs rank 0 alone runs it on the host and the other ranks exit."""
    if rank != 0:
        return None
    import oracle
    oracle.set_threads(oracle.host_threads())
    m = args.tokens
    weights = make_weights(gen=oracle)
    acts = make_activations(m, seed=5000, gen=oracle)
    # prepared once (the reference caches prepared weights), like our arm
    prepared = []
    for key, blocks in weights.items():
        _, members, k = layer_plan(key[0])[["qkv", "o", "gate_up", "down"].index(key[1])]
        ws, ss = [], []
        for (kind, n), b in zip(members, blocks):
            st, w, s = oracle.prepare_w8a8(kind, b, k, n)
            ws.append(w)
            ss.append(s)
        prepared.append((key, np.concatenate(ws), np.concatenate(ss), k))

    # each replica: quantize + exact int32 GEMM + rescale of every call
    def step():
        for _ in range(world):
            for key, w, s, k in prepared:
                oracle.matmul_w8a8(w, s, acts[key])

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    step_s = (time.perf_counter() - t0) / args.steps
    value = round(world * m / step_s, 2)
    line = {
        "impl": "reference",
        "metric": metric_name(m),
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_s * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 (W8A8, int32 accumulate, f32 out)",
        "data": "synthetic (random-init N(0,0.02^2) -> Q4_K/Q6_K weights, N(0,1) activations)",
        "config": step_config(m, world, len(prepared)),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": oracle.threads(), "kind": "port",
                         "sample": f"each step runs all {len(prepared)} MUL_MAT calls of the {LAYERS} layers on "
                                   f"{m} tokens, {world} time(s) (one per replica; the replicas reuse replica 0's "
                                   f"activations), quantize + int32 GEMM on {oracle.gemm_path(m, HIDDEN, HIDDEN)} + "
                                   "rescale on prepared weights"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


# ---------------------------------------------------------------------------
# FP16-executor variant (configs[3]: "the same GEMMs with fp16 weights")
# ---------------------------------------------------------------------------

def f16_calls():
    """(layer, name, member index, n, k) of every FP16-executor call of a step:
    each member of the model's MUL_MATs is one rocknpu_matmul_f16_f32_f32."""
    out = []
    for layer in range(LAYERS):
        for name, members, k in layer_plan(layer):
            for i, (_, n) in enumerate(members):
                out.append((layer, name, i, n, k))
    return out


def run_ours_f16(args, rank: int, world: int):
    """The model's MUL_MATs through the FP16 executor (K4, tcgen05 kind::f16):
    f16 weights ~ N(0, 0.02^2), f32 activations converted to f16 per call."""
    import torch
    import oracle
    import rocknpu_b200 as rk
    from rocknpu_b200 import device as dev

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    m = args.tokens
    hbm_peak, bf16_peak, peak_src = load_peaks()
    calls = f16_calls()
    t0 = time.time()
    w_host, a_host = {}, {}
    for idx, (layer, name, i, n, k) in enumerate(calls):
        w_host[idx] = rk.synth_normal(3000 + idx, n * k, 0.02).astype(np.float16).reshape(n, k)
    for layer in range(LAYERS):
        for name, _, k in layer_plan(layer):
            a_host[(layer, name)] = rk.synth_normal(5000 + 97 * rank + len(a_host), m * k).reshape(m, k)
    gen_s = time.time() - t0
    status = dev.new_status()
    w_dev = {idx: torch.from_numpy(w).cuda() for idx, w in w_host.items()}
    a_dev = {key: torch.from_numpy(a).cuda() for key, a in a_host.items()}
    a16 = {key: torch.empty(a.shape, dtype=torch.float16, device="cuda") for key, a in a_dev.items()}
    outs = {}
    for idx, (layer, name, i, n, k) in enumerate(calls):
        outs.setdefault((name, i), torch.empty((m, n), dtype=torch.float32, device="cuda"))

    def step():
        for key in a_dev:
            dev.convert_f16(a_dev[key], out=a16[key])
        for idx, (layer, name, i, n, k) in enumerate(calls):
            dev.gemm_f16(a16[(layer, name)], w_dev[idx], status, out=outs[(name, i)])

    def gemm_only():
        for idx, (layer, name, i, n, k) in enumerate(calls):
            dev.gemm_f16(a16[(layer, name)], w_dev[idx], status, out=outs[(name, i)])

    def graph_time(fn, reps):
        fn()
        torch.cuda.synchronize()
        g = new_graph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps, graph_kernel_nodes(g)

    with ClockSampler(torch.cuda.current_device()) as clocks:
        clocks.mark("t_start")
        ms, launches = graph_time(step, args.steps)
        clocks.mark("t_end")
    gemm_ms, _ = graph_time(gemm_only, max(5, args.steps))
    assert status.item() == 0
    flops = sum(2 * m * n * k for (_, _, _, n, k) in calls)
    byts = sum(2 * n * k + 2 * m * k + 4 * m * n for (_, _, _, n, k) in calls)
    tf = flops / (gemm_ms * 1e-3) / 1e12
    gbs = byts / (gemm_ms * 1e-3) / 1e9
    bound = "tensor" if flops / (bf16_peak * 1e12) >= byts / (hbm_peak * 1e9) else "hbm"
    roof = {"bound": bound, "achieved": round(tf if bound == "tensor" else gbs, 1),
            "peak": bf16_peak if bound == "tensor" else hbm_peak, "unit": "TFLOP/s" if bound == "tensor" else "GB/s",
            "frac": round(tf / bf16_peak if bound == "tensor" else gbs / hbm_peak, 4), "traffic": None,
            "kernel": "gemm_tc_kernel (K4, tcgen05 kind::f16)", "peak_source": f"{peak_src} bf16_tflops / hbm_gbs",
            "tensor_frac": round(tf / bf16_peak, 4), "hbm_frac": round(gbs / hbm_peak, 4),
            "gemm_ms_per_step": round(gemm_ms, 4), "gemm_launches_per_step": len(calls)}
    e2e = None
    if not args.no_e2e:
        ctx = rk.Context()
        h_a = {}
        for key, a in a_host.items():
            h_a[key] = rk.host_empty(a.shape)
            h_a[key][...] = a
        h_w = {idx: w.view(np.uint16) for idx, w in w_host.items()}
        h_o = {}
        for (_, name, i, n, _) in calls:
            if (name, i) not in h_o:
                h_o[(name, i)] = rk.host_empty((m, n))

        def e2e_step():
            for idx, (layer, name, i, n, k) in enumerate(calls):
                st = ctx.matmul_f16(h_w[idx], h_a[(layer, name)], h_o[(name, i)], m, k, n)
                if st != 0:
                    raise RuntimeError(f"rocknpu_matmul_f16_f32_f32 failed: {st}")
        e2e_step()
        t1 = time.perf_counter()
        e_steps = max(1, min(args.steps, 5))
        for _ in range(e_steps):
            e2e_step()
        e2e_s = (time.perf_counter() - t1) / e_steps
        h2d = sum(4 * m * k for (_, _, _, n, k) in calls)
        d2h = sum(4 * m * n for (_, _, _, n, k) in calls)
        e2e = {"value": round(m / e2e_s, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": round(e2e_s * 1e3, 3),
               "path": "rocknpu_matmul_f16_f32_f32 per member, rocknpu_b200_host_alloc host buffers"}
        ctx.close()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rows = min(m, 128)
        t1 = time.perf_counter()
        done = 0
        sample = [c for c in enumerate(calls)][:7]
        for idx, (layer, name, i, n, k) in sample:
            oracle.matmul_f16(w_host[idx].view(np.uint16), np.ascontiguousarray(a_host[(layer, name)][:rows]))
            done += 2 * rows * n * k
            if time.perf_counter() - t1 > args.cpu_seconds:
                break
        dt = time.perf_counter() - t1
        cpu = {"value": round(m / (dt * flops / done), 3), "unit": "tok/s", "cores": oracle.threads(), "kind": "port",
               "sample": f"FP16 oracle (f64 accumulation, lib.rs:1680-1699) on {rows} tokens of layer 0's calls, "
                         f"{dt:.1f} s, scaled by flops to one {LAYERS}-layer step"}
    return {
        "metric": metric_name(m).replace("Q4_K_M", "FP16-executor"),
        "value": round(m / (ms * 1e-3), 1), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 (f32 accumulate, f32 out)",
        "data": "synthetic (random-init N(0,0.02^2) f16 weights, N(0,1) activations)",
        "config": {"workload": workload_name(m).replace("q4_k_m", "f16"), "tokens_per_step": m, "layers": LAYERS,
                   "calls_per_step": len(calls), "parallelism": "replicas1"},
        "roofline": roof, "e2e": e2e, "cpu_baseline": cpu,
        "gpu_launches": launches * args.steps if launches is not None else None, "launches_per_step": launches,
        "clocks": clocks.summary(), "setup_s": round(gen_s, 1),
    }


# ---------------------------------------------------------------------------
# cfg5: the large-GEMM sharding sweep
# ---------------------------------------------------------------------------

CFG5_N, CFG5_K = 28672, 8192
CFG5_M = (128, 1024, 4096, 16384)


def cfg5_activations(m: int, device="cuda"):
    """X [m, 8192] ~ N(0, 1) with 1 % of the K channels (82, picked by seed 2)
    scaled x20: the outlier channels per-token int8 quantisation must absorb."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(1)
    x = torch.randn(m, CFG5_K, generator=g, device=device)
    ch = torch.from_numpy(np.random.default_rng(2).choice(CFG5_K, CFG5_K // 100, replace=False)).to(device)
    x[:, ch] *= 20.0
    return x


def _timed(fn, steps, warmup, dist):
    """Device time of `steps` calls after `warmup` (CUDA events on the current
    stream, barrier and synchronize on both sides, max over ranks), ms."""
    import torch
    for _ in range(warmup):
        fn()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


# Measured NVLink peer-copy rate per direction on this pool's B200s (GB/s):
# the receive bound of the all-gather.
PEER_GBS = 770.0


def cfg5_block(ms_list, steps, warmup, rank, world, route="peer", check=True):
    """BASELINE.json configs[4] on this process's GPU(s): the Q4_K weight
    N=28672 x K=8192 N-sharded over the ranks (strong scaling: the same GEMMs
    whatever the GPU count), per M one step = K2 quantisation of X on every
    rank + the rank's tcgen05 GEMM + the all-gather of the output columns
    (peer stores fused into the epilogue, or NCCL), so that every rank holds
    Y; the local GEMM alone on pre-quantised X gives the kernel's roofline
    fraction.  Plus the M=1 decode GEMV on the same weight.  With world > 1
    and `check`, sampled rows of the gathered Y on every rank are compared
    bit for bit with a single-GPU GEMM of the whole weight on rank 0.
    Returns (result dict, clock summary) on rank 0, (None, None) elsewhere."""
    import torch
    import rocknpu_b200 as rk
    from rocknpu_b200 import device as dev
    from rocknpu_b200 import shard

    hbm_peak, bf16_peak, peak_src = load_peaks()
    int8_peak = 2.0 * bf16_peak
    dist = None
    if world > 1:
        import torch.distributed as dist
    max_m = max(ms_list)
    t0 = time.time()
    rows = shard.shard_rows(CFG5_N, world)
    start, width = rows[rank]
    # this rank's rows of the seeded N(0, 0.02^2) weight (counter-based
    # generator: rows [start, start + width) are values [start*K, ...))
    vals = rk.synth_normal(0, width * CFG5_K, 0.02, first=start * CFG5_K).reshape(width, CFG5_K)
    blocks = rk.synth_encode(4, vals)
    blocks6 = rk.synth_encode(6, vals)  # the same weight as Q6_K, for the K5b Q6_K GEMV
    del vals
    sm = shard.ShardedMatmul(4, blocks, CFG5_K, CFG5_N, route=route, max_m=max_m, blocks_are_local=True)
    gen_s = time.time() - t0
    res = {"n": CFG5_N, "k": CFG5_K, "weight": "Q4_K, N(0, 0.02^2) seed 0", "rows_per_rank": width,
           "route": route if world > 1 else None, "setup_s": round(gen_s, 1), "gemm": {}}
    clocks = ClockSampler(torch.cuda.current_device())
    with clocks:
        clocks.mark("t_start")
        # M = 1 decode GEMVs first (K5 on int8 rows, K5b on the Q4_K blocks),
        # before the large GEMMs leave the GPU at its power cap
        x1 = cfg5_activations(1)
        gemv_ms = _timed(lambda: sm(x1), max(steps, 20), warmup, dist)
        a8, a_s = sm.quantize(x1)
        o1 = torch.empty(max(width, 1), dtype=torch.float32, device="cuda")
        gemv_local = _timed(lambda: dev.gemv_w8a8(a8, a_s, sm.w8, sm.w_scales, out=o1), max(steps, 50), warmup,
                            dist)
        gbytes = width * CFG5_K + 8 * width + CFG5_K + 4
        res["gemv_w8"] = {"kernel": "gemv_w8a8_kernel (int8 rows, dp4a)", "ms_per_step": round(gemv_ms, 4),
                          "us_local": round(gemv_local * 1e3, 2),
                          "gbs_local": round(gbytes / (gemv_local * 1e-3) / 1e9, 1),
                          "hbm_frac": round(gbytes / (gemv_local * 1e-3) / 1e9 / hbm_peak, 4),
                          "bytes": gbytes}
        # the same M = 1 product straight from this rank's Q4_K blocks (K5b):
        # 144 bytes per 256 weights instead of 256 + scales; then from the
        # same weight encoded as Q6_K (210 bytes per 256 weights)
        if width:
            layout = dev.kq_layout(4, torch.from_numpy(blocks).cuda(), CFG5_K, width)
            xf = x1.reshape(-1).contiguous()
            yq = torch.empty(width, dtype=torch.float32, device="cuda")
            kq_status = dev.new_status()
            kq_ms = _timed(lambda: dev.gemv_kq(4, layout, xf, width, kq_status, out=yq), max(steps, 50), warmup,
                           dist)
            torch.cuda.synchronize()
            assert kq_status.item() == 0, "gemv_kq status error"
            qbytes = layout.numel() + 4 * CFG5_K + 4 * width
            res["gemv_q4k"] = {"kernel": "kq::stage_kernel<Q4Fmt> (Q4_K code and header planes in bulk-copied row stages, codes and scales applied in registers, dp2a)",
                               "us_local": round(kq_ms * 1e3, 2),
                               "gbs_local": round(qbytes / (kq_ms * 1e-3) / 1e9, 1),
                               "hbm_frac": round(qbytes / (kq_ms * 1e-3) / 1e9 / hbm_peak, 4),
                               "bytes": qbytes, "vs_gemv_w8": round(gemv_local / kq_ms, 3)}
            del layout
            # and from Q6_K blocks of the same shape (210 bytes per 256 weights)
            layout = dev.kq_layout(6, torch.from_numpy(blocks6).cuda(), CFG5_K, width)
            q6_ms = _timed(lambda: dev.gemv_kq(6, layout, xf, width, kq_status, out=yq), max(steps, 50), warmup,
                           dist)
            torch.cuda.synchronize()
            assert kq_status.item() == 0, "gemv_kq status error"
            q6bytes = width * (CFG5_K // 256) * 210 + 4 * CFG5_K + 4 * width
            res["gemv_q6k"] = {"kernel": "kq::stage_kernel<Q6Fmt> (Q6_K ql/qh groups and d plane in bulk-copied row stages, dp2a)",
                               "us_local": round(q6_ms * 1e3, 2),
                               "gbs_local": round(q6bytes / (q6_ms * 1e-3) / 1e9, 1),
                               "hbm_frac": round(q6bytes / (q6_ms * 1e-3) / 1e9 / hbm_peak, 4),
                               "bytes": q6bytes}
            del layout, yq
            # K1 on the same rows (once per weight, at load time): Q4_K and
            # Q6_K blocks -> int8 rows + per-row scales
            pw = torch.empty((width, CFG5_K), dtype=torch.int8, device="cuda")
            ps = torch.empty(width, dtype=torch.float32, device="cuda")
            pst = dev.new_status()
            for kind, hb, bb, name in ((4, blocks, 144, "prep_q4k"), (6, blocks6, 210, "prep_q6k")):
                db = torch.from_numpy(hb).cuda()

                def prep(kind=kind, db=db):
                    return rk.lib().rocknpu_b200_prepare_w8(kind, db.data_ptr(), CFG5_K, width, pw.data_ptr(),
                                                            ps.data_ptr(), pst.data_ptr(),
                                                            torch.cuda.current_stream().cuda_stream)

                p_ms = _timed(prep, max(steps, 10), warmup, dist)
                torch.cuda.synchronize()
                assert pst.item() == 0, "prepare_w8 status error"
                pbytes = width * (CFG5_K // 256) * bb + width * CFG5_K + 4 * width
                res[name] = {"kernel": "prep_w8_q4k_lut_kernel (a thread per sub-block, 16-entry byte tables)"
                             if kind == 4 else "prep_w8_reg_kernel (dequantise in registers, absmax, int8)",
                             "us_local": round(p_ms * 1e3, 1),
                             "gbs_local": round(pbytes / (p_ms * 1e-3) / 1e9, 1),
                             "hbm_frac": round(pbytes / (p_ms * 1e-3) / 1e9 / hbm_peak, 4),
                             "bytes": pbytes}
                del db
            del pw, ps
        for m in ms_list:
            x = cfg5_activations(m)
            ms = _timed(lambda: sm(x), steps, warmup, dist)
            a8, a_s = sm.quantize(x)
            local = torch.empty((m, max(width, 1)), dtype=torch.float32, device="cuda")
            gemm_ms = _timed(lambda: dev.gemm_w8a8(a8, a_s, sm.w8, sm.w_scales, sm.status, out=local),
                             steps, warmup, dist)
            sm.check()
            ops = 2.0 * m * CFG5_N * CFG5_K
            local_ops = 2.0 * m * width * CFG5_K
            local_bytes = width * CFG5_K + m * CFG5_K + 4 * m * width + 4 * width + 4 * m
            tops_local = local_ops / (gemm_ms * 1e-3) / 1e12
            gbs_local = local_bytes / (gemm_ms * 1e-3) / 1e9
            bound = "tensor" if local_ops / (int8_peak * 1e12) >= local_bytes / (hbm_peak * 1e9) else "hbm"
            r = {"ms_per_step": round(ms, 4), "tops": round(ops / (ms * 1e-3) / 1e12, 1),
                 "gemm_ms_local": round(gemm_ms, 4), "gemm_tops_local": round(tops_local, 1),
                 "bound": bound,
                 "frac": round(tops_local / int8_peak if bound == "tensor" else gbs_local / hbm_peak, 4),
                 "tensor_frac": round(tops_local / int8_peak, 4), "hbm_frac": round(gbs_local / hbm_peak, 4)}
            if world > 1:
                recv = 4 * m * (CFG5_N - width)
                recv_ms = recv / (PEER_GBS * 1e9) * 1e3
                r.update({"recv_bytes_per_rank": recv, "recv_bound_ms": round(recv_ms, 4),
                          "floor_ms": round(max(recv_ms, gemm_ms), 4),
                          "job_vs_floor": round(max(recv_ms, gemm_ms) / ms, 4)})
            res["gemm"][str(m)] = r
            del x, a8, a_s, local
        clocks.mark("t_end")
    sm.check()
    if world > 1 and check:
        res["bitexact"] = _cfg5_shard_check(sm, max_m, rank, world, dist)
    sm.close()
    res["peak_source"] = f"{peak_src}: int8 = 2 x bf16_tflops {int8_peak:.0f} TOP/s, hbm_gbs {hbm_peak:.0f}"
    if rank != 0:
        return None, None
    return res, clocks.summary()


def _cfg5_shard_check(sm, m, rank, world, dist):
    """Sampled rows of the all-gathered Y: identical bits on every rank, and
    equal to a single-GPU GEMM of the whole weight on rank 0."""
    import torch
    import rocknpu_b200 as rk
    from rocknpu_b200 import device as dev
    x = cfg5_activations(m)
    y = sm(x)
    sample = torch.arange(0, m, max(1, m // 256), device="cuda")[:256]
    ys = y.index_select(0, sample).contiguous()
    sm.check()
    h = ys.view(torch.int32).to(torch.int64)
    sig = torch.stack([h.sum(), (h * torch.arange(1, h.shape[1] + 1, device="cuda")).sum()])
    sigs = [torch.empty_like(sig) for _ in range(world)]
    dist.all_gather(sigs, sig)
    same_on_ranks = all(torch.equal(s_, sigs[0]) for s_ in sigs)
    ok = torch.tensor([1], device="cuda")
    if rank == 0:
        vals = rk.synth_normal(0, CFG5_N * CFG5_K, 0.02).reshape(CFG5_N, CFG5_K)
        blocks = torch.from_numpy(rk.synth_encode(4, vals)).cuda()
        del vals
        status = dev.new_status()
        w8, ws = dev.prepare_w8(4, blocks, CFG5_K, CFG5_N, status)
        xs = x.index_select(0, sample).contiguous()
        a8, a_s = dev.quantize_rows(xs, status)
        ref = torch.empty((xs.shape[0], CFG5_N), dtype=torch.float32, device="cuda")
        dev.gemm_w8a8(a8, a_s, w8, ws, status, out=ref)
        torch.cuda.synchronize()
        ok[0] = int(status.item() == 0 and torch.equal(ref.view(torch.int32), ys.view(torch.int32)))
        del blocks, w8, ws, ref
    dist.broadcast(ok, 0)
    return {"rows_checked": int(sample.numel()), "m": m, "same_on_every_rank": bool(same_on_ranks),
            "equal_to_single_gpu": bool(ok.item()), "ok": bool(same_on_ranks and ok.item())}


def run_cfg5(args, rank: int, world: int):
    """--workload cfg5: the sweep of BASELINE.json configs[4] as its own line
    (whole-job TOP/s at the largest M is the value)."""
    import torch
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    ms_list = [int(v) for v in args.m_list.split(",")]
    res, clocks = cfg5_block(ms_list, args.steps, args.warmup, rank, world, route=args.route,
                             check=not args.no_check)
    if rank != 0:
        return None
    m = max(ms_list)
    r = res["gemm"][str(m)]
    hbm_peak, bf16_peak, peak_src = load_peaks()
    int8_peak = 2.0 * bf16_peak
    line = {
        "metric": f"W8A8 GEMM TOPS (cfg5 Q4_K N={CFG5_N} K={CFG5_K}, M={m}, N-sharded, Y all-gathered)",
        "value": r["tops"], "unit": "TOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8 (W8A8, int32 accumulate, f32 out)",
        "data": "synthetic (seeded N(0,0.02^2) -> Q4_K weights; N(0,1) activations, 1% channels x20)",
        "config": {"workload": "cfg5-large-gemm-sharding-sweep", "n": CFG5_N, "k": CFG5_K, "m_list": ms_list,
                   "parallelism": f"nshard{world}" + (f"-{args.route}" if world > 1 else ""),
                   "l2": "weights 235 MB int8 > L2 (streamed every step)"},
        "roofline": {"bound": r["bound"], "achieved": r["gemm_tops_local"], "peak": int8_peak, "unit": "TOP/s",
                     "frac": r["tensor_frac"], "traffic": None,
                     "kernel": "gemm_tc_kernel / gemm_pair_kernel (K3, tcgen05 kind::i8), this rank's rows",
                     "peak_source": f"{peak_src} (int8 = 2 x bf16_tflops)"},
        "sweep": res,
        "e2e": None,
        "cpu_baseline": None,
        "gpu_launches": None,
        "clocks": clocks,
    }
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=None, help="prompt tokens (default: the model's config)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-short", action="store_true", help="skip the pp128 companion measurement")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--workload", choices=list(MODELS) + ["cfg5"], default="tinyllama")
    ap.add_argument("--route", choices=["peer", "allgather"], default="peer",
                    help="cfg5 output exchange at N > 1")
    ap.add_argument("--m-list", default=",".join(str(m) for m in CFG5_M))
    ap.add_argument("--no-check", action="store_true", help="cfg5 at N > 1: skip the in-run bit check")
    ap.add_argument("--no-decode", action="store_true", help="skip the M=1 decode-token measurement")
    ap.add_argument("--no-cfg5", action="store_true",
                    help="default workload: skip the cfg5 GEMM/GEMV block (N=1) or the sharded block (N>1)")
    ap.add_argument("--f16", action="store_true", help="model workloads through the FP16 executor (one GPU)")
    args = ap.parse_args()
    if args.workload in MODELS:
        set_model(args.workload)
        if args.tokens is None:
            args.tokens = MODELS[args.workload]["tokens"]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        if args.impl == "reference":
            line = run_reference(args, rank, world)
        elif args.workload == "cfg5":
            line = run_cfg5(args, rank, world)
        elif args.f16:
            line = run_ours_f16(args, rank, world) if rank == 0 else None
        else:
            line = run_ours(args, rank, world)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
