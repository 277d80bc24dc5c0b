"""Build librocknpu.so (the C ABI + sm_100a kernels) in-tree with nvcc.

    python -m rocknpu_b200.build [--force]

Objects go to rocknpu_b200/_build/, the library to rocknpu_b200/librocknpu.so.
The CUDA runtime is linked statically and the driver is reached through
cudaGetDriverEntryPointByVersion, so the library loads (and reports zero
devices) on a machine without a GPU.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB = os.path.join(HERE, "librocknpu.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
              "--expt-relaxed-constexpr", "-I", INCLUDE]
SOURCES = ["quant.cu", "gemm.cu", "gemm_plain.cu", "gemm_fused.cu", "gemm_gather.cu", "gemm_pair.cu", "gemv.cu", "gemv_kq.cu", "gemv_q4k.cu", "gemv_q6k.cu", "noalloc.cu", "shard.cu", "capi.cpp", "plugin_rules.cpp", "sidecar.cpp", "synth.cpp", "hostmem.cpp", "plugin_graph.cpp"]
HEADERS = ["kernels.h", "ptx.cuh", "quant_math.cuh", "gemm_kernel.cuh", "gemv_stage.cuh"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: librocknpu.so cannot be built")


def _newest_header() -> float:
    paths = [os.path.join(CSRC, h) for h in HEADERS]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return max(os.path.getmtime(p) for p in paths)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdr = _newest_header()
    objs, jobs = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr):
            lang = [] if src.endswith(".cu") else ["-x", "cu"] if src in ("capi.cpp",) else []
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *lang, "-c", s, "-o", o]
            if src.startswith("gemm_"):
                cmd += ["-Xptxas", "-v"] if verbose else []
            jobs.append(cmd)
    if jobs:
        with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            results = list(ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs))
        for cmd, r in zip(jobs, results):
            if verbose and r.stderr:
                sys.stderr.write(r.stderr)
            if r.returncode != 0:
                sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
                raise RuntimeError(f"nvcc failed for {cmd[-3]}")
    if jobs or not os.path.exists(LIB):
        link = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(" ".join(link) + "\n" + r.stdout + r.stderr)
            raise RuntimeError("link of librocknpu.so failed")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
