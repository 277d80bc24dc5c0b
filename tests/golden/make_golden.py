"""Generate the committed golden fixtures for the K-quant / W8 path.

Run in a container that has the reference tree and gguf-py installed:

    python tests/golden/make_golden.py /path/to/RockNPU

Outputs (all small, seeded, deterministic):

* ``kquant_dequant.npz`` -- random Q4_K / Q5_K / Q6_K superblocks and their
  f32 dequantisation by gguf-py 0.19.0 (``gguf.quants.dequantize``), the
  published restatement of the block formats that the reference's
  third-party ``llama-gguf`` crate decodes (capi/src/lib.rs:5,732-733,986-988).
* ``w8_sidecar.npz`` -- per-row int8 weights and scales produced by the
  reference's own ``scripts/make_tinyllama_w8_sidecar_gguf.py::quantize_rows``
  (imported from the reference tree, run on the gguf-py dequantised rows).
  The plugin documents that sidecar as identical to its in-process
  conversion (ggml-rocknpu.cpp:160-163).
* ``sidecar_fnv.npz`` -- the sampled FNV-1a-64 source fingerprints of the
  W8 sidecar format, computed by the reference script's own
  ``source_sample_fnv1a64`` (the plugin's rocknpu_source_sample_fingerprint,
  ggml-rocknpu.cpp:123-146, must agree with it) for seeded byte arrays of
  every size class (whole-array and three-sample cases), and the complete
  sidecar files (``.w8``, ``.scale.f32``, ``.source.fnv1a64``) the script
  writes for a small Q4_K and Q6_K tensor.
* ``act_quant.npz`` -- the tie-heavy activation vector of the reference's
  quantisation test (capi/src/lib.rs:5680-5700: literal ties plus an LCG
  stream) with its int8 values and scale, computed here with an independent
  numpy restatement of ``quantize_symmetric_into`` (capi/src/lib.rs:614-654).
"""
from __future__ import annotations

import importlib.util
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def random_kquant_blocks(kind: int, nblocks: int, rng: np.random.Generator) -> np.ndarray:
    """Random but finite K-quant superblocks (every code path of the formats)."""
    size = {4: 144, 5: 176, 6: 210}[kind]
    blocks = rng.integers(0, 256, size=(nblocks, size), dtype=np.uint8)
    # finite fp16 super-scales of realistic and edge magnitudes
    mags = np.concatenate([
        rng.uniform(1e-4, 2e-2, size=nblocks - 4),
        np.array([0.0, 6.0e-8, 1.0, 65504.0 / 4096]),  # zero, fp16 subnormal, large
    ]).astype(np.float32)
    signs = np.where(rng.random(nblocks) < 0.1, -1.0, 1.0).astype(np.float32)
    d = (mags * signs).astype(np.float16)
    dmin = rng.uniform(0.0, 1e-2, size=nblocks).astype(np.float16)
    if kind in (4, 5):
        blocks[:, 0:2] = d.view(np.uint8).reshape(nblocks, 2)
        blocks[:, 2:4] = dmin.view(np.uint8).reshape(nblocks, 2)
    else:
        blocks[:, 208:210] = d.view(np.uint8).reshape(nblocks, 2)
    return blocks


def round_half_away(x: np.ndarray) -> np.ndarray:
    """Rust f32::round, exactly (f32 truncation + exact fractional part)."""
    t = np.trunc(x)
    frac = (x - t).astype(np.float32)  # exact for |x| < 2**23
    return (t + np.where(np.abs(frac) >= np.float32(0.5), np.sign(x), 0)).astype(np.float32)


def quantize_symmetric_np(values: np.ndarray):
    values = values.astype(np.float32)
    max_abs = np.float32(np.max(np.abs(values))) if values.size else np.float32(0)
    scale = np.float32(1.0) if max_abs == 0 else np.float32(max_abs / np.float32(127.0))
    q = np.clip(round_half_away((values / scale).astype(np.float32)), -127, 127).astype(np.int8)
    return q, scale


def tie_vector() -> np.ndarray:
    values = [-12.75, -7.5, -3.5, -1.5, -0.5, -0.49999997, 0.0, 0.49999997, 0.5, 1.5, 3.5, 7.5, 12.75]
    values = [np.float32(v) for v in values]
    state = 0x12345678
    for _ in range(2051):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        unit = np.float32(np.float32(state >> 8) / np.float32((1 << 24) - 1))
        values.append(np.float32((unit * np.float32(2.0) - np.float32(1.0)) * np.float32(17.0)))
    return np.array(values, dtype=np.float32)


def load_sidecar_script(ref_root: str):
    spec = importlib.util.spec_from_file_location(
        "rocknpu_sidecar", os.path.join(ref_root, "scripts", "make_tinyllama_w8_sidecar_gguf.py"))
    sidecar = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sidecar)
    return sidecar


FNV_SIZES = (1, 100, 4095, 4096, 12287, 12288, 12289, 13824, 30000, 100003)


def fnv_fixture(ref_root: str) -> None:
    from gguf import GGMLQuantizationType, dequantize
    sidecar = load_sidecar_script(ref_root)
    rng = np.random.default_rng(77)
    out = {"sizes": np.array(FNV_SIZES, dtype=np.int64)}
    hexes = []
    for size in FNV_SIZES:
        data = rng.integers(0, 256, size=size, dtype=np.uint8)
        hexes.append(sidecar.source_sample_fnv1a64(data))
    out["fnv_hex"] = np.array(hexes)
    # whole sidecar files of two small tensors
    for kind, qt in ((4, GGMLQuantizationType.Q4_K), (6, GGMLQuantizationType.Q6_K)):
        n, k = 20, 512
        blocks = random_kquant_blocks(kind, n * k // 256, rng)
        rows = dequantize(blocks.reshape(-1), qt).astype(np.float32).reshape(n, k)
        with tempfile.TemporaryDirectory() as tmp:
            base = os.path.join(tmp, "blk.0.t.weight")
            sidecar.quantize_rows(rows, __import__("pathlib").Path(base), 8)
            out[f"q{kind}_blocks"] = blocks
            out[f"q{kind}_w8_file"] = np.fromfile(base + ".w8", dtype=np.uint8)
            out[f"q{kind}_scale_file"] = np.fromfile(base + ".scale.f32", dtype=np.uint8)
            out[f"q{kind}_fnv_file"] = np.frombuffer(
                (sidecar.source_sample_fnv1a64(blocks.reshape(-1)) + "\n").encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "sidecar_fnv.npz"), **out)


def main() -> None:
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ROCKNPU_REFERENCE", "")
    if "--only" in sys.argv:
        which = sys.argv[sys.argv.index("--only") + 1]
        {"fnv": fnv_fixture}[which](ref_root)
        print("wrote", which, "fixture to", HERE)
        return
    from gguf import GGMLQuantizationType, dequantize

    rng = np.random.default_rng(20261201)
    kinds = {4: GGMLQuantizationType.Q4_K, 5: GGMLQuantizationType.Q5_K, 6: GGMLQuantizationType.Q6_K}
    out = {}
    for kind, qt in kinds.items():
        blocks = random_kquant_blocks(kind, 48, rng)
        deq = dequantize(blocks.reshape(-1), qt).astype(np.float32).reshape(-1)
        out[f"q{kind}_blocks"] = blocks
        out[f"q{kind}_dequant"] = deq
    np.savez_compressed(os.path.join(HERE, "kquant_dequant.npz"), **out)

    # W8 preparation through the reference's own sidecar quantiser.
    sidecar = load_sidecar_script(ref_root)
    w8 = {}
    n, k = 24, 1024
    for kind, qt in kinds.items():
        blocks = random_kquant_blocks(kind, n * k // 256, rng)
        # make each row's blocks share a realistic magnitude, keep edge rows
        rows = dequantize(blocks.reshape(-1), qt).astype(np.float32).reshape(n, k)
        with tempfile.TemporaryDirectory() as tmp:
            base = os.path.join(tmp, "t")
            sidecar.quantize_rows(rows, __import__("pathlib").Path(base), 8)
            wq = np.fromfile(base + ".w8", dtype=np.int8).reshape(n, k)
            ws = np.fromfile(base + ".scale.f32", dtype=np.float32)
        w8[f"q{kind}_blocks"] = blocks
        w8[f"q{kind}_w8"] = wq
        w8[f"q{kind}_scale"] = ws
        w8[f"q{kind}_shape"] = np.array([n, k], dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "w8_sidecar.npz"), **w8)

    ties = tie_vector()
    q, s = quantize_symmetric_np(ties)
    rows = rng.standard_normal((8, 512)).astype(np.float32)
    rows[1, :] = 0.0  # all-zero row -> scale 1.0
    rows[2, 7] = 300.0  # outlier channel
    qr = np.stack([quantize_symmetric_np(r)[0] for r in rows])
    sr = np.array([quantize_symmetric_np(r)[1] for r in rows], dtype=np.float32)
    np.savez_compressed(os.path.join(HERE, "act_quant.npz"), ties=ties, ties_q=q,
                        ties_scale=np.array([s], dtype=np.float32), rows=rows, rows_q=qr, rows_scale=sr)
    fnv_fixture(ref_root)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
