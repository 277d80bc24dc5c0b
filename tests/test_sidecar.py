"""W8 sidecar files (the plugin's disk cache of prepared weights).

Pinned by tests/golden/sidecar_fnv.npz, made by the reference's own
scripts/make_tinyllama_w8_sidecar_gguf.py (source_sample_fnv1a64 and
quantize_rows, imported from the reference tree by make_golden.py): the
fingerprint for every size class, and whole sidecar files for a Q4_K and a
Q6_K tensor.  CPU: fingerprint, writer and reader (including every rejection
of rocknpu_w8_sidecar_get, ggml-rocknpu.cpp:212-243).  GPU: the K1 preparation
reproduces the script's files byte for byte, and the lookup prefers a valid
sidecar over preparing.
"""
import os

import numpy as np
import pytest

import oracle
import rocknpu_b200 as rk
from rocknpu_b200 import sidecar

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = np.load(os.path.join(HERE, "golden", "sidecar_fnv.npz"))


def _fnv_inputs():
    rng = np.random.default_rng(77)
    return [rng.integers(0, 256, size=int(size), dtype=np.uint8) for size in FIX["sizes"]]


def test_fingerprint_matches_reference_script():
    for data, want in zip(_fnv_inputs(), FIX["fnv_hex"]):
        assert f"{sidecar.source_fingerprint(data):016x}" == str(want)
        assert f"{oracle.source_fingerprint(data):016x}" == str(want)


def test_fingerprint_random_sizes_against_oracle():
    rng = np.random.default_rng(3)
    for size in [0, 2, 8191, 12288, 12289, 20000, 1 << 20]:
        data = rng.integers(0, 256, size=size, dtype=np.uint8)
        assert sidecar.source_fingerprint(data) == oracle.source_fingerprint(data)


@pytest.mark.parametrize("kind", [4, 6])
def test_writer_reproduces_reference_files(tmp_path, kind):
    blocks = FIX[f"q{kind}_blocks"]
    w8 = FIX[f"q{kind}_w8_file"].view(np.int8).reshape(20, 512)
    scales = FIX[f"q{kind}_scale_file"].view(np.float32)
    name = "blk.0.t.weight"
    sidecar.write_sidecar(str(tmp_path), name, blocks, w8, scales)
    base = os.path.join(str(tmp_path), name)
    for ext, key in ((".w8", "w8_file"), (".scale.f32", "scale_file"), (".source.fnv1a64", "fnv_file")):
        assert np.array_equal(np.fromfile(base + ext, dtype=np.uint8), FIX[f"q{kind}_{key}"]), ext


def test_reader_accepts_valid_and_rejects_every_bad_case(tmp_path):
    blocks = FIX["q4_blocks"]
    w8 = FIX["q4_w8_file"].view(np.int8).reshape(20, 512)
    scales = FIX["q4_scale_file"].view(np.float32)
    d = str(tmp_path)
    name = "blk.3.ffn_up.weight"
    sidecar.write_sidecar(d, name, blocks, w8, scales)
    got = sidecar.read_sidecar(d, name, blocks, 512, 20)
    assert got is not None and np.array_equal(got[0], w8) and np.array_equal(got[1], scales)
    # a different source (a sampled byte changed) is stale
    other = blocks.copy().reshape(-1)
    other[10] ^= 1
    assert sidecar.read_sidecar(d, name, other, 512, 20) is None
    # wrong shape -> wrong file sizes
    assert sidecar.read_sidecar(d, name, blocks, 512, 19) is None
    assert sidecar.read_sidecar(d, name, blocks, 256, 20) is None
    # missing tensor
    assert sidecar.read_sidecar(d, "blk.9.attn_q.weight", blocks, 512, 20) is None
    # a non-positive or non-finite scale invalidates the sidecar
    base = os.path.join(d, name)
    for bad in (0.0, -1.0, np.nan, np.inf):
        s2 = scales.copy()
        s2[5] = bad
        s2.tofile(base + ".scale.f32")
        assert sidecar.read_sidecar(d, name, blocks, 512, 20) is None
    scales.tofile(base + ".scale.f32")
    # a malformed fingerprint file
    with open(base + ".source.fnv1a64", "w") as f:
        f.write("xyz\n")
    assert sidecar.read_sidecar(d, name, blocks, 512, 20) is None
    # uppercase hex is accepted (strtoull base 16 in the plugin)
    with open(base + ".source.fnv1a64", "w") as f:
        f.write(f"{sidecar.source_fingerprint(blocks):016X}\n")
    assert sidecar.read_sidecar(d, name, blocks, 512, 20) is not None
    # the writer refuses invalid scales
    with pytest.raises(RuntimeError):
        sidecar.write_sidecar(d, name, blocks, w8, np.zeros(20, dtype=np.float32))


def test_lookup_without_dir_or_conversion_returns_none(monkeypatch):
    monkeypatch.delenv("ROCKNPU_W8_SIDECAR_DIR", raising=False)
    monkeypatch.setenv("ROCKNPU_W8_CONVERT", "0")
    assert sidecar.prepared_w8("blk.0.x", 4, FIX["q4_blocks"], 512, 20) is None


# ---- GPU ------------------------------------------------------------------------

@pytest.mark.gpu
@pytest.mark.parametrize("kind", [4, 6])
def test_gpu_preparation_reproduces_reference_sidecar(kind):
    w8, scales = sidecar.prepare_on_gpu(kind, FIX[f"q{kind}_blocks"], 512, 20)
    assert np.array_equal(w8.view(np.uint8).reshape(-1), FIX[f"q{kind}_w8_file"])
    assert np.array_equal(scales.view(np.uint8), FIX[f"q{kind}_scale_file"])


@pytest.mark.gpu
def test_lookup_prefers_valid_sidecar_then_prepares(tmp_path, monkeypatch):
    blocks = FIX["q6_blocks"]
    name = "blk.1.attn_v.weight"
    w8, scales = sidecar.prepare_on_gpu(6, blocks, 512, 20)
    marked = w8.copy()
    marked[0, 0] = 77  # a recognisable sidecar, same sizes and fingerprint
    sidecar.write_sidecar(str(tmp_path), name, blocks, marked, scales)
    monkeypatch.setenv("ROCKNPU_W8_SIDECAR_DIR", str(tmp_path))
    monkeypatch.delenv("ROCKNPU_W8_CONVERT", raising=False)
    got = sidecar.prepared_w8(name, 6, blocks, 512, 20)
    assert got is not None and got[0][0, 0] == 77
    # stale sidecar -> prepared on the GPU
    other = blocks.copy().reshape(-1)
    other[-1] ^= 0x10
    got = sidecar.prepared_w8(name, 6, other, 512, 20)
    ref = sidecar.prepare_on_gpu(6, other, 512, 20)
    assert got is not None and np.array_equal(got[0], ref[0]) and np.array_equal(got[1], ref[1])
    # conversion off and no valid sidecar -> None
    monkeypatch.setenv("ROCKNPU_W8_CONVERT", "0")
    assert sidecar.prepared_w8(name, 6, other, 512, 20) is None
