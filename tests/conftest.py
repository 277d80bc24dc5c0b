"""Shared test setup: the `gpu` marker, in-tree builds, and seeded inputs."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")


def _have_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _have_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session", autouse=True)
def built_artifacts():
    """Build librocknpu.so and the oracle when stale (nvcc / gcc are present
    in this image; on the GPU box the prebuilt files are used)."""
    import shutil
    import oracle
    if shutil.which("gcc") or os.path.exists("/usr/bin/gcc"):
        try:
            oracle.build()
        except Exception:
            pass
    from rocknpu_b200 import build as b
    if shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc"):
        try:
            b.build()
        except Exception:
            if not os.path.exists(b.LIB):
                raise
    yield


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


def random_kquant_blocks(kind: int, nblocks: int, rng) -> np.ndarray:
    """Random finite K-quant superblocks exercising every bit of the format."""
    size = {4: 144, 5: 176, 6: 210}[kind]
    blocks = rng.integers(0, 256, size=(nblocks, size), dtype=np.uint8)
    d = (rng.uniform(1e-4, 2e-2, size=nblocks) * np.where(rng.random(nblocks) < 0.1, -1, 1)).astype(np.float16)
    dmin = rng.uniform(0.0, 1e-2, size=nblocks).astype(np.float16)
    if kind in (4, 5):
        blocks[:, 0:2] = d.view(np.uint8).reshape(nblocks, 2)
        blocks[:, 2:4] = dmin.view(np.uint8).reshape(nblocks, 2)
    else:
        blocks[:, 208:210] = d.view(np.uint8).reshape(nblocks, 2)
    return blocks.reshape(-1)
