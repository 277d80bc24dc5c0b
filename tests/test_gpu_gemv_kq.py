"""K5b: the decode GEMV that reads Q4_K / Q6_K blocks directly, against the
oracle's f32 dequantisation (gguf-pinned, tests/golden) times x.

Tolerance (north_star: the f32 output within 1e-3 relative): each output
must satisfy |y - ref| <= 1e-3 * |ref| + 2e-5 * sum_k |w_k x_k|, with ref the
f64 dot product of the oracle's f32 weights and x.  The second term only
matters where the dot product cancels (|ref| << sum |w x|); f32 accumulation
error is proportional to sum |w x|, and the kernel's measured error is about
1e-6 of it (asserted on the median as well).
"""
import numpy as np
import pytest

import oracle
import rocknpu_b200 as rk
from conftest import random_kquant_blocks

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _check(y, w, x):
    ref = w.astype(np.float64) @ x.astype(np.float64)
    mag = np.abs(w).astype(np.float64) @ np.abs(x).astype(np.float64)
    err = np.abs(y.astype(np.float64) - ref)
    bound = 1e-3 * np.abs(ref) + 2e-5 * mag
    bad = np.nonzero(err > bound)[0]
    assert bad.size == 0, f"{bad.size} rows outside the bound, first {bad[:5]}: {err[bad[:5]]} > {bound[bad[:5]]}"
    assert np.median(err / np.maximum(mag, 1e-30)) < 1e-5


def _run(kind, blocks, k, n, x):
    from rocknpu_b200 import device as dev
    d_blocks = torch.from_numpy(blocks).cuda()
    layout = dev.kq_layout(kind, d_blocks, k, n)
    status = dev.new_status()
    y = dev.gemv_kq(kind, layout, torch.from_numpy(x).cuda(), n, status)
    torch.cuda.synchronize()
    assert status.item() == 0
    return y.cpu().numpy()


@pytest.mark.parametrize("kind,k,n", [(4, 2048, 256), (4, 2048, 2560), (4, 5632, 2048), (4, 8192, 1003),
                                      (4, 256, 13), (4, 16384, 77), (6, 2048, 256), (6, 5632, 2048),
                                      (6, 8192, 1003), (6, 256, 9), (6, 12288, 40), (6, 24576, 9)])
def test_gemv_kq_random_blocks(rng, kind, k, n):
    """Random block bytes: every code, scale, min and sign of d."""
    blocks = random_kquant_blocks(kind, n * (k // 256), rng)
    x = rng.standard_normal(k).astype(np.float32)
    x[rng.choice(k, max(1, k // 100), replace=False)] *= 20.0  # outlier channels, as in configs[4]
    y = _run(kind, blocks, k, n, x)
    w = oracle.dequant(kind, blocks).reshape(n, k)
    _check(y, w, x)


@pytest.mark.parametrize("kind,k,n", [(4, 2048, 5632), (6, 2048, 2048), (6, 5632, 2048)])
def test_gemv_kq_model_weights(kind, k, n):
    """N(0, 0.02^2) weights encoded like the bench's (TinyLlama decode shapes)."""
    blocks = rk.synth_q_weights(kind, n, k, seed=300 + kind)
    x = rk.synth_normal(301, k)
    y = _run(kind, blocks, k, n, x)
    _check(y, oracle.dequant(kind, blocks).reshape(n, k), x)


def _q4k_head(h):
    """ggml Q4_K header bytes [b, 16] -> the decode layout's header: d, dmin
    unchanged, then per sub-block pair g the 24-bit value
    sc[2g] | sc[2g+1] << 6 | m[2g] << 12 | m[2g+1] << 18 at bytes 4 + 3g."""
    s = h[:, 4:16].astype(np.uint32)
    sc = np.zeros((h.shape[0], 8), np.uint32)
    mn = np.zeros((h.shape[0], 8), np.uint32)
    for j in range(4):
        sc[:, j] = s[:, j] & 63
        mn[:, j] = s[:, j + 4] & 63
        sc[:, j + 4] = (s[:, j + 8] & 15) | ((s[:, j] >> 6) << 4)
        mn[:, j + 4] = (s[:, j + 8] >> 4) | ((s[:, j + 4] >> 6) << 4)
    out = h.copy()
    for g in range(4):
        v = sc[:, 2 * g] | (sc[:, 2 * g + 1] << 6) | (mn[:, 2 * g] << 12) | (mn[:, 2 * g + 1] << 18)
        for i in range(3):
            out[:, 4 + 3 * g + i] = (v >> (8 * i)) & 255
    return out


def test_q6k_decode_layout_bytes(rng):
    """The Q6_K decode layout is 208 bytes per block (four 48-byte groups of
    ql / qh bytes, then the 16 scales regrouped per group), then the f16 d of
    every block and 16 bytes of padding."""
    from rocknpu_b200 import device as dev
    k, n = 1280, 7
    blocks = random_kquant_blocks(6, n * (k // 256), rng)
    lay = dev.kq_layout(6, torch.from_numpy(blocks).cuda(), k, n).cpu().numpy()
    b = blocks.reshape(-1, 210)
    nbt = b.shape[0]
    assert lay.size == nbt * 210 + 16
    body = np.zeros((nbt, 208), np.uint8)
    for G in range(4):
        h, c = G >> 1, G & 1
        body[:, 48 * G:48 * G + 16] = b[:, 64 * h + 16 * c:64 * h + 16 * c + 16]
        body[:, 48 * G + 16:48 * G + 32] = b[:, 64 * h + 32 + 16 * c:64 * h + 48 + 16 * c]
        body[:, 48 * G + 32:48 * G + 48] = b[:, 128 + 32 * h + 16 * c:128 + 32 * h + 16 * c + 16]
        for t in range(4):
            body[:, 192 + 4 * G + t] = b[:, 192 + 8 * h + c + 2 * t]
    assert np.array_equal(lay[:nbt * 208].reshape(-1, 208), body)
    assert np.array_equal(lay[nbt * 208:nbt * 210].reshape(-1, 2), b[:, 208:])


@pytest.mark.parametrize("k", [1280, 2560, 4096])
def test_q4k_decode_layout_bytes(rng, k):
    """Q4_K: two planes.  The code plane keeps each row's 128 * nb qs bytes,
    regrouped per step of 8 blocks (a short last step has nbs < 8): chunk j
    (qs bytes 16j .. 16j + 15) of the step's block i goes to 16-byte slot
    (j % 2) * 4 nbs + 4 i + j // 2.  Then a 16-byte header per block (d,
    dmin, and the scales and mins regrouped per sub-block pair)."""
    from rocknpu_b200 import device as dev
    n, nb = 7, k // 256
    b4 = random_kquant_blocks(4, n * nb, rng)
    lay4 = dev.kq_layout(4, torch.from_numpy(b4).cuda(), k, n).cpu().numpy()
    b4 = b4.reshape(n, nb, 144)
    assert lay4.size == b4.size
    want = np.zeros((n, nb * 8, 16), np.uint8)
    for b in range(nb):
        t, i = divmod(b, 8)
        nbs = min(8, nb - 8 * t)
        for j in range(8):
            want[:, 64 * t + (j % 2) * 4 * nbs + 4 * i + j // 2] = b4[:, b, 16 + 16 * j:32 + 16 * j]
    assert np.array_equal(lay4[:n * nb * 128].reshape(n, nb * 8, 16), want)
    assert np.array_equal(lay4[n * nb * 128:].reshape(-1, 16), _q4k_head(b4.reshape(-1, 144)[:, :16]))


def test_gemv_kq_rejects_bad_arguments():
    L = rk.lib()
    assert L.rocknpu_b200_kq_layout_bytes(5, 256, 1) == 0
    assert L.rocknpu_b200_kq_layout_bytes(4, 100, 1) == 0
    x = torch.zeros(512, device="cuda")
    y = torch.zeros(4, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    lay = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    assert L.rocknpu_b200_gemv_kq(4, lay.data_ptr(), 500, 4, x.data_ptr(), y.data_ptr(), st.data_ptr(),
                                  None) == rk.STATUS_INVALID_ARGUMENT  # k % 256
    assert L.rocknpu_b200_gemv_kq(4, lay.data_ptr() + 8, 256, 4, x.data_ptr(), y.data_ptr(), st.data_ptr(),
                                  None) == rk.STATUS_INVALID_ARGUMENT  # unaligned layout
    for kind in (4, 6):  # rows longer than 24576 are rejected before any work
        assert L.rocknpu_b200_gemv_kq(kind, lay.data_ptr(), 24576 + 256, 1, x.data_ptr(), y.data_ptr(), st.data_ptr(),
                                      None) == rk.STATUS_INVALID_ARGUMENT
