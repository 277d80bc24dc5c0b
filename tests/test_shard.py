"""Multi-GPU N-sharding: the row split, the all-gather layout and the peer route.

CPU: the product's row split against the oracle's restatement of the
reference's split_blocks (int8_decode_pool.rs:1505-1522), and a world-size-2
gloo run that shards a GEMM by that split, all-gathers rank-major blocks and
must reproduce the unsharded oracle result bit for bit.

GPU (one B200): the fused all-gather epilogue writing two copies, the
rank-major -> row-major gather kernel, a one-rank peer buffer and barrier.
GPU (two or more B200s, run when present): tests/shard_worker.py under
torchrun, both routes, bit-identical to the unsharded GEMM.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import oracle
import rocknpu_b200 as rk
from rocknpu_b200 import shard

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("n", [32, 64, 96, 256, 1184, 2048, 5632, 28672, 128256, 40])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_rows_is_the_reference_block_split(n, world):
    rows = shard.shard_rows(n, world)
    assert len(rows) == world
    blocks = (n + 31) // 32
    ref = oracle.split_blocks(blocks, 32, world)
    for r, (s, w) in enumerate(rows):
        if r < len(ref):
            assert s == ref[r][0]
            assert w == min(ref[r][1], n - s)
        else:
            assert w == 0
    # the shards tile [0, n) in rank order
    pos = 0
    for s, w in rows:
        if w:
            assert s == pos
            pos += w
    assert pos == n


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("kind,n,k,m", [(4, 2048, 512, 9), (6, 1184, 256, 16), (4, 96, 256, 5)])
def test_two_rank_gloo_shard_matches_unsharded_oracle(kind, n, k, m):
    import torch.multiprocessing as mp
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import shard_worker
    mp.spawn(shard_worker.cpu_worker, args=(2, _free_port(), kind, n, k, m, 11), nprocs=2, join=True)


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------

@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n_local,col0,ldo", [(128, 2048, 1024, 512, 2048), (77, 512, 608, 576, 1184),
                                                  (300, 1024, 256, 0, 256)])
def test_fused_gather_epilogue_writes_every_copy(m, k, n_local, col0, ldo):
    import ctypes

    import torch
    from rocknpu_b200 import device as dev
    rng = np.random.default_rng(m + n_local)
    a8 = torch.from_numpy(rng.integers(-127, 128, size=(m, k), dtype=np.int8)).cuda()
    a_s = torch.from_numpy(rng.uniform(1e-3, 1e-1, size=m).astype(np.float32)).cuda()
    w8 = torch.from_numpy(rng.integers(-127, 128, size=(n_local, k), dtype=np.int8)).cuda()
    w_s = torch.from_numpy(rng.uniform(1e-3, 1e-2, size=n_local).astype(np.float32)).cuda()
    status = dev.new_status()
    ref = dev.gemm_w8a8(a8, a_s, w8, w_s, status)
    outs = [torch.full((m, ldo), float("nan"), device="cuda") for _ in range(2)]
    ptrs = (ctypes.c_void_p * 2)(*[o.data_ptr() for o in outs])
    st = rk.lib().rocknpu_b200_gemm_w8a8_gather(a8.data_ptr(), k, a_s.data_ptr(), w8.data_ptr(), k, w_s.data_ptr(),
                                               ptrs, 2, col0, ldo, m, k, n_local, status.data_ptr(),
                                               torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    assert status.item() == 0
    for o in outs:
        assert torch.equal(o[:, col0:col0 + n_local].contiguous().view(torch.int32), ref.view(torch.int32))
        assert torch.isnan(o[:, :col0]).all() and torch.isnan(o[:, col0 + n_local:]).all()
    # arguments outside the output are rejected before any launch
    assert rk.lib().rocknpu_b200_gemm_w8a8_gather(a8.data_ptr(), k, a_s.data_ptr(), w8.data_ptr(), k,
                                                  w_s.data_ptr(), ptrs, 2, ldo - n_local + 1, ldo, m, k, n_local,
                                                  status.data_ptr(), None) == rk.STATUS_INVALID_ARGUMENT


@pytest.mark.gpu
@pytest.mark.parametrize("n,world,m", [(2048, 2, 64), (1184, 3, 17), (96, 8, 5), (28672, 8, 3)])
def test_gather_shards_kernel_layout(n, world, m):
    import ctypes

    import torch
    rows = shard.shard_rows(n, world)
    ld = max(w for _, w in rows)
    src = torch.randn(world * m * ld, device="cuda")
    out = torch.full((m, n), float("nan"), device="cuda")
    starts = (ctypes.c_size_t * world)(*[s for s, _ in rows])
    widths = (ctypes.c_size_t * world)(*[w for _, w in rows])
    assert rk.lib().rocknpu_b200_gather_shards(src.data_ptr(), m * ld, ld, m, world, starts, widths, out.data_ptr(),
                                               n, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    s3 = src.view(world, m, ld).cpu().numpy()
    exp = np.concatenate([s3[r, :, :w] for r, (_, w) in enumerate(rows) if w], axis=1)
    assert np.array_equal(out.cpu().numpy(), exp)


@pytest.mark.gpu
def test_single_rank_sharded_matmul_and_peer_buffer():
    import torch
    from rocknpu_b200 import device as dev
    k, n, m = 1024, 640, 33
    blocks = rk.synth_q_weights(4, n, k, seed=5)
    x = torch.from_numpy(rk.synth_normal(6, m * k).reshape(m, k)).cuda()
    sm = shard.ShardedMatmul(4, blocks, k, n, max_m=64)
    y = sm(x)
    sm.check()
    status = dev.new_status()
    w8, ws = dev.prepare_w8(4, torch.from_numpy(blocks).cuda(), k, n, status)
    a8, a_s = dev.quantize_rows(x, status)
    ref = dev.gemm_w8a8(a8, a_s, w8, ws, status)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int32), ref.view(torch.int32))
    # a one-rank peer buffer: mapping, tensor view and barrier (epochs advance)
    buf = shard.PeerBuffer(m * n * 4)
    t = buf.tensor((m, n))
    t.copy_(ref)
    for _ in range(3):
        buf.barrier(status)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert torch.equal(t, ref)
    buf.close()


def _gpu_count() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.gpu
@pytest.mark.parametrize("route", ["peer", "allgather"])
def test_multi_gpu_sharded_routes_bit_identical(route):
    world = min(_gpu_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "shard_worker.py"), "--route", route]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
