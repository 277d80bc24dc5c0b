"""Rank programs of the N-sharding tests (not collected by pytest).

* ``cpu_worker``: one gloo rank on the CPU.  It takes its weight rows from
  the product's row split (rocknpu_b200.shard.shard_rows), computes them with
  the oracle, all-gathers the rank-major blocks and lays them out row-major,
  and checks the result against the unsharded oracle result bit for bit.
  It also checks the handle exchange (shard.exchange) in rank order.
* ``python tests/shard_worker.py --route peer|allgather`` under torchrun: one
  GPU rank of the sharded CUDA path, checked bit for bit against the same
  GEMM run unsharded on that rank's GPU.  Exits non-zero on a mismatch.
"""
from __future__ import annotations

import argparse
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def cpu_worker(rank: int, world: int, port: int, kind: int, n: int, k: int, m: int, seed: int) -> None:
    import torch
    import torch.distributed as dist

    import oracle
    import rocknpu_b200 as rk
    from rocknpu_b200 import shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rows = shard.shard_rows(n, world)
        shard_ld = max(w for _, w in rows)
        blocks = rk.synth_q_weights(kind, n, k, seed=seed, sigma=0.02)
        a = rk.synth_normal(seed + 1, m * k).reshape(m, k)
        row_bytes = k // 256 * rk.BLOCK_BYTES[kind]
        start, width = rows[rank]
        slot = np.zeros((m, shard_ld), dtype=np.float32)
        if width:
            st, w8, ws = oracle.prepare_w8a8(kind, blocks[start * row_bytes:(start + width) * row_bytes], k, width)
            assert st == 0
            st, y = oracle.matmul_w8a8(w8, ws, a)
            assert st == 0
            slot[:, :width] = y
        gathered = [torch.zeros(m * shard_ld, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(slot.reshape(-1)))
        full = np.empty((m, n), dtype=np.float32)
        for r, (s, w) in enumerate(rows):
            full[:, s:s + w] = gathered[r].numpy().reshape(m, shard_ld)[:, :w]
        st, w8, ws = oracle.prepare_w8a8(kind, blocks, k, n)
        st, ref = oracle.matmul_w8a8(w8, ws, a)
        assert np.array_equal(full.view(np.uint32), ref.view(np.uint32)), f"rank {rank}: sharded result differs"
        got = shard.exchange(bytes([rank + 1]) * shard.IPC_HANDLE_BYTES)
        assert got == [bytes([r + 1]) * shard.IPC_HANDLE_BYTES for r in range(world)], "exchange out of order"
    finally:
        dist.destroy_process_group()


def gpu_main(route: str) -> int:
    import torch
    import torch.distributed as dist

    import rocknpu_b200 as rk
    from rocknpu_b200 import device as dev
    from rocknpu_b200 import shard

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    failures = 0
    try:
        # the last shape is long-K enough that each rank's GEMM runs two-SM
        # pair tiles at two ranks (one-SM tiles at more)
        for kind, n, k, m in [(4, 2048, 2048, 128), (6, 1184, 512, 77), (4, 5632, 2048, 512), (4, 96, 256, 3),
                              (4, 2048, 2048, 1), (4, 8192, 4096, 2048)]:
            blocks = rk.synth_q_weights(kind, n, k, seed=n + k, sigma=0.02)
            x = torch.from_numpy(rk.synth_normal(7 + m, m * k).reshape(m, k)).cuda()
            sm = shard.ShardedMatmul(kind, blocks, k, n, route=route, max_m=m)
            ys = []
            for rep in range(3):  # three calls: both peer buffers, then the first again
                y = sm(x * (rep + 1))
                ys.append(y.clone())
            sm.check()
            status = dev.new_status()
            w8, ws = dev.prepare_w8(kind, torch.from_numpy(blocks).cuda(), k, n, status)
            for rep in range(3):
                a8, a_s = dev.quantize_rows(x * (rep + 1), status)
                ref = dev.gemm_w8a8(a8, a_s, w8, ws, status)
                torch.cuda.synchronize()
                if not torch.equal(ys[rep].view(torch.int32), ref.view(torch.int32)):
                    print(f"rank {rank}: {route} kind={kind} n={n} k={k} m={m} call {rep} differs", flush=True)
                    failures += 1
            assert status.item() == 0
            sm.close()
            dist.barrier()
    finally:
        dist.destroy_process_group()
    if rank == 0 and failures == 0:
        print(f"sharded {route} route: {world} ranks bit-identical to one GPU", flush=True)
    return 1 if failures else 0


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--route", choices=["peer", "allgather"], default="peer")
    sys.exit(gpu_main(ap.parse_args().route))
