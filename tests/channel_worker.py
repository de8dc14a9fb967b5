"""Worker of the HAL channel test (launched by torchrun from
tests/test_sharded_gpu.py): every rank opens a HAL device and joins one
channel (the id made by rank 0 is passed over the gloo process group), then
runs ONE command buffer holding its N-shard matmul dispatch followed by an
all-gather collective of the shards, and an all-reduce of a vector. Rank 0
checks the gathered result against the CPU oracle."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests"))


def main() -> None:
    import numpy as np
    import torch.distributed as dist
    import __graft_entry__ as ge

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    pkg = ge.load_package()
    hal = pkg.hal
    try:
        obj = [hal.channel_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        dev = hal.Device(local)
        ch = hal.Channel(dev, obj[0], rank, world, timeout_s=60)
        assert (ch.rank, ch.count) == (rank, world)
        M, N, K = 512, 256 * world, 384
        n = N // world
        rng = np.random.default_rng(7)  # same inputs on every rank
        a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
        b = rng.uniform(-1, 1, (K, N)).astype(np.float16)
        bs = np.ascontiguousarray(b[:, rank * n:(rank + 1) * n])
        # the shard is computed transposed (C_r^T = B_r^T A^T), so that the
        # all-gather of the ranks' [n, M] blocks is C^T [N, M] with no layout step
        ab, bb = dev.allocate(a.nbytes), dev.allocate(bs.nbytes)
        ab.write(np.ascontiguousarray(a.T))         # A^T [K, M] -> the rhs [K, M]
        bb.write(np.ascontiguousarray(bs.T))        # B_r^T [n, K] -> the lhs
        shard = dev.allocate(n * M * 4)
        full = dev.allocate(N * M * 4)
        vec = np.full(1000, rank + 1, np.float32)
        vb, vs = dev.allocate(vec.nbytes), dev.allocate(vec.nbytes)
        vb.write(vec)
        cb = dev.command_buffer()
        cb.begin()
        cb.dispatch("matmul_f16", [n, M, K, 2], [bb, ab, shard])
        cb.collective(ch, "all_gather", "f32", shard, full, n * M)
        cb.collective(ch, "all_reduce_sum", "f32", vb, vs, 1000)
        cb.end()
        done = dev.semaphore(0)
        for i in (1, 2):  # recorded once, submitted twice
            dev.execute(cb, wait=(done, i - 1), signal=(done, i))
            done.wait(i, timeout_s=60)
        got = np.frombuffer(full.read(), np.float32).reshape(N, M).T
        s = np.frombuffer(vs.read(), np.float32)
        assert np.all(s == world * (world + 1) / 2), s[:4]
        if rank == 0:
            from oracle import oracle
            from _support import baseline_check
            baseline_check(oracle.matmul_f32(a, b), got, f"{world}-rank HAL channel all-gather")
        for x in (cb, done, ab, bb, shard, full, vb, vs):
            x.close()
        dist.barrier()
        ch.close()
        dev.close()
        if rank == 0:
            print("channel ok", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
