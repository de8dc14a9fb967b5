"""Worker of the 2-rank sharded-matmul test (launched by torchrun from
tests/test_sharded_gpu.py): each rank computes its N-shard, the fused
all-gather path and the NCCL baseline must give the same full C, and rank 0
checks a row sample against the CPU oracle."""
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
    import torch
    import torch.distributed as dist
    import __graft_entry__ as ge

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    pkg = ge.load_package()
    try:
        M, N, K = 1024, 2048, 512
        rng = np.random.default_rng(11)  # same inputs on every rank
        a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
        b = rng.uniform(-1, 1, (K, N)).astype(np.float16)
        sm = pkg.sharded.ShardedMatmul(M, N, K, device=dev)
        b0, b1 = sm.begin, sm.end
        ad = torch.from_numpy(a).to(dev)
        bd = torch.from_numpy(np.ascontiguousarray(b[:, b0:b1])).to(dev)
        fused = sm.fused(ad, bd).clone()
        shard = torch.empty(M, b1 - b0, dtype=torch.float16, device=dev)
        gathered = torch.empty(world * M, b1 - b0, dtype=torch.float16, device=dev)
        nccl = sm.nccl(ad, bd, shard_out=shard, gathered=gathered)
        torch.cuda.synchronize()
        assert torch.equal(fused, nccl), "fused all-gather differs from the NCCL path"
        if rank == 0:
            from oracle import oracle
            from _support import baseline_check
            rows = np.arange(0, M, 37)
            want = oracle.matmul_f32(a[rows], b)
            baseline_check(want, fused[torch.from_numpy(rows).to(dev)].float().cpu().numpy(),
                           "2-rank sharded")
        # back-to-back fused steps with new data each time: every step's
        # gathered C must hold this step's tiles from every rank (the peer
        # barrier after the GEMM publishes the peers' stores)
        for it in range(12):
            bd.mul_(-1.0 if it % 2 else 0.5)
            f = sm.fused(ad, bd).clone()
            n = sm.nccl(ad, bd, shard_out=shard, gathered=gathered)
            torch.cuda.synchronize()
            assert torch.equal(f, n), f"fused step {it} differs from the NCCL path"
        assert pkg.device_status() == 0
        dist.barrier()
        sm.close()
        # configuration 2 split along N: the GEMM (M > 16) and the GEMV
        # (M <= 16), fused all-gather against the NCCL baseline and the oracle
        N8, K8 = 2752, 1024
        w8 = rng.integers(-127, 128, (K8, N8), dtype=np.int8)
        s8 = rng.uniform(0.001, 0.02, N8).astype(np.float16)
        for M8 in (600, 3):
            x8 = rng.standard_normal((M8, K8)).astype(np.float16)
            sw = pkg.sharded.ShardedMatmulW8(M8, N8, K8, device=dev,
                                            workspace=pkg.w8a16_workspace(dev))
            c0, c1 = sw.begin, sw.end
            xd = torch.from_numpy(x8).to(dev)
            wd = torch.from_numpy(np.ascontiguousarray(w8[:, c0:c1])).to(dev)
            sd = torch.from_numpy(np.ascontiguousarray(s8[c0:c1])).to(dev)
            fused8 = sw.fused(xd, wd, sd).clone()
            shard8 = torch.empty(M8, c1 - c0, dtype=torch.float16, device=dev)
            gath8 = torch.empty(world * M8, c1 - c0, dtype=torch.float16, device=dev)
            nccl8 = sw.nccl(xd, wd, sd, shard_out=shard8, gathered=gath8)
            torch.cuda.synchronize()
            assert torch.equal(fused8, nccl8), f"w8 M={M8}: fused all-gather differs from NCCL"
            if rank == 0:
                from oracle import oracle
                from _support import baseline_check
                baseline_check(oracle.matmul_w8a16_f32(x8, w8, s8),
                               fused8.float().cpu().numpy(), f"2-rank w8 M={M8}")
            dist.barrier()
            sw.close()
        assert pkg.device_status() == 0
        if rank == 0:
            print("sharded ok", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
