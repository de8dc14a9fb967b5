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
        assert pkg.device_status() == 0
        dist.barrier()
        sm.close()
        if rank == 0:
            print("sharded ok", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
