"""GPU parity of the N-sharded matmul pieces: the
GEMM's all-gather epilogue (tested on one GPU with the replicas in local
memory), the layout step of the NCCL baseline, and, when the box has two or
more GPUs, the whole fused path across ranks (torchrun, NCCL)."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from _support import baseline_check

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
REPO = Path(__file__).resolve().parent.parent


def test_allgather_epilogue_writes_every_replica(cuda_pkg, oracle):
    import ctypes
    lib = cuda_pkg._native.load()
    rng = np.random.default_rng(21)
    M, K, Nfull, G = 300, 200, 1024, 4
    col0, n = 256, 512  # this "rank" owns columns [256, 768)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (K, n)).astype(np.float16)
    ad, bd = torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV)
    outs = [torch.full((M, Nfull), float("nan"), dtype=torch.float16, device=DEV) for _ in range(G)]
    reps = (ctypes.c_void_p * (G - 1))(*[o.data_ptr() + col0 * 2 for o in outs[1:]])
    cuda_pkg._native.check(lib.hxb_matmul_f16_allgather(
        ad.data_ptr(), K, bd.data_ptr(), n, 0, outs[0].data_ptr() + col0 * 2, reps, G - 1,
        Nfull, M, n, K, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    want = oracle.matmul_f32(a, b)
    first = outs[0].cpu().numpy()
    baseline_check(want, first[:, col0:col0 + n].astype(np.float32), "allgather local")
    for o in outs:
        h = o.cpu().numpy()
        assert np.array_equal(h[:, col0:col0 + n].view(np.int16), first[:, col0:col0 + n].view(np.int16))
        assert np.isnan(h[:, :col0].astype(np.float32)).all() and np.isnan(h[:, col0 + n:].astype(np.float32)).all()
    assert cuda_pkg.device_status() == 0


@pytest.mark.parametrize("M,K,n,col0", [(600, 512, 1376, 2752),   # GEMM, ragged last tile
                                        (300, 320, 272, 16),       # GEMM, one partial tile
                                        (5, 1024, 1376, 1376),     # GEMV + block copy
                                        (16, 256, 96, 0)])
def test_w8_allgather_epilogue_writes_every_replica(cuda_pkg, oracle, M, K, n, col0):
    """hxb_matmul_w8a16_allgather with the replicas in local memory: every
    replica gets the shard's columns bit for bit and nothing else (the
    epilogue clips rows past M and columns past the shard)."""
    import ctypes
    lib = cuda_pkg._native.load()
    rng = np.random.default_rng(M + n)
    G, Nfull = 4, col0 + n + 32
    a = rng.standard_normal((M, K)).astype(np.float16)
    w = rng.integers(-127, 128, (K, n), dtype=np.int8)
    s = rng.uniform(0.001, 0.02, n).astype(np.float16)
    ad, wd, sd = (torch.from_numpy(x).to(DEV) for x in (a, w, s))
    outs = [torch.full((M, Nfull), float("nan"), dtype=torch.float16, device=DEV)
            for _ in range(G)]
    reps = (ctypes.c_void_p * (G - 1))(*[o.data_ptr() + col0 * 2 for o in outs[1:]])
    ws = cuda_pkg.w8a16_workspace(DEV)
    for workspace in (None, ws):
        for o in outs:
            o.fill_(float("nan"))
        cuda_pkg._native.check(lib.hxb_matmul_w8a16_allgather(
            ad.data_ptr(), K, wd.data_ptr(), n, sd.data_ptr(), outs[0].data_ptr() + col0 * 2,
            reps, G - 1, Nfull, M, n, K,
            workspace.data_ptr() if workspace is not None else None,
            workspace.numel() if workspace is not None else 0,
            torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        first = outs[0].cpu().numpy()
        baseline_check(oracle.matmul_w8a16_f32(a, w, s),
                       first[:, col0:col0 + n].astype(np.float32), f"w8 allgather {M}x{K}x{n}")
        for o in outs:
            h = o.cpu().numpy()
            assert np.array_equal(h[:, col0:col0 + n].view(np.int16),
                                  first[:, col0:col0 + n].view(np.int16))
            assert np.isnan(h[:, :col0].astype(np.float32)).all()
            assert np.isnan(h[:, col0 + n:].astype(np.float32)).all()
    assert cuda_pkg.device_status() == 0


def test_attention_head_split_covers_every_head(cuda_pkg, oracle):
    """Configuration 3 split by heads: each "rank" computes its contiguous
    head group; the groups together give the unsplit result bit for bit."""
    B, H, S, D = 2, 6, 256, 128
    g = torch.Generator(device=DEV).manual_seed(9)
    q, k, v = (torch.randn(B * H, S, D, device=DEV, generator=g).half() for _ in range(3))
    whole = cuda_pkg.attention(q, k, v)
    parts = []
    for r in range(4):
        h0, h1 = cuda_pkg.sharded.head_range(B * H, 4, r)
        parts.append(cuda_pkg.attention(q[h0:h1], k[h0:h1], v[h0:h1]))
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(parts), whole)


def test_gather_column_blocks(cuda_pkg):
    lib = cuda_pkg._native.load()
    G, M, n = 4, 77, 40
    src = torch.randn(G, M, n, device=DEV).half()
    dst = torch.empty(M, G * n, dtype=torch.float16, device=DEV)
    cuda_pkg._native.check(lib.hxb_gather_column_blocks_f16(
        src.data_ptr(), dst.data_ptr(), G, M, n, G * n, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    want = src.permute(1, 0, 2).reshape(M, G * n)
    assert torch.equal(dst, want)


def test_sharded_single_rank_fused(cuda_pkg, oracle):
    sharded = cuda_pkg.sharded
    M, N, K = 512, 768, 320
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    sm = sharded.ShardedMatmul(M, N, K, device=torch.device(DEV))
    out = sm.fused(torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV))
    torch.cuda.synchronize()
    baseline_check(oracle.matmul_f32(a, b), out.float().cpu().numpy(), "sharded world=1")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs on one box")
def test_sharded_two_ranks_fused_matches_nccl_and_oracle():
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1",
           "--master-port", "29531", str(REPO / "tests" / "sharded_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "sharded ok" in r.stdout


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs on one box")
def test_hal_channel_two_ranks():
    """HAL collectives (the reference's channel.c returns UNIMPLEMENTED): a
    command buffer with a matmul dispatch and NCCL all-gather / all-reduce
    collectives, recorded once and submitted twice on each of 2 ranks."""
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1",
           "--master-port", "29533", str(REPO / "tests" / "channel_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "channel ok" in r.stdout
