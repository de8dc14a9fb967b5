"""Parity at the BASELINE configurations' full sizes (configs 2, 3 and 5):
every output row or head against the oracle where the oracle finishes in
seconds, a fixed row sample plus size-independent identities where it does
not, and the 64 tile-sweep shapes (configuration 5b), each run with the tile
plan the baked sweep table gives it."""
from __future__ import annotations

import ctypes
import itertools

import numpy as np
import pytest
import torch

from _support import baseline_check

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_cfg2_w8a16_every_row(cuda_pkg, oracle):
    """Configuration 2 (4096 x 4096 x 11008, A ~ N(0,1), W ~ U{-127..127},
    scale ~ U[0.001, 0.02]): all 4096 rows against the oracle, through the
    data-parallel dispatch and the stream-K entry (which plans its own
    schedule for this shape)."""
    M, K, N = 4096, 4096, 11008
    rng = np.random.default_rng(20)
    a = rng.standard_normal((M, K)).astype(np.float16)
    w = rng.integers(-127, 128, (K, N), dtype=np.int8)
    s = rng.uniform(0.001, 0.02, N).astype(np.float16)
    ad, wd, sd = (torch.from_numpy(x).to(DEV) for x in (a, w, s))
    c = cuda_pkg.matmul_w8a16(ad, wd, sd)
    c_sk = cuda_pkg.matmul_w8a16(ad, wd, sd, workspace=cuda_pkg.w8a16_workspace(DEV))
    torch.cuda.synchronize()
    ref = oracle.matmul_w8a16_f32(a, w, s)
    baseline_check(ref, c.float().cpu().numpy(), "cfg 2, all rows")
    baseline_check(ref, c_sk.float().cpu().numpy(), "cfg 2 stream-K, all rows")
    assert cuda_pkg.device_status() == 0


def test_cfg3_attention_every_head(cuda_pkg, oracle):
    """Configuration 3 ([4, 32, 2048, 128] f16 ~ N(0,1), scale 1/sqrt(128),
    non-causal): all 128 heads against the oracle."""
    B, H, S, D = 4, 32, 2048, 128
    rng = np.random.default_rng(30)
    q, k, v = (rng.standard_normal((B * H, S, D)).astype(np.float16) for _ in range(3))
    qd, kd, vd = (torch.from_numpy(x).to(DEV).view(B, H, S, D) for x in (q, k, v))
    out = cuda_pkg.attention(qd, kd, vd)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy().reshape(B * H, S, D)
    ref = oracle.attention_f32(q, k, v)
    for h in range(B * H):
        baseline_check(ref[h], got[h], f"cfg 3 head {h}")
    assert cuda_pkg.device_status() == 0


def test_cfg5_single_gpu_full_size(cuda_pkg, oracle):
    """Configuration 5 on one GPU (16384 x 8192 x 28672, U[-1, 1]): a 64-row
    sample spread over every 128-row tile band against the oracle, the
    exact identity C(2 A) == 2 C(A) on the whole output (doubling is exact in
    f32, and in f16 away from overflow and the subnormal range), and the
    transposed-B form."""
    M, K, N = 16384, 8192, 28672
    g = torch.Generator(device=DEV).manual_seed(50)
    a = (torch.rand(M, K, device=DEV, generator=g) * 2 - 1).half()
    b = (torch.rand(K, N, device=DEV, generator=g) * 2 - 1).half()
    c = cuda_pkg.matmul(a, b)
    rows = np.unique(np.concatenate([np.arange(0, M, M // 48), [1, 127, 128, M - 1]]))[:64]
    a_rows = a[torch.from_numpy(rows).to(DEV)].cpu().numpy()
    b_h = b.cpu().numpy()
    got = c[torch.from_numpy(rows).to(DEV)].float().cpu().numpy()
    baseline_check(oracle.matmul_f32(a_rows, b_h), got, "cfg 5 row sample")
    c2 = cuda_pkg.matmul(a * 2, b)
    torch.cuda.synchronize()
    # f16 subnormals (|c| < 2^-14) round on a fixed grid, where doubling is
    # not exact; everywhere else the identity is bit-exact
    normal = c.abs() >= 2.0 ** -13
    assert normal.float().mean() > 0.9999
    assert torch.equal(c2[normal], (c * 2)[normal]), "C(2A) != 2 C(A)"
    del c2, normal
    bt = b.t().contiguous()
    ct = cuda_pkg.matmul(a, bt, transpose_b=True)
    torch.cuda.synchronize()
    assert torch.equal(ct, c), "rhs-transposed dispatch differs"
    assert cuda_pkg.device_status() == 0


SWEEP = [128, 512, 2048, 8192]


@pytest.mark.parametrize("M,N,K", list(itertools.product(SWEEP, SWEEP, SWEEP)))
def test_cfg5b_sweep_shape_with_table_plan(cuda_pkg, oracle, M, N, K):
    """Every configuration-5b shape through hxb_matmul_f16, which takes its
    tile plan (block_n, group_m) from the baked sweep table; the plan is
    checked to be the one the table holds, and up to 256 rows (all when
    M <= 512) are compared with the oracle."""
    lib = cuda_pkg._native.load()
    bn, gm, sk, pair = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    cuda_pkg._native.check(lib.hxb_plan_matmul_f16(M, N, K, 0, sms, ctypes.byref(bn),
                                                   ctypes.byref(gm), ctypes.byref(sk),
                                                   ctypes.byref(pair)))
    assert bn.value in (64, 128, 256, 512) and gm.value >= 1 and sk.value in (1, 2, 4, 8)
    assert pair.value in (1, 2) and (pair.value == 1 or sk.value == 1)
    rng = np.random.default_rng(M + 3 * N + 7 * K)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    c = cuda_pkg.matmul(torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV))
    torch.cuda.synchronize()
    rows = np.arange(M) if M <= 512 else np.linspace(0, M - 1, 256).astype(np.int64)
    got = c.float().cpu().numpy()[rows]
    baseline_check(oracle.matmul_f32(a[rows], b), got,
                   f"sweep {M}x{N}x{K} (block_n {bn.value}, group_m {gm.value}, "
                   f"split_k {sk.value})")
    assert cuda_pkg.device_status() == 0
