"""Parity of the stream-K schedules of the int8-weight GEMM
(hxb_matmul_w8a16_streamk): K split across CTAs when whole tiles would leave
SMs idle -- over all tiles, or over the last partial wave after whole-tile
waves -- partial sums added by the CTA that owns the tile's first K-block.

Shapes are the decoder block's M = 512 projections (64 and 344 output tiles
of 128 weight columns x 256 rows on 148 SMs) and small ragged cases where one
tile is cut into many pieces."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _support import baseline_check

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
FLAG_BYTES = 4096


def _inputs(M, K, N, seed):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K)).astype(np.float16)
    w = rng.integers(-127, 128, (K, N), dtype=np.int8)
    s = rng.uniform(0.001, 0.02, N).astype(np.float16)
    r = rng.standard_normal((M, N)).astype(np.float16)
    return a, w, s, r


def _t(x):
    return torch.from_numpy(x).to(DEV)


@pytest.mark.parametrize("M,K,N,res", [
    (512, 4096, 4096, True),     # decoder O projection: 64 tiles, stream-K
    (512, 11008, 4096, True),    # decoder down projection: stream-K
    (512, 4096, 12288, False),   # decoder qkv: 192 tiles, stream-K over all
    (512, 4096, 22016, False),   # decoder gate|up: 344 tiles, two whole waves + stream-K tail
    (4096, 4096, 11008, False),  # BASELINE cfg 2: 1376 tiles, nine whole waves + stream-K tail
    (300, 7992, 23008, True),    # ragged M, K and N, two whole waves + stream-K tail
    (129, 4000, 272, True),      # ragged K and M, stream-K over 3 tiles
    (100, 8192, 144, False),     # 2 tiles cut into 16 pieces each
    (200, 320, 528, False),      # too little K to split: data-parallel
])
def test_streamk_vs_oracle(cuda_pkg, oracle, M, K, N, res):
    a, w, s, r = _inputs(M, K, N, seed=M * 7 + N)
    ws = cuda_pkg.w8a16_workspace(DEV)
    ad, wd, sd, rd = _t(a), _t(w), _t(s), _t(r)
    got = cuda_pkg.matmul_w8a16(ad, wd, sd, residual=rd if res else None, workspace=ws)
    again = cuda_pkg.matmul_w8a16(ad, wd, sd, residual=rd if res else None, workspace=ws)
    torch.cuda.synchronize()
    assert cuda_pkg.device_status() == 0
    # every finaliser cleared the flags it consumed; partial sums are added in
    # a fixed order, so a second call is bit-identical
    assert int(ws[:FLAG_BYTES].count_nonzero()) == 0
    assert torch.equal(got, again)
    rows = np.arange(M) if M * K * N <= 2**31 else np.array(
        [r for r in (0, 1, 190, 191, 255, 256, 299, 383, 384, 511, 2047, 4095) if r < M])
    ref = oracle.matmul_w8a16_f32(a[rows], w, s)
    if res:
        ref = ref + r[rows].astype(np.float32)
    baseline_check(ref, got[torch.from_numpy(rows).to(DEV)].float().cpu().numpy(),
                   f"w8 stream-K {M}x{K}x{N}")


def test_streamk_matches_data_parallel(cuda_pkg):
    """The split changes only the f32 summation order of the tensor-core
    accumulation, so against the data-parallel schedule most f16 results are
    bit-identical and the rest differ by rounding: within the BASELINE bar
    (1e-2 + one f16 ulp), and within a few ulp where the scaled product and the
    residual cancel."""
    M, K, N = 512, 4096, 4096
    a, w, s, r = _inputs(M, K, N, seed=5)
    ad, wd, sd, rd = _t(a), _t(w), _t(s), _t(r)
    sk = cuda_pkg.matmul_w8a16(ad, wd, sd, residual=rd, workspace=cuda_pkg.w8a16_workspace(DEV))
    dp = cuda_pkg.matmul_w8a16(ad, wd, sd, residual=rd)
    torch.cuda.synchronize()
    sk, dp = sk.float().cpu().numpy(), dp.float().cpu().numpy()
    big = np.maximum(np.abs(sk), np.abs(dp)).astype(np.float16)
    ulp = np.spacing(big).astype(np.float64)
    d = np.abs(sk.astype(np.float64) - dp)
    assert (d <= 1e-2 + ulp).all(), float((d - ulp).max())
    assert float((d == 0).mean()) > 0.5, float((d == 0).mean())


def test_streamk_graph_replay(cuda_pkg):
    """Captured once, replayed: the flags each replay raises are cleared by the
    same replay, so every replay computes the same result."""
    M, K, N = 512, 4096, 4096
    a, w, s, r = _inputs(M, K, N, seed=6)
    ad, wd, sd, rd = _t(a), _t(w), _t(s), _t(r)
    ws = cuda_pkg.w8a16_workspace(DEV)
    out = torch.empty(M, N, dtype=torch.float16, device=DEV)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        cuda_pkg.matmul_w8a16(ad, wd, sd, residual=rd, workspace=ws, out=out)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    first = out.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        cuda_pkg.matmul_w8a16(ad, wd, sd, residual=rd, workspace=ws, out=out)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, first)
    assert int(ws[:FLAG_BYTES].count_nonzero()) == 0
    assert cuda_pkg.device_status() == 0


def test_streamk_rejects_missing_workspace(cuda_pkg):
    lib = cuda_pkg._native.load()
    a = torch.zeros(256, 256, dtype=torch.float16, device=DEV)
    w = torch.zeros(256, 256, dtype=torch.int8, device=DEV)
    s = torch.ones(256, dtype=torch.float16, device=DEV)
    c = torch.empty(256, 256, dtype=torch.float16, device=DEV)
    rc = lib.hxb_matmul_w8a16_streamk(a.data_ptr(), 256, w.data_ptr(), 256, s.data_ptr(), None,
                                      c.data_ptr(), 256, 256, 256, 256, None, 0,
                                      torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert b"workspace" in lib.hxb_last_error_message()


@pytest.mark.parametrize("M,K,N,res", [
    (1, 4096, 11008, False),   # BASELINE configuration 2b, M = 1: 43 strips x 64 k tiles
    (16, 4096, 11008, True),   # M = 16, the decoder residual form
    (5, 1000, 1104, True),     # ragged K (a zero-filled tail tile), N not a strip multiple
    (9, 64, 16, False),        # one tile: a single SM, no partial sums
    (8, 8192, 272, False),     # 2 strips x 128 k tiles over every SM: many contributors
    (12, 11008, 4096, True),   # decoder down projection at decode batch 12
])
def test_gemv_all_sms_vs_oracle(cuda_pkg, oracle, M, K, N, res):
    """M <= 16 with the workspace: the GEMV that spreads the weight tiles over
    every SM and adds the partial sums of strips shared between SMs."""
    a, w, s, r = _inputs(M, K, N, seed=M * 11 + N + K)
    ws = cuda_pkg.w8a16_workspace(DEV)
    ad, wd, sd, rd = _t(a), _t(w), _t(s), _t(r)
    got = cuda_pkg.matmul_w8a16(ad, wd, sd, residual=rd if res else None, workspace=ws)
    again = cuda_pkg.matmul_w8a16(ad, wd, sd, residual=rd if res else None, workspace=ws)
    plain = cuda_pkg.matmul_w8a16(ad, wd, sd, residual=rd if res else None)
    torch.cuda.synchronize()
    assert cuda_pkg.device_status() == 0
    assert int(ws[:FLAG_BYTES].count_nonzero()) == 0
    assert torch.equal(got, again)
    ref = oracle.matmul_w8a16_f32(a, w, s)
    if res:
        ref = ref + r.astype(np.float32)
    baseline_check(ref, got.float().cpu().numpy(), f"gemv all-SM {M}x{K}x{N}")
    baseline_check(ref, plain.float().cpu().numpy(), f"gemv strip-per-SM {M}x{K}x{N}")


def test_gemv_all_sms_graph_replay(cuda_pkg):
    """Flags left zero by every launch: replays of a captured graph agree."""
    a, w, s, _ = _inputs(1, 4096, 11008, seed=5)
    ws = cuda_pkg.w8a16_workspace(DEV)
    ad, wd, sd = _t(a), _t(w), _t(s)
    out = torch.empty(1, 11008, dtype=torch.float16, device=DEV)
    cuda_pkg.matmul_w8a16(ad, wd, sd, workspace=ws, out=out)
    torch.cuda.synchronize()
    first = out.clone()
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g):
            for _ in range(3):
                cuda_pkg.matmul_w8a16(ad, wd, sd, workspace=ws, out=out)
    for _ in range(5):
        out.zero_()
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    assert int(ws[:FLAG_BYTES].count_nonzero()) == 0
    assert cuda_pkg.device_status() == 0
