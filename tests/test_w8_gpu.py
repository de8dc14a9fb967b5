"""Parity of the int8-weight matmul dispatch."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _support import baseline_check

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(M, K, N, seed=0):
    """BASELINE configuration 2 distributions: A ~ N(0,1) f16, W ~ U{-127..127}
    int8, scale ~ U[0.001, 0.02] f16."""
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K)).astype(np.float16)
    w = rng.integers(-127, 128, (K, N), dtype=np.int8)
    s = rng.uniform(0.001, 0.02, N).astype(np.float16)
    return a, w, s


@pytest.mark.parametrize("M,K,N", [(256, 4096, 11008), (1, 4096, 11008), (16, 4096, 11008),
                                   (200, 320, 528), (5, 64, 48), (129, 1000, 272),
                                   (16, 200, 4112), (3, 4104, 96),
                                   # N <= 128: the one-CTA kernel (one weight block)
                                   (300, 512, 128), (40, 2048, 112)])
def test_w8a16_vs_oracle(cuda_pkg, oracle, M, K, N):
    a, w, s = _inputs(M, K, N, seed=M + N)
    c = cuda_pkg.matmul_w8a16(torch.from_numpy(a).to(DEV), torch.from_numpy(w).to(DEV),
                              torch.from_numpy(s).to(DEV))
    torch.cuda.synchronize()
    baseline_check(oracle.matmul_w8a16_f32(a, w, s), c.float().cpu().numpy(),
                   f"w8 {M}x{K}x{N}")
    assert cuda_pkg.device_status() == 0


def test_w8a16_full_size_properties(cuda_pkg, oracle):
    """Full BASELINE size (4096 x 4096 x 11008): sampled rows against the
    oracle, plus the size-independent identity C(2*scale) == 2*C(scale),
    exact because doubling is exact in f32 and in f16."""
    M, K, N = 4096, 4096, 11008
    a, w, s = _inputs(M, K, N, seed=1)
    ad, wd, sd = (torch.from_numpy(x).to(DEV) for x in (a, w, s))
    c = cuda_pkg.matmul_w8a16(ad, wd, sd)
    c2 = cuda_pkg.matmul_w8a16(ad, wd, sd * 2)
    torch.cuda.synchronize()
    # f16 subnormals (|c| < 2^-14) round on a fixed grid, where doubling is
    # not exact; everywhere else the identity is bit-exact.
    normal = c.abs() >= 2.0 ** -13
    assert normal.float().mean() > 0.999
    assert torch.equal(c2[normal], (c * 2)[normal])
    rows = np.array([0, 1, 127, 128, 2047, 4095])
    ref = oracle.matmul_w8a16_f32(a[rows], w, s)
    baseline_check(ref, c[torch.from_numpy(rows).to(DEV)].float().cpu().numpy(), "w8 rows")


def test_w8a16_exact_dequant_index_math(cuda_pkg):
    """Bit-exact index math: with one-hot activations each output row is one
    weight row times its column scale, rounded once to f16."""
    K, N = 256, 384
    rng = np.random.default_rng(2)
    w = rng.integers(-127, 128, (K, N), dtype=np.int8)
    s = rng.uniform(0.001, 0.02, N).astype(np.float16)
    ks = np.array([0, 1, 63, 64, 200, 255])
    a = np.zeros((len(ks), K), np.float16)
    a[np.arange(len(ks)), ks] = 1
    c = cuda_pkg.matmul_w8a16(torch.from_numpy(a).to(DEV), torch.from_numpy(w).to(DEV),
                              torch.from_numpy(s).to(DEV))
    torch.cuda.synchronize()
    want = (w[ks].astype(np.float32) * s.astype(np.float32)).astype(np.float16)
    assert np.array_equal(c.cpu().numpy(), want)


def test_w8a16_rejects_unaligned_weight_pitch(cuda_pkg):
    """int8 weight rows must be a multiple of 16 bytes (TMA pitch rule)."""
    a = torch.zeros(4, 64, dtype=torch.float16, device=DEV)
    w = torch.zeros(64, 520, dtype=torch.int8, device=DEV)
    s = torch.ones(520, dtype=torch.float16, device=DEV)
    with pytest.raises(cuda_pkg.HxbError, match="ldw%16"):
        cuda_pkg.matmul_w8a16(a, w, s)
