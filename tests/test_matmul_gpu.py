"""Parity of the tcgen05 f16 matmul dispatch (through the C ABI) with the
oracle and with the reference's golden micro-model outputs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _support import (baseline_check, compare, golden_expected, golden_inputs,
                      golden_manifest, select_rows)

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _guarded_empty(shape, dtype, guard=4096):
    """Output tensor inside a buffer with canary bands on both sides."""
    n = int(np.prod(shape))
    buf = torch.empty(n + 2 * guard, dtype=dtype, device=DEV)
    buf.view(torch.int16 if dtype == torch.float16 else torch.int32).fill_(0x7E7E)
    canary = buf.clone()
    return buf[guard:guard + n].view(shape), buf, canary, guard


def _check_canary(buf, canary, guard):
    # compare bit patterns: the canary is a NaN pattern, and NaN != NaN
    iv = torch.int16 if buf.dtype == torch.float16 else torch.int32
    b, c = buf.view(iv), canary.view(iv)
    assert torch.equal(b[:guard], c[:guard]), "write before the output buffer"
    assert torch.equal(b[-guard:], c[-guard:]), "write past the output buffer"


def test_hmx_known_answer_bit_exact(cuda_pkg, oracle):
    """accumulator_test.c:14-42: exactly representable inputs, sparse weight;
    single MMA and two accumulating MMAs (as matmul + init) must be exact."""
    a, w, e1 = oracle.hmx_known_answer(1)
    _, _, e2 = oracle.hmx_known_answer(2)
    at, wt = torch.from_numpy(a).to(DEV), torch.from_numpy(w).to(DEV)
    c1 = cuda_pkg.matmul(at, wt)
    c2 = cuda_pkg.matmul(at, wt, init=c1.clone())
    torch.cuda.synchronize()
    assert np.array_equal(c1.cpu().numpy(), e1)
    assert np.array_equal(c2.cpu().numpy(), e2)


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (128, 256, 64), (256, 512, 2048),
                                   (4096, 4096, 1024), (300, 200, 100), (1, 8, 8)])
@pytest.mark.parametrize("out", [torch.float16, torch.float32])
def test_matmul_vs_oracle(cuda_pkg, oracle, M, N, K, out):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    c, buf, canary, guard = _guarded_empty((M, N), out)
    cuda_pkg.matmul(torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV),
                    out_dtype=out, out=c)
    torch.cuda.synchronize()
    _check_canary(buf, canary, guard)
    baseline_check(oracle.matmul_f32(a, b), c.float().cpu().numpy(), f"{M}x{N}x{K}")
    assert cuda_pkg.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (17, 19, 23), (129, 257, 65)])
def test_matmul_transposed_rhs_vs_oracle(cuda_pkg, oracle, M, N, K):
    rng = np.random.default_rng(42)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    bt = rng.uniform(-1, 1, (N, K)).astype(np.float16)
    c = cuda_pkg.matmul(torch.from_numpy(a).to(DEV), torch.from_numpy(bt).to(DEV),
                        transpose_b=True, out_dtype=torch.float32)
    torch.cuda.synchronize()
    baseline_check(oracle.matmul_f32(a, bt, transpose_b=True), c.cpu().numpy())


@pytest.mark.parametrize("out", [torch.float16, torch.float32])
def test_matmul_init_is_added(cuda_pkg, oracle, out):
    """linalg.matmul accumulates into its DPS init (hmx.c:334-336)."""
    rng = np.random.default_rng(9)
    M, N, K = 200, 384, 320
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    init = rng.standard_normal((M, N)).astype(np.float16 if out == torch.float16 else np.float32)
    c = cuda_pkg.matmul(torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV),
                        out_dtype=out, init=torch.from_numpy(init).to(DEV))
    torch.cuda.synchronize()
    baseline_check(oracle.matmul_f32(a, b, init=init.astype(np.float32)),
                   c.float().cpu().numpy())


def _golden_matmul_keys():
    return [k for k, e in golden_manifest().items() if "matmul" in e["model"]]


@pytest.mark.parametrize("key", _golden_matmul_keys())
def test_matmul_vs_reference_golden(cuda_pkg, oracle, key):
    """The reference's micro models (integration_tests/models/micro/hmx/* and
    matmul-1024x1024x1024-f16) under their own model.yaml tolerances, and the
    BASELINE bar against the oracle."""
    entry = golden_manifest()[key]
    a, b = golden_inputs(key)
    transposed = "rhs-transposed" in key
    out = torch.float16 if entry["out_dtype"] == "float16" else torch.float32
    ad, bd = a.to(DEV), b.to(DEV)
    if a.dim() == 3:
        got = torch.stack([cuda_pkg.matmul(ad[i], bd[i], out_dtype=out)
                           for i in range(a.shape[0])])
        ref = np.stack([oracle.matmul_f32(a[i].numpy(), b[i].numpy())
                        for i in range(a.shape[0])])
    else:
        got = cuda_pkg.matmul(ad, bd, transpose_b=transposed, out_dtype=out)
        ref = oracle.matmul_f32(a.numpy(), b.numpy(), transpose_b=transposed)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    exp, rows = golden_expected(key)
    tol = entry["tolerances"]
    c = compare(exp, select_rows(got, rows), tol["atol"], tol["rtol"])
    assert c.close, f"{key}: {c}"
    assert c.rel_l2_percent <= tol["relative_l2_percent"], f"{key}: {c}"
    baseline_check(ref, got.astype(np.float32), key)


def test_matmul_strided_operands(cuda_pkg, oracle):
    """Row pitches larger than the extent, including pitches that need the
    re-pitch workspace (odd element counts)."""
    rng = np.random.default_rng(4)
    M, N, K = 70, 90, 110
    abig = rng.uniform(-1, 1, (M, K + 5)).astype(np.float16)
    bbig = rng.uniform(-1, 1, (K, N + 3)).astype(np.float16)
    ad = torch.from_numpy(abig).to(DEV)[:, :K]
    bd = torch.from_numpy(bbig).to(DEV)[:, :N]
    c = cuda_pkg.matmul(ad, bd, out_dtype=torch.float32)
    torch.cuda.synchronize()
    baseline_check(oracle.matmul_f32(abig[:, :K], bbig[:, :N]), c.cpu().numpy())


def test_bad_arguments_raise(cuda_pkg):
    a = torch.zeros(4, 8, dtype=torch.float16, device=DEV)
    b = torch.zeros(8, 4, dtype=torch.float16, device=DEV)
    lib = cuda_pkg._native.load()
    # ldc < N
    st = lib.hxb_matmul_f16(a.data_ptr(), 8, b.data_ptr(), 4, 0, None, a.data_ptr(), 2, 0,
                            4, 4, 8, None, 0, None)
    assert st == 1
    # workspace required but missing: ldb = 4 (8-byte rows) breaks the
    # 16-byte TMA pitch rule, so B must be re-pitched
    st = lib.hxb_matmul_f16(a.data_ptr(), 8, b.data_ptr(), 4, 0, None, a.data_ptr(), 4, 0,
                            4, 4, 8, None, 0, None)
    assert st == 1
    assert b"workspace" in lib.hxb_last_error_message()


@pytest.mark.parametrize("M,N,K,bn,sk,tb,out", [
    (1024, 1024, 1024, 256, 4, False, torch.float16),
    (1024, 1024, 1024, 128, 2, False, torch.float32),
    (512, 512, 8192, 128, 8, False, torch.float16),
    (128, 8192, 2048, 256, 4, True, torch.float16),
    (300, 200, 1000, 64, 4, False, torch.float32),  # ragged M, N and K
    (129, 257, 520, 128, 8, True, torch.float16),   # K-blocks not divisible by the split
    (64, 64, 128, 64, 2, False, torch.float16),
])
def test_split_k_cluster_kernel(cuda_pkg, oracle, M, N, K, bn, sk, tb, out):
    """The split-K kernel (a cluster of split_k CTAs per tile, partials summed
    through distributed shared memory) against the oracle, with canary bands
    around the output."""
    lib = cuda_pkg._native.load()
    rng = np.random.default_rng(M + N + K + sk)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (N, K) if tb else (K, N)).astype(np.float16)
    c, buf, canary, guard = _guarded_empty((M, N), out)
    ad, bd = torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV)
    cuda_pkg._native.check(lib.hxb_matmul_f16_tiled(
        ad.data_ptr(), K, bd.data_ptr(), K if tb else N, int(tb), c.data_ptr(), N,
        0 if out == torch.float16 else 1, M, N, K, bn, 1, sk, 1,
        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    _check_canary(buf, canary, guard)
    baseline_check(oracle.matmul_f32(a, b, transpose_b=tb), c.float().cpu().numpy(),
                   f"split-k {sk} bn {bn} {M}x{N}x{K}")
    # deterministic: the cluster sums its partials in rank order
    c2 = torch.empty_like(c)
    cuda_pkg._native.check(lib.hxb_matmul_f16_tiled(
        ad.data_ptr(), K, bd.data_ptr(), K if tb else N, int(tb), c2.data_ptr(), N,
        0 if out == torch.float16 else 1, M, N, K, bn, 1, sk, 1,
        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(c, c2)
    assert cuda_pkg.device_status() == 0


@pytest.mark.parametrize("M,N,K,bn,gm,tb,out", [
    (1024, 1024, 1024, 256, 4, False, torch.float16),
    (1024, 1024, 1024, 128, 1, True, torch.float32),
    (2048, 4096, 2048, 256, 8, False, torch.float16),   # more tiles than SM pairs
    (300, 200, 1000, 256, 1, False, torch.float32),     # ragged: the second CTA's rows past M
    (129, 264, 520, 128, 2, True, torch.float16),       # one tile row, ragged everything
    (4096, 384, 4096, 128, 16, False, torch.float16),
    (512, 8192, 512, 256, 4, True, torch.float16),
    # 512-column pair tiles: two N = 256 MMA chunks per A stage, one accumulator
    (2048, 4096, 2048, 512, 8, False, torch.float16),
    (300, 1000, 1000, 512, 1, True, torch.float32),
    (1024, 1536, 512, 512, 4, False, torch.float32),
])
def test_cta_pair_kernel(cuda_pkg, oracle, M, N, K, bn, gm, tb, out):
    """The CTA-pair kernel (256-row tiles, cta_group::2 MMAs issued by the
    leader CTA, each CTA loading half of A and half of B) against the oracle,
    with canary bands around the output, and bit-identical on a rerun."""
    lib = cuda_pkg._native.load()
    rng = np.random.default_rng(M + 2 * N + 3 * K + bn)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (N, K) if tb else (K, N)).astype(np.float16)
    c, buf, canary, guard = _guarded_empty((M, N), out)
    ad, bd = torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV)

    def run(dst):
        cuda_pkg._native.check(lib.hxb_matmul_f16_tiled(
            ad.data_ptr(), K, bd.data_ptr(), K if tb else N, int(tb), dst.data_ptr(), N,
            0 if out == torch.float16 else 1, M, N, K, bn, gm, 1, 2,
            torch.cuda.current_stream().cuda_stream))

    run(c)
    torch.cuda.synchronize()
    _check_canary(buf, canary, guard)
    baseline_check(oracle.matmul_f32(a, b, transpose_b=tb), c.float().cpu().numpy(),
                   f"cta pair bn {bn} {M}x{N}x{K}")
    c2 = torch.empty_like(c)
    run(c2)
    torch.cuda.synchronize()
    assert torch.equal(c, c2)
    assert cuda_pkg.device_status() == 0


def test_cta_pair_rejects_split_and_narrow_tiles(cuda_pkg):
    """A CTA pair takes block_n 128, 256 or 512 and no K split; 512 needs a pair."""
    lib = cuda_pkg._native.load()
    a = torch.zeros(256, 256, dtype=torch.float16, device=DEV)
    for bn, sk, pair in ((64, 1, 2), (256, 2, 2), (512, 1, 1)):
        st = lib.hxb_matmul_f16_tiled(a.data_ptr(), 256, a.data_ptr(), 256, 0, a.data_ptr(), 256,
                                      0, 256, 256, 256, bn, 1, sk, pair, None)
        assert st == 1


def test_split_k_with_init_through_the_planner(cuda_pkg, oracle):
    """hxb_matmul_f16 with a C_init on a shape the planner splits."""
    lib = cuda_pkg._native.load()
    import ctypes
    M, N, K = 256, 512, 4096
    bn, gm, sk = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    cuda_pkg._native.check(lib.hxb_plan_matmul_f16(M, N, K, 0, 148, ctypes.byref(bn),
                                                   ctypes.byref(gm), ctypes.byref(sk), None))
    rng = np.random.default_rng(31)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    init = rng.standard_normal((M, N)).astype(np.float32)
    c = cuda_pkg.matmul(torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV),
                        out_dtype=torch.float32, init=torch.from_numpy(init).to(DEV))
    torch.cuda.synchronize()
    baseline_check(oracle.matmul_f32(a, b, init=init), c.cpu().numpy(),
                   f"planned {M}x{N}x{K} split {sk.value}")
