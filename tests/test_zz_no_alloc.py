"""hxb_matmul_f16_noalloc: the f16 matmul for callers that cannot allocate.

A compiled dispatch function only holds the buffers its runtime bound to it,
and code recording a CUDA stream capture may not call cudaMalloc, so neither
can hand hxb_matmul_f16 the workspace it needs for operands whose row pitch is
not a multiple of 16 bytes. hxb_matmul_f16_noalloc re-pitches into a scratch
array built into the library instead. These tests call it through the C ABI
and check it against hxb_matmul_f16 given a workspace from torch and against
the CPU oracle on the unpadded operands, on two different calls in a row (the
scratch keeps the previous call's bytes, so the second call would show stale
data if any were read).

The file is named so that pytest collects it last.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _support import baseline_check

DEV = "cuda:0"
F16, F32 = 0, 1


def _call_both(pkg, oracle, M, N, K, pad_a, pad_b, out_dtype, seed):
    lib = pkg._native.load()
    rng = np.random.default_rng(seed)
    a_big = torch.from_numpy(rng.uniform(-1, 1, (M, K + pad_a)).astype(np.float16)).to(DEV)
    b_big = torch.from_numpy(rng.uniform(-1, 1, (K, N + pad_b)).astype(np.float16)).to(DEV)
    lda, ldb = K + pad_a, N + pad_b
    dt = torch.float16 if out_dtype == F16 else torch.float32
    ws_bytes = lib.hxb_matmul_f16_workspace_bytes(a_big.data_ptr(), lda, b_big.data_ptr(), ldb,
                                                  0, M, N, K)
    assert ws_bytes > 0, "the case must exercise the re-pitch scratch"
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    want = torch.empty(M, N, dtype=dt, device=DEV)
    got = torch.full((M, N), float("nan"), dtype=dt, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    pkg._native.check(lib.hxb_matmul_f16(a_big.data_ptr(), lda, b_big.data_ptr(), ldb, 0, None,
                                         want.data_ptr(), N, out_dtype, M, N, K,
                                         ws.data_ptr(), ws_bytes, stream))
    pkg._native.check(lib.hxb_matmul_f16_noalloc(a_big.data_ptr(), lda, b_big.data_ptr(), ldb,
                                                 0, None, got.data_ptr(), N, out_dtype,
                                                 M, N, K, stream))
    torch.cuda.synchronize()
    ref = oracle.matmul_f32(a_big[:, :K].cpu().numpy(), b_big[:, :N].cpu().numpy())
    return ref, want.float().cpu().numpy(), got.float().cpu().numpy()


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice(cuda_pkg, oracle):
    # Two calls in a row with different shapes and pitches: the second one
    # re-pitches different data into the same scratch.
    cases = [(70, 90, 110, 5, 3, F32, 1), (129, 257, 65, 1, 7, F16, 2)]
    for M, N, K, pad_a, pad_b, out_dtype, seed in cases:
        ref, want, got = _call_both(cuda_pkg, oracle, M, N, K, pad_a, pad_b, out_dtype, seed)
        assert np.isfinite(got).all()
        baseline_check(want, got, f"noalloc {M}x{N}x{K} vs workspace entry point")
        baseline_check(ref, got, f"noalloc {M}x{N}x{K} vs oracle")
        baseline_check(ref, want, f"workspace entry point {M}x{N}x{K} vs oracle")
    assert cuda_pkg.device_status() == 0


def test_noalloc_rejects_operands_beyond_scratch(pkg):
    """Host-side check, made before any device work: an operand whose
    re-pitched copy exceeds the built-in scratch is refused with a message."""
    lib = pkg._native.load()
    M, K, N = 4096, 4097, 64  # lda = 4097 elements: 8194-byte rows, re-pitch needed
    need = lib.hxb_matmul_f16_workspace_bytes(0x100000, K, 0x200000, N, 0, M, N, K)
    assert need > 32 * 1024 * 1024
    status = lib.hxb_matmul_f16_noalloc(0x100000, K, 0x200000, N, 0, None, 0x300000, N,
                                        F16, M, N, K, None)
    assert status == 1  # HXB_STATUS_INVALID_ARGUMENT
    assert b"built-in scratch" in lib.hxb_last_error_message()
