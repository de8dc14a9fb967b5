"""The bounded-wait failure path of the kernels, run on the GPU without a
fault: hxb_selftest_wait_timeout makes the same bounded mbarrier wait every
pipelined kernel uses run out after a few milliseconds (nothing ever arrives
at its barrier), with a bulk copy in flight and TMEM held. The kernel must
return, report the timeout through the device status word, let the copy
land, free its TMEM, and leave the context usable for the next dispatch."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _support import baseline_check

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("limit_ms", [2, 20])
def test_bounded_wait_runs_out_and_context_survives(cuda_pkg, oracle, limit_ms):
    lib = cuda_pkg._native.load()
    cuda_pkg.device_status(clear=True)
    src = torch.arange(1024, dtype=torch.int32, device=DEV)  # 4096 bytes
    result = torch.full((4,), -1, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    cuda_pkg._native.check(lib.hxb_selftest_wait_timeout(limit_ms * 1_000_000, src.data_ptr(),
                                                         result.data_ptr(), stream))
    e1.record()
    torch.cuda.synchronize()
    took_ms = e0.elapsed_time(e1)
    assert limit_ms * 0.9 <= took_ms < limit_ms + 50, took_ms
    assert result.tolist() == [0, 1, 1, 1]  # no wait succeeded, abort raised, copy landed, TMEM freed
    assert cuda_pkg.device_status(clear=False) & 1  # stays set until cleared
    assert cuda_pkg.device_status(clear=True) & 1
    assert cuda_pkg.device_status(clear=False) == 0
    # the next dispatch on the same device (a TMEM-allocating tcgen05 GEMM) is correct
    rng = np.random.default_rng(limit_ms)
    a = (rng.random((256, 320)) * 2 - 1).astype(np.float16)
    b = (rng.random((320, 384)) * 2 - 1).astype(np.float16)
    c = cuda_pkg.matmul(torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV),
                        out_dtype=torch.float32)
    torch.cuda.synchronize()
    baseline_check(oracle.matmul_f32(a, b), c.cpu().numpy(), "matmul after a timed-out wait")
    assert cuda_pkg.device_status() == 0


def test_selftest_rejects_long_limits(cuda_pkg):
    lib = cuda_pkg._native.load()
    src = torch.zeros(1024, dtype=torch.int32, device=DEV)
    res = torch.zeros(4, dtype=torch.int32, device=DEV)
    assert lib.hxb_selftest_wait_timeout(2_000_000_000, src.data_ptr(), res.data_ptr(), None) == 1
    assert b"outside" in lib.hxb_last_error_message()
