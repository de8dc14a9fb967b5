"""Executable-library and HAL ABI (include/hxb200_hal.h) on the host: the
library query and its export table, argument checking of the dispatch
functions before any device access, and the driver without a GPU.

The shapes mirror plugins/runtime/hexagon/dsp/rt/executable_library.h:40-250
(query, export table, dispatch state) and plugins/runtime/hexagon/api.h:55-114
(driver / device options and creation)."""
from __future__ import annotations

import ctypes

import pytest
import torch


def _exports(pkg):
    lib = pkg._native.load()
    p = lib.hxb_executable_library_query(pkg._native.EXECUTABLE_LIBRARY_VERSION_1, None)
    assert p
    return ctypes.cast(p, ctypes.POINTER(pkg._native.ExecutableLibrary)).contents.exports


def _call(pkg, ordinal, constants, ptrs, lengths):
    ex = _exports(pkg)
    fn_addr = ctypes.cast(ex.ptrs, ctypes.POINTER(ctypes.c_void_p))[ordinal]
    fn = pkg._native.DispatchFn(fn_addr)
    c = (ctypes.c_uint32 * 16)(*(list(constants) + [0] * (16 - len(constants))))
    bp = (ctypes.c_void_p * max(1, len(ptrs)))(*ptrs)
    bl = (ctypes.c_size_t * max(1, len(lengths)))(*lengths)
    env = pkg._native.ExecutableEnvironment(None, None, None, 0)
    ds = pkg._native.DispatchState(1, 1, 1, 1, 1, 1, len(ptrs), ctypes.addressof(c),
                                   ctypes.addressof(bp), ctypes.addressof(bl), None)
    return fn(ctypes.addressof(env), ctypes.addressof(ds), None)


def test_library_query_and_exports(pkg):
    info = pkg.hal.library()
    assert info["version"] == 0x48420001
    assert info["imports"] == 0
    assert [e["name"] for e in info["exports"]] == [
        "matmul_f16", "matmul_w8a16", "attention_f16", "decoder_block_w8a16",
        "attention_gqa_f16"]
    for e in info["exports"]:
        assert e["flags"] & 0x1 and e["flags"] & 0x2      # resources valid, tensor core
        assert 100_000 < e["smem_bytes"] <= 232_448       # one CTA per SM
        assert e["threads"] in (192, 384, 512)
    # the reference's own version code ('HX') and any other are refused
    assert pkg.hal.library(0x48580001) is None
    assert pkg.hal.library(0x48420002) is None


def test_dispatch_functions_check_bindings_before_device_access(pkg):
    lib = pkg._native.load()
    fake = [0x10000 * (i + 1) for i in range(13)]
    # matmul_f16 with 2 bindings (needs 3 or 4)
    assert _call(pkg, 0, [64, 64, 64, 0], fake[:2], [1 << 20] * 2) == 1
    assert b"bindings" in lib.hxb_last_error_message()
    # matmul_f16 with a too-short C binding (64 x 64 f32 = 16 KB)
    assert _call(pkg, 0, [64, 64, 64, 2], fake[:3], [8192, 8192, 8192]) == 1
    assert b"needs 16384" in lib.hxb_last_error_message()
    # matmul_w8a16: scale binding shorter than 2 N bytes
    assert _call(pkg, 1, [16, 256, 64], fake[:4], [2048, 16384, 100, 8192]) == 1
    assert b"binding 2" in lib.hxb_last_error_message()
    # attention: null binding
    ptrs = fake[:4]
    ptrs[2] = 0
    assert _call(pkg, 2, [2, 128, 128, 128, 0, 0], ptrs, [1 << 20] * 4) == 1
    assert b"null" in lib.hxb_last_error_message()
    # decoder block: 12 bindings (needs 13)
    assert _call(pkg, 3, [1, 8, 0, 128, 1, 128, 256, 0, 0], fake[:12], [1 << 24] * 12) == 1
    # GQA attention: K cache binding shorter than B * Hkv * kv_rows * D * 2
    gqa = [1, 9, 3, 64, 0, 64, 128, 64, 0, 1, 0]
    assert _call(pkg, 4, gqa, fake[:4], [1 << 20, 3 * 128 * 64 * 2 - 2, 1 << 20, 1 << 20]) == 1
    assert b"binding 1" in lib.hxb_last_error_message()
    # extents whose byte count overflows 64 bits
    assert _call(pkg, 0, [0xFFFFFFFF] * 3 + [0], fake[:3], [1 << 20] * 3) in (1,)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU path")
def test_driver_without_gpu(pkg):
    d = pkg.hal.Driver()
    assert d.device_count() == 0
    with pytest.raises(pkg.HxbError, match="no CUDA device"):
        d.create_device(0)
    d.close()


def test_options_initialize_defaults(pkg):
    lib = pkg._native.load()
    o = pkg._native.DriverOptions()
    o.default_device_options.ordinal = 7
    o.default_device_options.scratch_bytes = 9
    lib.hxb_hal_driver_options_initialize(ctypes.byref(o))
    assert o.default_device_options.ordinal == 0
    assert o.default_device_options.scratch_bytes == 0
