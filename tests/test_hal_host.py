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
    assert d.available_devices() == []
    with pytest.raises(pkg.HxbError, match="no CUDA device"):
        d.create_device(0)
    with pytest.raises(pkg.HxbError, match="no CUDA device"):
        d.create_device_by_id(0)
    d.close()


def test_options_initialize_defaults(pkg):
    lib = pkg._native.load()
    o = pkg._native.DriverOptions()
    o.default_device_options.scratch_bytes = 9
    o.default_device_options.queue_wait_timeout_ns = 5
    lib.hxb_hal_driver_options_initialize(ctypes.byref(o))
    assert o.default_device_options.scratch_bytes == 0
    assert o.default_device_options.queue_wait_timeout_ns == 10_000_000_000


def test_device_create_checks_options_before_the_gpu(pkg):
    """create_params flags and a queue wait bound past the maximum are refused
    before any device is touched (iree_hal_hexagon_device_create, api.h:93-96)."""
    lib = pkg._native.load()
    out = ctypes.c_void_p()
    o = pkg._native.DeviceOptions(0, 61_000_000_000)
    st = lib.hxb_hal_device_create(pkg._native.StringView.of("b200"), 0, ctypes.byref(o), None,
                                   pkg._native.Allocator(), ctypes.byref(out))
    assert st == 1 and b"maximum" in lib.hxb_last_error_message()
    params = pkg._native.DeviceCreateParams(1)
    st = lib.hxb_hal_device_create(pkg._native.StringView.of("b200"), 0, None,
                                   ctypes.byref(params), pkg._native.Allocator(),
                                   ctypes.byref(out))
    assert st == 2 and not out.value


def test_driver_module_registry(pkg, monkeypatch):
    """The factory of registration/driver_module.c:65-120: the registry lists
    the b200 driver, creates it by name, refuses other names with UNAVAILABLE
    and a second registration with ALREADY_EXISTS; its try_create reads the
    driver options from the environment and rejects malformed values."""
    lib = pkg._native.load()
    reg = pkg.hal.Registry()
    assert reg.drivers() == [("b200", "NVIDIA B200 (sm_100a) CUDA driver")]
    drv = reg.create("b200")
    assert drv.handle
    drv.close()
    with pytest.raises(pkg.HxbError, match="UNAVAILABLE.*hexagon"):
        reg.create("hexagon")
    assert lib.hxb_hal_driver_module_register(reg.handle) == 7  # ALREADY_EXISTS
    monkeypatch.setenv("HXB_HAL_QUEUE_WAIT_TIMEOUT_MS", "12x")
    with pytest.raises(pkg.HxbError, match="HXB_HAL_QUEUE_WAIT_TIMEOUT_MS"):
        reg.create("b200")
    monkeypatch.setenv("HXB_HAL_QUEUE_WAIT_TIMEOUT_MS", "250")
    monkeypatch.setenv("HXB_HAL_SCRATCH_BYTES", "1048576")
    reg.create("b200").close()
    reg.close()


def test_registry_asks_factories_in_order(pkg):
    """A second factory (here written in Python against the C struct) is
    listed after the b200 one and gets the names b200 does not provide."""
    nat = pkg._native
    calls = []
    infos = (nat.DriverInfo * 1)(nat.DriverInfo(nat.StringView.of("other"),
                                                nat.StringView.of("Other driver")))

    @nat.DriverEnumerateFn
    def enumerate_fn(self, count, out):
        count[0] = 1
        out[0] = ctypes.cast(infos, ctypes.POINTER(nat.DriverInfo))
        return 0

    @nat.DriverTryCreateFn
    def try_create_fn(self, name, alloc, out):
        calls.append(ctypes.string_at(name.data, name.size))
        return 6

    factory = nat.DriverFactory(None, enumerate_fn, try_create_fn)
    reg = pkg.hal.Registry()
    lib = nat.load()
    assert lib.hxb_hal_driver_registry_register_factory(reg.handle, ctypes.byref(factory)) == 0
    assert [d[0] for d in reg.drivers()] == ["b200", "other"]
    with pytest.raises(pkg.HxbError, match="UNAVAILABLE"):
        reg.create("other")
    assert calls == [b"other"]
    reg.close()


def test_host_allocator_owns_host_objects(pkg):
    """Host objects come from the allocator passed at creation and go back to
    it on release (iree_allocator_t semantics: CALLOC then FREE)."""
    nat = pkg._native
    lib = nat.load()
    live, log = {}, []

    @nat.AllocatorCtl
    def ctl(self, command, params, inout):
        if command == 1:  # CALLOC
            n = ctypes.cast(params, ctypes.POINTER(ctypes.c_size_t))[0]
            buf = ctypes.create_string_buffer(n)
            live[ctypes.addressof(buf)] = buf
            inout[0] = ctypes.addressof(buf)
            log.append(("calloc", n))
            return 0
        if command == 3:  # FREE
            live.pop(inout[0], None)
            log.append(("free", 0))
            return 0
        return 2

    alloc = nat.Allocator(None, ctl)
    out = ctypes.c_void_p()
    assert lib.hxb_hal_driver_create(nat.StringView.of("b200"), None, alloc,
                                     ctypes.byref(out)) == 0
    assert len(live) == 1 and log[0][0] == "calloc"
    lib.hxb_hal_driver_release(out)
    assert not live and log[-1][0] == "free"


def test_channel_id_and_argument_checks(pkg):
    """Channels (the HAL collectives the reference leaves unimplemented,
    plugins/runtime/hexagon/channel.c:37-56): an id can be made without a GPU;
    channel creation checks its arguments before touching a device."""
    ida, idb = pkg.hal.channel_id(), pkg.hal.channel_id()
    assert len(ida) == 128 and ida != idb
    lib = pkg._native.load()
    out = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(ida, 128)
    assert lib.hxb_hal_channel_create(None, buf, 0, 2, 10**9, ctypes.byref(out)) == 1
    assert lib.hxb_hal_channel_rank(None) == -1 and lib.hxb_hal_channel_count(None) == 0
