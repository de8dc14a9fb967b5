"""Python mirror of the executable-library and HAL-runtime ABI
(include/hxb200_hal.h), the shapes of the reference's runtime plugin
(plugins/runtime/hexagon/api.h:55-114; dsp/rt/executable_library.h:40-250):
a driver creates devices, a device owns buffers, timeline semaphores and
command buffers of dispatches of the library's exports, and queue execution
orders them.

Every call goes to libhxb200.so; errors raise HxbError with the library's
message.
"""
from __future__ import annotations

import ctypes
import struct

from . import _native
from ._native import check

COLLECTIVES = {"all_gather": 0, "all_reduce_sum": 1, "reduce_scatter_sum": 2, "broadcast": 3}
DTYPES = {"f16": 0, "f32": 1, "i8": 2}

EXPORTS = {"matmul_f16": 0, "matmul_w8a16": 1, "attention_f16": 2, "decoder_block_w8a16": 3,
           "attention_gqa_f16": 4}


def f32_bits(x: float) -> int:
    """A float as the u32 push constant the exports read."""
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


def library(version: int = _native.EXECUTABLE_LIBRARY_VERSION_1) -> dict | None:
    """The executable library's header and export table, or None when
    `version` is not the one it was built with."""
    lib = _native.load()
    p = lib.hxb_executable_library_query(version, None)
    if not p:
        return None
    libs = ctypes.cast(p, ctypes.POINTER(_native.ExecutableLibrary)).contents
    ex = libs.exports
    exports = []
    for i in range(ex.count):
        a = ex.attrs[i]
        exports.append({"name": ex.names[i].decode(), "flags": a.flags,
                        "smem_bytes": a.smem_bytes, "threads": a.threads})
    return {"version": libs.header.contents.version, "imports": libs.imports.count,
            "exports": exports}


class Driver:
    """A driver (hxb_hal_driver_create); `options` sets the default device
    options of the devices it creates by id."""

    def __init__(self, identifier: str = "b200", scratch_bytes: int = 0,
                 queue_wait_timeout_ns: int = 0, handle=None):
        self._lib = _native.load()
        if handle is not None:  # a driver a factory created
            self.handle = handle
            return
        o = _native.DriverOptions()
        self._lib.hxb_hal_driver_options_initialize(ctypes.byref(o))
        o.default_device_options.scratch_bytes = scratch_bytes
        if queue_wait_timeout_ns:
            o.default_device_options.queue_wait_timeout_ns = queue_wait_timeout_ns
        h = ctypes.c_void_p()
        check(self._lib.hxb_hal_driver_create(_native.StringView.of(identifier), ctypes.byref(o),
                                              _native.Allocator(), ctypes.byref(h)))
        self.handle = h

    def device_count(self) -> int:
        n = ctypes.c_int32()
        check(self._lib.hxb_hal_driver_query_device_count(self.handle, ctypes.byref(n)))
        return n.value

    def available_devices(self) -> list[dict]:
        n = ctypes.c_int32()
        check(self._lib.hxb_hal_driver_query_available_devices(self.handle, None, 0,
                                                               ctypes.byref(n)))
        infos = (_native.DeviceInfo * max(1, n.value))()
        check(self._lib.hxb_hal_driver_query_available_devices(self.handle, infos, n.value,
                                                               ctypes.byref(n)))
        return [{"device_id": i.device_id, "path": i.path.decode(), "name": i.name.decode()}
                for i in infos[:n.value]]

    def create_device_by_id(self, device_id: int = 0) -> "Device":
        h = ctypes.c_void_p()
        check(self._lib.hxb_hal_driver_create_device_by_id(self.handle, device_id, None,
                                                           _native.Allocator(), ctypes.byref(h)))
        return Device(handle=h)

    def create_device(self, ordinal: int = 0, scratch_bytes: int = 0,
                      queue_wait_timeout_ns: int = 0) -> "Device":
        return Device(ordinal, scratch_bytes, queue_wait_timeout_ns)

    def close(self) -> None:
        if self.handle:
            self._lib.hxb_hal_driver_release(self.handle)
            self.handle = None


class Registry:
    """A driver registry (hxb_hal_driver_registry_*) with the b200 module
    registered, as a tool registers driver modules at start-up."""

    def __init__(self, register_b200: bool = True):
        self._lib = _native.load()
        h = ctypes.c_void_p()
        check(self._lib.hxb_hal_driver_registry_create(_native.Allocator(), ctypes.byref(h)))
        self.handle = h
        if register_b200:
            check(self._lib.hxb_hal_driver_module_register(self.handle))

    def drivers(self) -> list[tuple[str, str]]:
        n = ctypes.c_int32()
        check(self._lib.hxb_hal_driver_registry_enumerate(self.handle, None, 0, ctypes.byref(n)))
        infos = (_native.DriverInfo * max(1, n.value))()
        check(self._lib.hxb_hal_driver_registry_enumerate(self.handle, infos, n.value,
                                                          ctypes.byref(n)))
        return [(ctypes.string_at(i.driver_name.data, i.driver_name.size).decode(),
                 ctypes.string_at(i.full_name.data, i.full_name.size).decode())
                for i in infos[:n.value]]

    def create(self, name: str) -> Driver:
        h = ctypes.c_void_p()
        check(self._lib.hxb_hal_driver_registry_try_create(
            self.handle, _native.StringView.of(name), _native.Allocator(), ctypes.byref(h)))
        return Driver(handle=h)

    def close(self) -> None:
        if self.handle:
            self._lib.hxb_hal_driver_registry_release(self.handle)
            self.handle = None


class Device:
    """A device on CUDA device `ordinal` (hxb_hal_device_create; the ordinal is
    the domain id)."""

    def __init__(self, ordinal: int = 0, scratch_bytes: int = 0,
                 queue_wait_timeout_ns: int = 0, handle=None):
        self._lib = _native.load()
        if handle is not None:
            self.handle = handle
            return
        o = _native.DeviceOptions()
        self._lib.hxb_hal_device_options_initialize(ctypes.byref(o))
        o.scratch_bytes = scratch_bytes
        if queue_wait_timeout_ns:
            o.queue_wait_timeout_ns = queue_wait_timeout_ns
        h = ctypes.c_void_p()
        check(self._lib.hxb_hal_device_create(_native.StringView.of("b200"), ordinal,
                                              ctypes.byref(o), None, _native.Allocator(),
                                              ctypes.byref(h)))
        self.handle = h

    @property
    def stream(self) -> int:
        return self._lib.hxb_hal_device_queue_stream(self.handle) or 0

    @property
    def lost(self) -> bool:
        return bool(self._lib.hxb_hal_device_is_lost(self.handle))

    def allocate(self, nbytes: int) -> "Buffer":
        return Buffer(self, nbytes)

    def semaphore(self, initial: int = 0) -> "Semaphore":
        return Semaphore(self, initial)

    def command_buffer(self, binding_capacity: int = 0) -> "CommandBuffer":
        return CommandBuffer(self, binding_capacity)

    def execute(self, command_buffer: "CommandBuffer | None", wait=None, signal=None,
                bindings=None) -> None:
        """Queue `command_buffer` after `wait` = (semaphore, value) is reached;
        then set `signal` = (semaphore, value). `bindings` is the binding
        table: a list of Buffers or (Buffer, offset, length). Does not block."""
        ws, wv = (wait[0].handle, wait[1]) if wait else (None, 0)
        ss, sv = (signal[0].handle, signal[1]) if signal else (None, 0)
        table = None
        if bindings is not None:
            entries = []
            for b in bindings:
                buf, off, ln = (b, 0, b.nbytes) if isinstance(b, Buffer) else b
                entries.append(_native.BufferBinding(buf.handle, off, ln))
            arr = (_native.BufferBinding * max(1, len(entries)))(*entries)
            table = _native.BindingTable(len(entries), arr)
        check(self._lib.hxb_hal_device_queue_execute(
            self.handle, ws, wv, command_buffer.handle if command_buffer else None,
            ctypes.byref(table) if table is not None else None, ss, sv))

    def close(self) -> None:
        if self.handle:
            self._lib.hxb_hal_device_release(self.handle)
            self.handle = None


def slot(index: int, offset: int = 0, length: int = 0) -> _native.BufferRef:
    """A binding that names slot `index` of the binding table given at
    submission (`offset`/`length` bytes inside that binding)."""
    return _native.BufferRef(None, offset, length, index, 0)


class Buffer:
    def __init__(self, device: Device, nbytes: int):
        self._lib = device._lib
        h = ctypes.c_void_p()
        check(self._lib.hxb_hal_buffer_allocate(device.handle, nbytes, ctypes.byref(h)))
        self.handle = h
        self.nbytes = nbytes

    @property
    def device_pointer(self) -> int:
        return self._lib.hxb_hal_buffer_device_pointer(self.handle) or 0

    def write(self, data, offset: int = 0) -> None:
        """Copies a host buffer (bytes or a contiguous numpy array) in."""
        mv = memoryview(data).cast("B")
        buf = (ctypes.c_char * len(mv)).from_buffer_copy(mv)
        check(self._lib.hxb_hal_buffer_write(self.handle, offset, buf, len(mv)))

    def read(self, nbytes: int | None = None, offset: int = 0) -> bytes:
        n = self.nbytes - offset if nbytes is None else nbytes
        buf = (ctypes.c_char * n)()
        check(self._lib.hxb_hal_buffer_read(self.handle, offset, buf, n))
        return bytes(buf)

    def ref(self, offset: int = 0, length: int | None = None) -> _native.BufferRef:
        return _native.BufferRef(self.handle, offset,
                                 self.nbytes - offset if length is None else length, 0, 0)

    def close(self) -> None:
        if self.handle:
            self._lib.hxb_hal_buffer_release(self.handle)
            self.handle = None


class Semaphore:
    def __init__(self, device: Device, initial: int):
        self._lib = device._lib
        h = ctypes.c_void_p()
        check(self._lib.hxb_hal_semaphore_create(device.handle, initial, ctypes.byref(h)))
        self.handle = h

    @property
    def value(self) -> int:
        v = ctypes.c_uint64()
        check(self._lib.hxb_hal_semaphore_query(self.handle, ctypes.byref(v)))
        return v.value

    def signal(self, value: int) -> None:
        check(self._lib.hxb_hal_semaphore_signal(self.handle, value))

    def wait(self, value: int, timeout_s: float = 10.0) -> None:
        check(self._lib.hxb_hal_semaphore_wait(self.handle, value, int(timeout_s * 1e9)))

    def close(self) -> None:
        if self.handle:
            self._lib.hxb_hal_semaphore_release(self.handle)
            self.handle = None


class CommandBuffer:
    def __init__(self, device: Device, binding_capacity: int = 0):
        self._lib = device._lib
        h = ctypes.c_void_p()
        check(self._lib.hxb_hal_command_buffer_create(device.handle, binding_capacity,
                                                      ctypes.byref(h)))
        self.handle = h

    def begin(self) -> None:
        check(self._lib.hxb_hal_command_buffer_begin(self.handle))

    def dispatch(self, export: str | int, constants, bindings) -> None:
        """Records one dispatch: `bindings` are Buffers or BufferRefs
        (slot(i) for a binding-table slot)."""
        ordinal = EXPORTS[export] if isinstance(export, str) else int(export)
        c = (ctypes.c_uint32 * max(1, len(constants)))(*[int(x) & 0xFFFFFFFF for x in constants])
        refs = [b.ref() if isinstance(b, Buffer) else b for b in bindings]
        arr = (_native.BufferRef * max(1, len(refs)))(*refs)
        check(self._lib.hxb_hal_command_buffer_dispatch(self.handle, ordinal, c, len(constants),
                                                        arr, len(refs)))

    def collective(self, channel: "Channel", op: str, dtype: str, send, recv,
                   count: int) -> None:
        """Records a collective (COLLECTIVES) of `count` elements from `send`
        into `recv` (Buffers or BufferRefs) over `channel`."""
        refs = [b.ref() if isinstance(b, Buffer) else b for b in (send, recv)]
        check(self._lib.hxb_hal_command_buffer_collective(
            self.handle, channel.handle, COLLECTIVES[op], DTYPES[dtype], refs[0], refs[1],
            count))

    def end(self) -> None:
        check(self._lib.hxb_hal_command_buffer_end(self.handle))

    def close(self) -> None:
        if self.handle:
            self._lib.hxb_hal_command_buffer_release(self.handle)
            self.handle = None


def channel_id() -> bytes:
    """A fresh channel id (rank 0 makes it and shares it with the others)."""
    lib = _native.load()
    buf = ctypes.create_string_buffer(128)
    check(lib.hxb_hal_channel_id_create(buf))
    return buf.raw


class Channel:
    """`rank` of `count` devices running collectives together (an NCCL
    communicator under hxb_hal_channel_create)."""

    def __init__(self, device: Device, channel_id: bytes, rank: int, count: int,
                 timeout_s: float = 60.0):
        self._lib = device._lib
        idb = ctypes.create_string_buffer(bytes(channel_id), 128)
        h = ctypes.c_void_p()
        check(self._lib.hxb_hal_channel_create(device.handle, idb, rank, count,
                                               int(timeout_s * 1e9), ctypes.byref(h)))
        self.handle = h

    @property
    def rank(self) -> int:
        return self._lib.hxb_hal_channel_rank(self.handle)

    @property
    def count(self) -> int:
        return self._lib.hxb_hal_channel_count(self.handle)

    def close(self) -> None:
        if self.handle:
            self._lib.hxb_hal_channel_release(self.handle)
            self.handle = None
