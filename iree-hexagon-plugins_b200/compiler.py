"""Python mirror of the compiler half of the B200 drop-in
(include/hxb200_compiler.h): compile linalg-on-tensors MLIR text into an
executable of B200 dispatches, wrap it as the hal.executable.binary the IREE
target would emit, and load / invoke it on a HAL device -- the
`iree-compile` -> `iree-run-module` path of the reference
(examples/compiling.md, examples/running.md), with the target's decisions
logged the way the reference's planner traces them.

Every call goes to libhxb200.so; errors raise HxbError with the library's
message (and, for compilation, the compiler's log).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _native
from ._native import HxbError, check

ELEMENT_DTYPES = {0: np.float16, 1: np.float32, 2: np.int8}


@dataclass
class Executable:
    data: bytes
    log: str

    def binary_mlir(self, symbol: str = "b200") -> str:
        """The executable as the target's serializeExecutable would emit it
        (a hal.executable.binary with format and MIME type)."""
        lib = _native.load()
        buf = ctypes.create_string_buffer(self.data, len(self.data))
        out = ctypes.c_void_p()
        check(lib.hxb_executable_binary_mlir(buf, len(self.data), symbol.encode(),
                                             ctypes.byref(out)))
        try:
            return ctypes.string_at(out.value).decode()
        finally:
            lib.hxb_compiler_free(out)


def compile_mlir(text: str, *, matmul: bool = True, w8a16: bool = True,
                 attention: bool = True, num_sms: int = 0) -> Executable:
    """Compiles MLIR text; raises HxbError (with the compiler's log) when a
    function holds an operation the target forms no dispatch for."""
    lib = _native.load()
    opts = _native.CompilerOptions()
    lib.hxb_compiler_options_initialize(ctypes.byref(opts))
    opts.enable_matmul, opts.enable_w8a16, opts.enable_attention = int(matmul), int(w8a16), \
        int(attention)
    opts.num_sms = num_sms
    raw = text.encode()
    blob, size, log = ctypes.c_void_p(), ctypes.c_size_t(), ctypes.c_void_p()
    status = lib.hxb_compile_mlir(raw, len(raw), ctypes.byref(opts), ctypes.byref(blob),
                                  ctypes.byref(size), ctypes.byref(log))
    log_text = ctypes.string_at(log.value).decode() if log.value else ""
    lib.hxb_compiler_free(log)
    if status != 0:
        raise HxbError(status, log_text.strip())
    try:
        return Executable(ctypes.string_at(blob.value, size.value), log_text)
    finally:
        lib.hxb_compiler_free(blob)


class Module:
    """An executable loaded on a HAL device (hal.Device)."""

    def __init__(self, device, executable: Executable):
        self._lib = _native.load()
        self.device = device
        self._blob = ctypes.create_string_buffer(executable.data, len(executable.data))
        h = ctypes.c_void_p()
        check(self._lib.hxb_module_load(device.handle, self._blob, len(executable.data),
                                        ctypes.byref(h)))
        self.handle = h

    def functions(self) -> list[str]:
        n = self._lib.hxb_module_function_count(self.handle)
        return [self._lib.hxb_module_function_name(self.handle, i).decode() for i in range(n)]

    def signature(self, name: str) -> tuple[list, list]:
        """([(dtype, shape)] of the arguments, same for the results)."""
        na, nr = ctypes.c_int32(), ctypes.c_int32()
        check(self._lib.hxb_module_signature(self.handle, name.encode(), ctypes.byref(na),
                                             ctypes.byref(nr), None, 0))
        descs = (_native.TensorDesc * max(1, na.value + nr.value))()
        check(self._lib.hxb_module_signature(self.handle, name.encode(), ctypes.byref(na),
                                             ctypes.byref(nr), descs, na.value + nr.value))
        sig = [(ELEMENT_DTYPES[d.element_type], tuple(d.dims[:d.rank])) for d in descs]
        return sig[:na.value], sig[na.value:na.value + nr.value]

    def dispatch_count(self, name: str) -> int:
        return self._lib.hxb_module_dispatch_count(self.handle, name.encode())

    def invoke(self, name: str, args, results, wait=None, signal=None) -> None:
        """Queues function `name` over HAL buffers (hal.Buffer); `wait` /
        `signal` are (semaphore, value) pairs. Does not block."""
        def table(bufs):
            arr = (_native.BufferBinding * max(1, len(bufs)))(
                *[_native.BufferBinding(b.handle, 0, b.nbytes) for b in bufs])
            return arr
        a, r = table(args), table(results)
        ws, wv = (wait[0].handle, wait[1]) if wait else (None, 0)
        ss, sv = (signal[0].handle, signal[1]) if signal else (None, 0)
        check(self._lib.hxb_module_invoke(self.handle, name.encode(), a, len(args), r,
                                          len(results), ws, wv, ss, sv))

    def close(self) -> None:
        if self.handle:
            self._lib.hxb_module_release(self.handle)
            self.handle = None
