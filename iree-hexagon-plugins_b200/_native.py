"""ctypes binding of libhxb200.so, the C ABI declared in include/hxb200.h.

Nothing here computes: every call goes to the CUDA library. If the library is
missing or cannot be loaded the import fails loudly -- there is no CPU
fallback anywhere in the product path.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libhxb200.so"

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_vp = ctypes.c_void_p
c_size = ctypes.c_size_t
c_u64 = ctypes.c_uint64
c_float = ctypes.c_float

# name -> (restype, argtypes). Kept 1:1 with include/*.h; a test checks that
# the library exports every function the headers declare.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "hxb_abi_version": (c_int, []),
    "hxb_last_error_message": (ctypes.c_char_p, []),
    "hxb_device_status": (c_int, [c_int, ctypes.POINTER(c_int)]),
    "hxb_selftest_wait_timeout": (c_int, [c_u64, c_vp, c_vp, c_vp]),
    "hxb_matmul_f16": (c_int, [c_vp, c_i64, c_vp, c_i64, c_int, c_vp, c_vp, c_i64,
                               c_int, c_i64, c_i64, c_i64, c_vp, c_size, c_vp]),
    "hxb_matmul_f16_workspace_bytes": (c_size, [c_vp, c_i64, c_vp, c_i64, c_int,
                                                c_i64, c_i64, c_i64]),
    "hxb_matmul_f16_noalloc": (c_int, [c_vp, c_i64, c_vp, c_i64, c_int, c_vp, c_vp,
                                       c_i64, c_int, c_i64, c_i64, c_i64, c_vp]),
    "hxb_plan_matmul_f16": (c_int, [c_i64, c_i64, c_i64, c_int, c_int, ctypes.POINTER(c_int),
                                    ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                                    ctypes.POINTER(c_int)]),
    "hxb_matmul_f16_tiled": (c_int, [c_vp, c_i64, c_vp, c_i64, c_int, c_vp, c_i64, c_int,
                                     c_i64, c_i64, c_i64, c_int, c_int, c_int, c_int, c_vp]),
    "hxb_matmul_w8a16": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_i64,
                                 c_i64, c_i64, c_i64, c_vp]),
    "hxb_plan_matmul_w8a16": (c_int, [c_i64, c_i64, c_i64, c_int, ctypes.POINTER(c_int),
                                      ctypes.POINTER(c_int), ctypes.POINTER(ctypes.c_int32),
                                      c_i64, ctypes.POINTER(c_i64)]),
    "hxb_attention_f16": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64,
                                  c_i64, c_float, c_int, c_vp]),
    "hxb_matmul_w8a16_residual": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp,
                                          c_i64, c_i64, c_i64, c_i64, c_vp]),
    "hxb_matmul_w8a16_workspace_bytes": (c_size, [c_i64, c_i64, c_i64]),
    "hxb_matmul_w8a16_streamk": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64,
                                         c_i64, c_i64, c_i64, c_vp, c_size, c_vp]),
    "hxb_attention_f16_bshd": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                       c_i64, c_i64, c_i64, c_i64, c_i64, c_float, c_int,
                                       c_vp]),
    "hxb_attention_gqa_f16": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64,
                                      c_i64, c_i64, c_i64, c_i64, c_float, c_int, c_int, c_vp,
                                      c_size, c_vp]),
    "hxb_attention_gqa_workspace_bytes": (c_size, [c_i64, c_i64, c_i64, c_i64, c_i64, c_i64]),
    "hxb_rmsnorm_f16": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_float, c_vp]),
    "hxb_rope_f16": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_float, c_vp]),
    "hxb_swiglu_f16": (c_int, [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "hxb_matmul_f16_allgather": (c_int, [c_vp, c_i64, c_vp, c_i64, c_int, c_vp, c_vp, c_int,
                                         c_i64, c_i64, c_i64, c_i64, c_vp]),
    "hxb_matmul_w8a16_allgather": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_int,
                                           c_i64, c_i64, c_i64, c_i64, c_vp, c_size, c_vp]),
    "hxb_peer_barrier": (c_int, [c_vp, c_int, c_int, ctypes.c_uint32, c_vp]),
    "hxb_gather_column_blocks_f16": (c_int, [c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "hxb_ipc_get_handle": (c_int, [c_vp, c_vp, ctypes.POINTER(c_i64)]),
    "hxb_ipc_open": (c_int, [c_vp, c_i64, ctypes.POINTER(c_vp)]),
    "hxb_ipc_close": (c_int, [c_vp, c_i64]),
    "hxb_decoder_block_workspace_bytes": (c_size, [c_vp, c_i64, c_i64]),
    "hxb_decoder_block_cached_workspace_bytes": (c_size, [c_vp, c_i64, c_i64]),
    "hxb_decoder_block_w8a16_cached": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp,
                                               c_i64, c_vp, c_size, c_vp]),
    "hxb_kv_cache_write_f16": (c_int, [c_vp, c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64,
                                       c_i64, c_i64, c_vp]),
    "hxb_decoder_block_w8a16": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp,
                                        c_size, c_vp]),
    # include/hxb200_hal.h: executable library
    "hxb_executable_library_query": (c_vp, [ctypes.c_uint32, c_vp]),
    # include/hxb200_hal.h: HAL runtime
    "hxb_hal_device_options_initialize": (None, [c_vp]),
    "hxb_hal_driver_options_initialize": (None, [c_vp]),
    "hxb_hal_driver_create": (c_int, ["StringView", c_vp, "Allocator", ctypes.POINTER(c_vp)]),
    "hxb_hal_driver_query_device_count": (c_int, [c_vp, ctypes.POINTER(ctypes.c_int32)]),
    "hxb_hal_driver_query_available_devices": (c_int, [c_vp, c_vp, ctypes.c_int32,
                                                       ctypes.POINTER(ctypes.c_int32)]),
    "hxb_hal_driver_create_device_by_id": (c_int, [c_vp, c_u64, c_vp, "Allocator",
                                                   ctypes.POINTER(c_vp)]),
    "hxb_hal_driver_release": (None, [c_vp]),
    "hxb_hal_device_create": (c_int, ["StringView", c_int, c_vp, c_vp, "Allocator",
                                      ctypes.POINTER(c_vp)]),
    "hxb_hal_device_release": (None, [c_vp]),
    "hxb_hal_device_queue_stream": (c_vp, [c_vp]),
    "hxb_hal_device_is_lost": (c_int, [c_vp]),
    "hxb_hal_driver_registry_create": (c_int, ["Allocator", ctypes.POINTER(c_vp)]),
    "hxb_hal_driver_registry_release": (None, [c_vp]),
    "hxb_hal_driver_registry_register_factory": (c_int, [c_vp, c_vp]),
    "hxb_hal_driver_registry_enumerate": (c_int, [c_vp, c_vp, ctypes.c_int32,
                                                  ctypes.POINTER(ctypes.c_int32)]),
    "hxb_hal_driver_registry_try_create": (c_int, [c_vp, "StringView", "Allocator",
                                                   ctypes.POINTER(c_vp)]),
    "hxb_hal_driver_module_register": (c_int, [c_vp]),
    "hxb_hal_buffer_allocate": (c_int, [c_vp, c_u64, ctypes.POINTER(c_vp)]),
    "hxb_hal_buffer_device_pointer": (c_vp, [c_vp]),
    "hxb_hal_buffer_byte_length": (c_u64, [c_vp]),
    "hxb_hal_buffer_write": (c_int, [c_vp, c_u64, c_vp, c_u64]),
    "hxb_hal_buffer_read": (c_int, [c_vp, c_u64, c_vp, c_u64]),
    "hxb_hal_buffer_release": (None, [c_vp]),
    "hxb_hal_semaphore_create": (c_int, [c_vp, c_u64, ctypes.POINTER(c_vp)]),
    "hxb_hal_semaphore_query": (c_int, [c_vp, ctypes.POINTER(c_u64)]),
    "hxb_hal_semaphore_signal": (c_int, [c_vp, c_u64]),
    "hxb_hal_semaphore_wait": (c_int, [c_vp, c_u64, c_u64]),
    "hxb_hal_semaphore_release": (None, [c_vp]),
    "hxb_hal_command_buffer_create": (c_int, [c_vp, ctypes.c_uint32, ctypes.POINTER(c_vp)]),
    "hxb_hal_command_buffer_begin": (c_int, [c_vp]),
    "hxb_hal_command_buffer_dispatch": (c_int, [c_vp, ctypes.c_uint32,
                                                ctypes.POINTER(ctypes.c_uint32), ctypes.c_uint32,
                                                c_vp, ctypes.c_uint32]),
    "hxb_hal_command_buffer_end": (c_int, [c_vp]),
    "hxb_hal_command_buffer_release": (None, [c_vp]),
    # include/hxb200_compiler.h: the target's compiler stand-in and its runtime
    "hxb_compiler_options_initialize": (None, [c_vp]),
    "hxb_compile_mlir": (c_int, [ctypes.c_char_p, c_size, c_vp, ctypes.POINTER(c_vp),
                                 ctypes.POINTER(c_size), ctypes.POINTER(c_vp)]),
    "hxb_compiler_free": (None, [c_vp]),
    "hxb_executable_binary_mlir": (c_int, [c_vp, c_size, ctypes.c_char_p, ctypes.POINTER(c_vp)]),
    "hxb_module_load": (c_int, [c_vp, c_vp, c_size, ctypes.POINTER(c_vp)]),
    "hxb_module_release": (None, [c_vp]),
    "hxb_module_function_count": (ctypes.c_int32, [c_vp]),
    "hxb_module_function_name": (ctypes.c_char_p, [c_vp, ctypes.c_int32]),
    "hxb_module_signature": (c_int, [c_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32),
                                     ctypes.POINTER(ctypes.c_int32), c_vp, ctypes.c_int32]),
    "hxb_module_dispatch_count": (ctypes.c_int32, [c_vp, ctypes.c_char_p]),
    "hxb_module_invoke": (c_int, [c_vp, ctypes.c_char_p, c_vp, ctypes.c_uint32, c_vp,
                                  ctypes.c_uint32, c_vp, c_u64, c_vp, c_u64]),
    "hxb_hal_channel_id_create": (c_int, [c_vp]),
    "hxb_hal_channel_create": (c_int, [c_vp, c_vp, ctypes.c_int32, ctypes.c_int32, c_u64,
                                       ctypes.POINTER(c_vp)]),
    "hxb_hal_channel_rank": (ctypes.c_int32, [c_vp]),
    "hxb_hal_channel_count": (ctypes.c_int32, [c_vp]),
    "hxb_hal_channel_release": (None, [c_vp]),
    "hxb_hal_command_buffer_collective": (c_int, [c_vp, c_vp, c_int, c_int, "BufferRef",
                                                  "BufferRef", c_u64]),
    "hxb_hal_device_queue_execute": (c_int, [c_vp, c_vp, c_u64, c_vp, c_vp, c_vp, c_u64]),
}


# ----------------------------------------------- include/hxb200_hal.h structs

EXECUTABLE_LIBRARY_VERSION_1 = 0x48420001


class ExecutableEnvironment(ctypes.Structure):
    _fields_ = [("constants", c_vp), ("stream", c_vp), ("scratch", c_vp),
                ("scratch_bytes", c_u64)]


class DispatchState(ctypes.Structure):
    _fields_ = [("workgroup_size_x", ctypes.c_uint32), ("workgroup_size_y", ctypes.c_uint32),
                ("workgroup_size_z", ctypes.c_uint16), ("workgroup_count_x", ctypes.c_uint32),
                ("workgroup_count_y", ctypes.c_uint32), ("workgroup_count_z", ctypes.c_uint16),
                ("binding_count", ctypes.c_uint8), ("constants", c_vp),
                ("binding_ptrs", c_vp), ("binding_lengths", c_vp), ("reserved", c_vp)]


DispatchFn = ctypes.CFUNCTYPE(c_int, c_vp, c_vp, c_vp)


class DispatchAttrs(ctypes.Structure):
    _fields_ = [("flags", c_u64), ("smem_bytes", c_u64), ("threads", c_u64)]


class ExportTable(ctypes.Structure):
    _fields_ = [("count", ctypes.c_uint32), ("ptrs", c_vp), ("attrs", ctypes.POINTER(DispatchAttrs)),
                ("names", ctypes.POINTER(ctypes.c_char_p))]


class ImportTable(ctypes.Structure):
    _fields_ = [("count", ctypes.c_uint32), ("symbols", c_vp)]


class LibraryHeader(ctypes.Structure):
    _fields_ = [("version", ctypes.c_uint32)]


class ExecutableLibrary(ctypes.Structure):
    _fields_ = [("header", ctypes.POINTER(LibraryHeader)), ("imports", ImportTable),
                ("exports", ExportTable)]


class StringView(ctypes.Structure):
    """hxb_string_view_t."""
    _fields_ = [("data", ctypes.c_char_p), ("size", c_size)]

    @classmethod
    def of(cls, text: str | bytes) -> "StringView":
        b = text.encode() if isinstance(text, str) else bytes(text)
        return cls(b, len(b))


AllocatorCtl = ctypes.CFUNCTYPE(c_int, c_vp, c_int, c_vp, ctypes.POINTER(c_vp))


class Allocator(ctypes.Structure):
    """hxb_allocator_t; Allocator() is the C library's malloc / free."""
    _fields_ = [("self", c_vp), ("ctl", AllocatorCtl)]


class DeviceOptions(ctypes.Structure):
    _fields_ = [("scratch_bytes", c_u64), ("queue_wait_timeout_ns", c_u64)]


class DeviceCreateParams(ctypes.Structure):
    _fields_ = [("flags", c_u64)]


class DeviceInfo(ctypes.Structure):
    _fields_ = [("device_id", c_u64), ("path", ctypes.c_char * 32), ("name", ctypes.c_char * 96)]


class DriverInfo(ctypes.Structure):
    _fields_ = [("driver_name", StringView), ("full_name", StringView)]


DriverEnumerateFn = ctypes.CFUNCTYPE(c_int, c_vp, ctypes.POINTER(c_size),
                                     ctypes.POINTER(ctypes.POINTER(DriverInfo)))
DriverTryCreateFn = ctypes.CFUNCTYPE(c_int, c_vp, StringView, Allocator, ctypes.POINTER(c_vp))


class DriverFactory(ctypes.Structure):
    _fields_ = [("self", c_vp), ("enumerate", DriverEnumerateFn),
                ("try_create", DriverTryCreateFn)]


class CompilerOptions(ctypes.Structure):
    _fields_ = [("enable_matmul", ctypes.c_int32), ("enable_w8a16", ctypes.c_int32),
                ("enable_attention", ctypes.c_int32), ("num_sms", ctypes.c_int32)]


class TensorDesc(ctypes.Structure):
    _fields_ = [("element_type", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("dims", c_i64 * 8)]


class BufferBinding(ctypes.Structure):
    _fields_ = [("buffer", c_vp), ("offset", c_u64), ("length", c_u64)]


class BindingTable(ctypes.Structure):
    _fields_ = [("count", ctypes.c_uint32), ("bindings", ctypes.POINTER(BufferBinding))]


class DriverOptions(ctypes.Structure):
    _fields_ = [("default_device_options", DeviceOptions)]


class BufferRef(ctypes.Structure):
    """hxb_hal_buffer_ref_t: a buffer range, or (buffer None) a table slot."""
    _fields_ = [("buffer", c_vp), ("offset", c_u64), ("length", c_u64),
                ("buffer_slot", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


class DecoderW8(ctypes.Structure):
    """hxb_decoder_w8_t of include/hxb200.h."""

    _fields_ = [("hidden", c_i64), ("heads", c_i64), ("head_dim", c_i64), ("ffn", c_i64),
                ("rms_eps", c_float), ("rope_theta", c_float),
                ("attn_norm", c_vp), ("w_qkv", c_vp), ("s_qkv", c_vp),
                ("w_o", c_vp), ("s_o", c_vp), ("ffn_norm", c_vp),
                ("w_gate_up", c_vp), ("s_gate_up", c_vp),
                ("w_down", c_vp), ("s_down", c_vp)]

STATUS_NAMES = {
    0: "OK",
    1: "INVALID_ARGUMENT",
    2: "UNSUPPORTED",
    3: "CUDA_ERROR",
    4: "RESOURCE_EXHAUSTED",
    5: "DEVICE_TIMEOUT",
    6: "UNAVAILABLE",
    7: "ALREADY_EXISTS",
}

DTYPE_F16, DTYPE_F32, DTYPE_I8 = 0, 1, 2


class HxbError(RuntimeError):
    """A non-OK status from the dispatch library."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_lib: ctypes.CDLL | None = None


def load(path: Path | None = None) -> ctypes.CDLL:
    """Loads (once) and types the dispatch library."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise OSError(
            f"{p} is missing: build it with `python iree-hexagon-plugins_b200/build.py` "
            "(nvcc, sm_100a). There is no fallback implementation.")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        # struct-by-value arguments are named, the structs are defined below
        fn.argtypes = [globals()[a] if isinstance(a, str) else a for a in args]
    if path is None:
        _lib = lib
    return lib


def check(status: int) -> None:
    if status != 0:
        msg = load().hxb_last_error_message()
        raise HxbError(status, msg.decode() if msg else "")
