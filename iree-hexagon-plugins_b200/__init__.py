"""B200 (sm_100a) implementation of the iree-hexagon-plugins hot path.

The package directory holds the CUDA kernels and C ABI (csrc/, built into
libhxb200.so by build.py) and the Python host mirror of the reference's
plugin/operator surface. Because the directory name is not a Python
identifier it is imported as `iree_hexagon_plugins_b200` through
`__graft_entry__.load_package()`.
"""
from . import _native
from ._native import HxbError
from . import compiler, hal, sharded
from .dispatch import (DecoderBlockW8, attention, attention_bshd, attention_gqa,
                       attention_gqa_workspace_bytes, device_status, kv_cache_write, matmul,
                       matmul_w8a16, rmsnorm, rope_, swiglu, w8a16_workspace)

__all__ = ["compiler", "hal", "sharded", "HxbError", "DecoderBlockW8", "attention", "attention_bshd",
           "attention_gqa", "attention_gqa_workspace_bytes", "device_status",
           "kv_cache_write", "matmul", "matmul_w8a16", "rmsnorm", "rope_", "swiglu",
           "w8a16_workspace", "_native"]
