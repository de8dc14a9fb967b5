"""The C ABI library loads and exports everything include/*.h declares.

CPU-only: no call here reaches a GPU. Argument validation that happens
before any device access is exercised too.
"""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
INCLUDE = REPO / "include"


def declared_functions() -> set[str]:
    names = set()
    for h in sorted(INCLUDE.glob("*.h")):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"#[^\n]*", "", text)
        # struct/enum bodies (function-pointer members) and typedef'd
        # function pointer types are not exports
        text = re.sub(r"\b(struct|enum|union)\s*\w*\s*\{[^{}]*\}", "", text, flags=re.S)
        text = re.sub(r"typedef[^;]*;", "", text, flags=re.S)
        for m in re.finditer(r"\b([A-Za-z_]\w*)\s*\(", text):
            name = m.group(1)
            if name in {"sizeof", "if", "while", "for", "return", "defined"}:
                continue
            names.add(name)
    return names


def exported_symbols(lib: Path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True,
                         text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_headers_declare_functions():
    names = declared_functions()
    assert "hxb_matmul_f16" in names and "hxb_matmul_w8a16" in names
    assert "hxb_attention_f16" in names


def test_library_exports_every_declared_function(pkg):
    lib_path = pkg._native.LIB_PATH
    exported = exported_symbols(lib_path)
    missing = sorted(declared_functions() - exported)
    assert not missing, f"declared in include/*.h but not exported: {missing}"


def test_python_binding_covers_every_declared_function(pkg):
    missing = sorted(declared_functions() - set(pkg._native.SIGNATURES))
    assert not missing, f"no ctypes signature for: {missing}"


def test_abi_version(pkg):
    assert pkg._native.load().hxb_abi_version() == 1


def test_shape_validation_needs_no_device(pkg):
    lib = pkg._native.load()
    # M = 0 is rejected before any device access
    st = lib.hxb_matmul_f16(None, 1, None, 1, 0, None, None, 1, 0, 0, 1, 1, None, 0, None)
    assert st == 1
    assert b"must be >= 1" in lib.hxb_last_error_message()
    st = lib.hxb_matmul_w8a16(None, 1, None, 1, None, None, 1, 4, 4, 0, None)
    assert st == 1


def test_workspace_query_is_host_only(pkg):
    lib = pkg._native.load()
    # aligned pointers and pitches need no workspace
    assert lib.hxb_matmul_f16_workspace_bytes(0x1000, 64, 0x2000, 64, 0, 64, 64, 64) == 0
    # K = 23 (46-byte rows) breaks the 16-byte TMA pitch rule for A
    need = lib.hxb_matmul_f16_workspace_bytes(0x1000, 23, 0x2000, 24, 0, 17, 19, 23)
    assert need >= 17 * 24 * 2


def test_no_cpu_fallback_when_library_missing(pkg, tmp_path):
    with pytest.raises(OSError, match="no fallback"):
        pkg._native.load(tmp_path / "libhxb200.so")


def test_planner_uses_the_baked_sweep_table(pkg):
    """Shapes measured by the offline tile sweep (csrc/tile_table.inc) are
    answered from the table, before the cost model."""
    import ctypes
    import re
    lib = pkg._native.load()
    table = (Path(__file__).resolve().parent.parent / "iree-hexagon-plugins_b200" / "csrc" /
             "tile_table.inc").read_text()
    rows = [tuple(int(v) for v in m.groups())
            for m in re.finditer(
                r"\{(\d+), (\d+), (\d+), (\d+), (\d+), (\d+), (\d+), (\d+)\}", table)]
    assert len(rows) >= 64
    for M, N, K, bmode, bn, gm, sk, pair in rows:
        b, g, k, p = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
        assert lib.hxb_plan_matmul_f16(M, N, K, bmode, 148, ctypes.byref(b), ctypes.byref(g),
                                       ctypes.byref(k), ctypes.byref(p)) == 0
        assert (b.value, g.value, k.value, p.value) == (bn, gm, max(sk, 1), max(pair, 1)), \
            (M, N, K)


def test_rope_rejects_unaligned_pairs_before_device_access(pkg):
    """RoPE moves f16 pairs: an odd leading dimension or a base that is not
    4-byte aligned is refused on the host, before any launch."""
    lib = pkg._native.load()
    st = lib.hxb_rope_f16(0x100000, 3 * 128 + 1, 4, 2, 128, 4, 0, 10000.0, None)
    assert st == 1 and b"even" in lib.hxb_last_error_message()
    st = lib.hxb_rope_f16(0x100002, 256, 4, 2, 128, 4, 0, 10000.0, None)
    assert st == 1 and b"4-byte" in lib.hxb_last_error_message()
