"""The compiler half of the drop-in on the host (no GPU): the B200 target's
stand-in compiles linalg-on-tensors MLIR into an executable of dispatches,
following the reference's HMX eligibility rules
(plugins/compiler/hexagon/CodeGen/Strategy/Planning/Strategies/
ContractionStrategy.cpp:26-213, CodeGen/Transforms/
HexagonSpecializeHmxContractions.cpp:29-60), bakes the tile plan of every
matmul dispatch, and serialises the executable as a hal.executable.binary
(Target/HexagonExecutableSerialization.cpp:622-635). When the reference
checkout is present, its own example inputs (examples/matmul/matmul.mlir,
examples/attention_layer/attention_layer.mlir) are compiled too."""
from __future__ import annotations

import ctypes
import os
import re
import struct
from pathlib import Path

import pytest

import mlir_gen

REF = Path(os.environ.get("HXB_REFERENCE_ROOT", "/root/reference"))


def _compile(pkg, text, **kw):
    return pkg.compiler.compile_mlir(text, **kw)


def _dispatches(exe):
    """(ordinal, constants, bindings) of every dispatch of every function,
    decoded from the executable's documented layout."""
    b = exe.data
    assert b[:4] == b"HXBX"
    i = 4
    (ver,) = struct.unpack_from("<I", b, i)
    i += 4
    (n,) = struct.unpack_from("<I", b, i)
    i += 4
    fmt = b[i:i + n].decode()
    i += n
    assert ver == 1 and fmt == "cuda-sm100a-hxb-v1"
    (nf,) = struct.unpack_from("<I", b, i)
    i += 4
    funcs = {}
    for _ in range(nf):
        (n,) = struct.unpack_from("<I", b, i)
        i += 4
        name = b[i:i + n].decode()
        i += n
        descs = []
        for _ in range(2):
            (nd,) = struct.unpack_from("<I", b, i)
            i += 4
            lst = []
            for _ in range(nd):
                e, r = struct.unpack_from("<II", b, i)
                i += 8
                dims = struct.unpack_from(f"<{r}Q", b, i)
                i += 8 * r
                lst.append((e, dims))
            descs.append(lst)
        (nt,) = struct.unpack_from("<I", b, i)
        i += 4
        trans = struct.unpack_from(f"<{nt}Q", b, i)
        i += 8 * nt
        (nd,) = struct.unpack_from("<I", b, i)
        i += 4
        ds = []
        for _ in range(nd):
            ordinal, nc = struct.unpack_from("<II", b, i)
            i += 8
            consts = struct.unpack_from(f"<{nc}I", b, i)
            i += 4 * nc
            (nb,) = struct.unpack_from("<I", b, i)
            i += 4
            binds = []
            for _ in range(nb):
                binds.append(struct.unpack_from("<IIQQ", b, i))
                i += 24
            ds.append((ordinal, consts, binds))
        funcs[name] = {"args": descs[0], "results": descs[1], "transients": trans,
                       "dispatches": ds}
    assert i == len(b)
    return funcs


def test_matmul_f32_out_with_baked_tile_plan(pkg):
    lib = pkg._native.load()
    exe = _compile(pkg, mlir_gen.matmul(1024, 1024, 1024, out="f32"))
    f = _dispatches(exe)["matmul"]
    assert f["args"] == [(0, (1024, 1024)), (0, (1024, 1024))]
    assert f["results"] == [(1, (1024, 1024))]
    [(ordinal, c, binds)] = f["dispatches"]
    assert ordinal == 0 and c[:4] == (1024, 1024, 1024, 2)
    bn, gm, sk, pair = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    assert lib.hxb_plan_matmul_f16(1024, 1024, 1024, 0, 148, ctypes.byref(bn),
                                   ctypes.byref(gm), ctypes.byref(sk), ctypes.byref(pair)) == 0
    # the planner's choice, baked in
    assert c[4:] == (bn.value, gm.value, sk.value, pair.value)
    # A = argument 0, B = argument 1, C = result 0; no init binding (zero fill)
    assert [(k, idx) for k, idx, _, _ in binds] == [(0, 0), (0, 1), (1, 0)]
    assert "accept" in exe.log and "block_n" in exe.log


def test_matmul_init_is_a_binding(pkg):
    f = _dispatches(_compile(pkg, mlir_gen.matmul(64, 48, 40, init=True)))["matmul"]
    [(_, c, binds)] = f["dispatches"]
    assert len(binds) == 4 and binds[3][:2] == (0, 2)  # C_init = argument 2


def test_batch_matmul_tiles_batch_to_one(pkg):
    """selectHmxStrategy tiles batch to 1: one dispatch per batch, each
    binding its slice of the operands."""
    f = _dispatches(_compile(pkg, mlir_gen.matmul(128, 96, 64, batch=4, transpose_b=True)))["matmul"]
    assert len(f["dispatches"]) == 4
    for b, (_, c, binds) in enumerate(f["dispatches"]):
        assert c[3] & 1  # rhs transposed
        assert binds[0][2] == b * 128 * 64 * 2 and binds[1][2] == b * 96 * 64 * 2
        assert binds[2][2] == b * 128 * 96 * 4


def test_generic_contraction_from_f16_is_specialised(pkg):
    """torch's matmul(a.float(), b.float()): the f16 -> f32 extensions fold
    into the contraction, which is taken like the named matmul it
    specialises to (HexagonSpecializeHmxContractions.cpp:29-60)."""
    f = _dispatches(_compile(pkg, mlir_gen.matmul(64, 80, 96, f32_inputs_from_f16=True)))
    [(ordinal, c, _)] = f["matmul"]["dispatches"]
    assert ordinal == 0 and c[:3] == (64, 80, 96)
    f = _dispatches(_compile(pkg, mlir_gen.matmul(32, 16, 48, batch=3, transpose_b=True,
                                                  f32_inputs_from_f16=True)))
    assert len(f["matmul"]["dispatches"]) == 3


def test_chained_matmuls_use_a_transient(pkg):
    f = _dispatches(_compile(pkg, mlir_gen.matmul_chain(128, 64, 96, 32)))["chain"]
    assert f["transients"] == (128 * 64 * 2,)
    (o1, _, b1), (o2, _, b2) = f["dispatches"]
    assert b1[2][:2] == (2, 0) and b2[0][:2] == (2, 0)  # written, then read


def test_w8a16_linear(pkg):
    exe = _compile(pkg, mlir_gen.w8a16(300, 512, 1104))
    f = _dispatches(exe)["linear"]
    [(ordinal, c, binds)] = f["dispatches"]
    assert ordinal == 1 and c == (300, 1104, 512)
    assert [b[:2] for b in binds] == [(0, 0), (0, 1), (0, 2), (1, 0)]
    assert f["results"] == [(0, (300, 1104))]  # f16: the truncf is folded
    assert "truncf folded" in exe.log


def test_sdpa_chain_is_one_attention_dispatch(pkg):
    exe = _compile(pkg, mlir_gen.sdpa(4, 256, 128))
    funcs = _dispatches(exe)
    assert list(funcs) == ["main$async"]  # @main is a wrapper
    [(ordinal, c, binds)] = funcs["main$async"]["dispatches"]
    assert ordinal == 2 and c[:5] == (4, 256, 256, 128, 0)
    scale = struct.unpack("<f", struct.pack("<I", c[5]))[0]
    assert scale == pytest.approx(128 ** -0.5, rel=1e-6)
    assert "skip @main" in exe.log and "attention_f16 dispatch" in exe.log


def test_rejections_follow_the_hmx_rules(pkg):
    # f32 inputs are not HMX element types (hasHmxElementTypes)
    text = mlir_gen.matmul(32, 32, 32).replace("xf16>", "xf32>")
    with pytest.raises(pkg.HxbError, match="hasHmxElementTypes"):
        _compile(pkg, text)
    # an elementwise op the target forms no dispatch for: error with its line
    text = mlir_gen.w8a16(16, 64, 32).replace("arith.truncf %in : f32 to f16",
                                              "math.tanh %in : f32")
    with pytest.raises(pkg.HxbError, match=r"line \d+: linalg\.(generic|matmul)"):
        _compile(pkg, text)
    # matmul dispatches switched off (the enable-hmx-matmul gate)
    with pytest.raises(pkg.HxbError):
        _compile(pkg, mlir_gen.matmul(32, 32, 32), matmul=False)
    with pytest.raises(pkg.HxbError, match="line 1"):
        _compile(pkg, "module { func.func @f(%a: tensor<4xf16>) -> tensor<4xf16> { return %a")


def test_executable_binary_mlir(pkg):
    exe = _compile(pkg, mlir_gen.matmul(32, 32, 32))
    text = exe.binary_mlir("matmul_dispatch_0")
    m = re.match(r'hal\.executable\.binary @matmul_dispatch_0 attributes \{data = dense<\[(.*)\]> : '
                 r'vector<(\d+)xi8>, format = "cuda-sm100a-hxb-v1", mime_type = '
                 r'"application/x-hxb200-dispatch-table"\}', text)
    assert m and int(m.group(2)) == len(exe.data)
    data = bytes(int(x) & 0xFF for x in m.group(1).split(", "))
    assert data == exe.data


@pytest.mark.skipif(not (REF / "examples").is_dir(), reason="reference checkout not present")
def test_reference_examples_compile():
    """The reference's own example inputs, read from its checkout."""
    import __graft_entry__ as ge
    pkg = ge.load_package()
    exe = pkg.compiler.compile_mlir((REF / "examples/matmul/matmul.mlir").read_text())
    f = _dispatches(exe)["matmul"]
    assert f["dispatches"][0][1][:4] == (32, 32, 32, 2)  # f32 result
    exe = pkg.compiler.compile_mlir((REF / "examples/attention_layer/attention_layer.mlir")
                                    .read_text())
    funcs = _dispatches(exe)
    [(ordinal, c, _)] = funcs["main$async"]["dispatches"]
    assert ordinal == 2 and c[:5] == (4, 1024, 1024, 128, 0)
    scale = struct.unpack("<f", struct.pack("<I", c[5]))[0]
    assert scale == pytest.approx(128 ** -0.5, rel=1e-6)


@pytest.mark.parametrize("dialect", ["iree_tensor_ext", "flow"])
def test_dispatch_form_of_a_target_backend(pkg, dialect):
    """The form serializeExecutable receives (a dispatch function over
    interface bindings) compiles to the same matmul dispatch: read-only
    bindings are the arguments, the written one the result."""
    exe = _compile(pkg, mlir_gen.dispatch_matmul(128, 64, 256, dialect=dialect))
    [(name, f)] = _dispatches(exe).items()
    assert name == "matmul_dispatch_0_matmul_128x64x256_f16xf16xf32"
    assert f["args"] == [(0, (128, 256)), (0, (256, 64))] and f["results"] == [(1, (128, 64))]
    [(ordinal, c, binds)] = f["dispatches"]
    assert ordinal == 0 and c[:4] == (128, 64, 256, 2)
    assert [b[:2] for b in binds] == [(0, 0), (0, 1), (1, 0)]
    assert "binding 2 -> result 0" in exe.log


def test_iree_plugin_sources_call_the_declared_abi():
    """The IREE-side plugin sources (built only inside an IREE checkout) call
    only functions and use only macros this library's headers declare."""
    from test_abi import declared_functions
    root = Path(__file__).resolve().parent.parent / "iree-hexagon-plugins_b200" / "plugins"
    headers = "".join(p.read_text() for p in (Path(__file__).resolve().parent.parent /
                                              "include").glob("*.h"))
    declared = declared_functions()
    seen = set()
    for src in list(root.rglob("*.cpp")) + list(root.rglob("*.c")):
        text = src.read_text()
        for name in re.findall(r"\b(hxb_\w+)\s*\(", text):
            seen.add(name)
            assert name in declared, f"{src.name} calls undeclared {name}"
        for macro in re.findall(r"\b(HXB_[A-Z0-9_]+)\b", text):
            assert macro in headers, f"{src.name} uses undeclared {macro}"
    assert {"hxb_compile_mlir", "hxb_hal_driver_create"} <= seen
