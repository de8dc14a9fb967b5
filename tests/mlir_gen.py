"""Writers of linalg-on-tensors MLIR for the compiler stand-in's tests.

Each function returns the text of a module in the pretty-printed form that
torch-mlir and IREE produce for the reference's inputs: a func.func over
tensors (matmul, the int8-weight linear) or an IREE coarse-fences entry over
!hal.buffer_view arguments (the decomposed scaled-dot-product attention,
whose op sequence is that of F.scaled_dot_product_attention lowered to
linalg: f16 -> f32 extension, the square root of the softmax scale applied to
Q and to K^T, batch_matmul, row max, subtract, exp, row sum, divide, the
fully-masked-row select, batch_matmul with V, truncation to f16). The shapes
are parameters, so the GPU tests can run them at the reference examples'
sizes without reading the reference checkout.
"""
from __future__ import annotations


def _t(shape, elem):
    return "tensor<" + "x".join(str(d) for d in shape) + "x" + elem + ">"


def matmul(M, N, K, *, out="f32", init=False, transpose_b=False, batch=None,
           f32_inputs_from_f16=False, name="matmul") -> str:
    """C = A . B (+ init). transpose_b: B is [N, K]. batch: a leading batch
    dimension (named batch_matmul). f32_inputs_from_f16: the torch form
    matmul(a.float(), b.float()) -- f16 arguments extended to f32 by
    elementwise generics feeding a generic contraction."""
    bdim = [batch] if batch else []
    a_shape = bdim + [M, K]
    b_shape = bdim + ([N, K] if transpose_b else [K, N])
    c_shape = bdim + [M, N]
    A, B, C = _t(a_shape, "f16"), _t(b_shape, "f16"), _t(c_shape, out)
    args = [f"%a: {A}", f"%b: {B}"] + ([f"%init: {C}"] if init else [])
    lines = ["module {", f"  func.func @{name}({', '.join(args)}) -> {C} {{"]
    if init:
        acc = "%init"
    else:
        lines += [f"    %zero = arith.constant 0.0 : {out}",
                  f"    %empty = tensor.empty() : {C}",
                  f"    %acc = linalg.fill ins(%zero : {out}) outs(%empty : {C}) -> {C}"]
        acc = "%acc"
    if not f32_inputs_from_f16:
        if batch:
            op = "linalg.batch_matmul_transpose_b" if transpose_b else "linalg.batch_matmul"
        else:
            op = "linalg.matmul_transpose_b" if transpose_b else "linalg.matmul"
        lines += [f"    %r = {op}",
                  f"        ins(%a, %b : {A}, {B})",
                  f"        outs({acc} : {C}) -> {C}"]
    else:
        rank = len(a_shape)
        dims = ", ".join(f"d{i}" for i in range(rank))
        ident = f"affine_map<({dims}) -> ({dims})>"
        par = ", ".join(['"parallel"'] * rank)
        for v, shape in (("a", a_shape), ("b", b_shape)):
            T16, T32 = _t(shape, "f16"), _t(shape, "f32")
            lines += [f"    %{v}e = tensor.empty() : {T32}",
                      f"    %{v}32 = linalg.generic {{indexing_maps = [{ident}, {ident}], "
                      f"iterator_types = [{par}]}} "
                      f"ins(%{v} : {T16}) outs(%{v}e : {T32}) {{",
                      "    ^bb0(%in: f16, %out: f32):",
                      "      %x = arith.extf %in : f16 to f32",
                      "      linalg.yield %x : f32",
                      f"    }} -> {T32}"]
        # contraction dims: [b,] m, n, k
        nb = 1 if batch else 0
        d = [f"d{i}" for i in range(nb + 3)]
        bd = d[:nb]
        m, n, k = d[nb], d[nb + 1], d[nb + 2]
        all_d = ", ".join(d)
        amap = f"affine_map<({all_d}) -> ({', '.join(bd + [m, k])})>"
        bmap = f"affine_map<({all_d}) -> ({', '.join(bd + ([n, k] if transpose_b else [k, n]))})>"
        cmap = f"affine_map<({all_d}) -> ({', '.join(bd + [m, n])})>"
        its = ", ".join(['"parallel"'] * (nb + 2) + ['"reduction"'])
        A32, B32 = _t(a_shape, "f32"), _t(b_shape, "f32")
        lines += [f"    %r = linalg.generic {{indexing_maps = [{amap}, {bmap}, {cmap}], "
                  f"iterator_types = [{its}]}} ins(%a32, %b32 : {A32}, {B32}) outs({acc} : {C}) {{",
                  f"    ^bb0(%x: f32, %y: f32, %z: {out}):",
                  f"      %p = arith.mulf %x, %y : f32",
                  f"      %s = arith.addf %z, %p : f32",
                  f"      linalg.yield %s : f32",
                  f"    }} -> {C}"]
    lines += [f"    return %r : {C}", "  }", "}"]
    return "\n".join(lines) + "\n"


def matmul_chain(M, N, K, P) -> str:
    """D = (A . B) . E with f16 results: the intermediate lives in a
    transient buffer between two dispatches."""
    A, B, E = _t([M, K], "f16"), _t([K, N], "f16"), _t([N, P], "f16")
    C, D = _t([M, N], "f16"), _t([M, P], "f16")
    return f"""module {{
  func.func @chain(%a: {A}, %b: {B}, %e: {E}) -> {D} {{
    %zero = arith.constant 0.0 : f16
    %c0 = tensor.empty() : {C}
    %c = linalg.fill ins(%zero : f16) outs(%c0 : {C}) -> {C}
    %ab = linalg.matmul ins(%a, %b : {A}, {B}) outs(%c : {C}) -> {C}
    %d0 = tensor.empty() : {D}
    %d = linalg.fill ins(%zero : f16) outs(%d0 : {D}) -> {D}
    %r = linalg.matmul ins(%ab, %e : {C}, {E}) outs(%d : {D}) -> {D}
    return %r : {D}
  }}
}}
"""


def w8a16(M, K, N, name="linear") -> str:
    """C[M, N] f16 = truncf(sum_k extf(A[m, k]) * (sitofp(W[k, n]) * extf(s[n]))),
    the int8-weight linear with a per-output-channel scale."""
    A, W, S = _t([M, K], "f16"), _t([K, N], "i8"), _t([N], "f16")
    C32, C16 = _t([M, N], "f32"), _t([M, N], "f16")
    return f"""#a_map = affine_map<(d0, d1, d2) -> (d0, d2)>
#w_map = affine_map<(d0, d1, d2) -> (d2, d1)>
#s_map = affine_map<(d0, d1, d2) -> (d1)>
#c_map = affine_map<(d0, d1, d2) -> (d0, d1)>
#id2 = affine_map<(d0, d1) -> (d0, d1)>
module {{
  func.func @{name}(%a: {A}, %w: {W}, %s: {S}) -> {C16} {{
    %zero = arith.constant 0.0 : f32
    %e = tensor.empty() : {C32}
    %acc = linalg.fill ins(%zero : f32) outs(%e : {C32}) -> {C32}
    %mm = linalg.generic {{indexing_maps = [#a_map, #w_map, #s_map, #c_map], iterator_types = ["parallel", "parallel", "reduction"]}} ins(%a, %w, %s : {A}, {W}, {S}) outs(%acc : {C32}) {{
    ^bb0(%x: f16, %q: i8, %sc: f16, %o: f32):
      %wf = arith.sitofp %q : i8 to f32
      %sf = arith.extf %sc : f16 to f32
      %ws = arith.mulf %wf, %sf : f32
      %xf = arith.extf %x : f16 to f32
      %p = arith.mulf %xf, %ws : f32
      %r = arith.addf %o, %p : f32
      linalg.yield %r : f32
    }} -> {C32}
    %e16 = tensor.empty() : {C16}
    %out = linalg.generic {{indexing_maps = [#id2, #id2], iterator_types = ["parallel", "parallel"]}} ins(%mm : {C32}) outs(%e16 : {C16}) {{
    ^bb0(%in: f32, %o2: f16):
      %t = arith.truncf %in : f32 to f16
      linalg.yield %t : f16
    }} -> {C16}
    return %out : {C16}
  }}
}}
"""


def sdpa(BH, S, D, scale_sqrt=None) -> str:
    """The decomposed, non-causal scaled-dot-product attention over
    [BH, S, D] f16 Q, K, V as an IREE coarse-fences entry (@main$async over
    buffer views and fences) plus its synchronous @main wrapper."""
    if scale_sqrt is None:
        scale_sqrt = D ** -0.25
    Q16, Q32 = _t([BH, S, D], "f16"), _t([BH, S, D], "f32")
    KT = _t([BH, D, S], "f32")
    SS = _t([BH, S, S], "f32")
    R, R1 = _t([BH, S], "f32"), _t([BH, S, 1], "f32")
    RI = _t([BH, S], "i64")
    B1, BB = _t([BH, S, 1], "i1"), _t([BH, S, S], "i1")
    par3 = '["parallel", "parallel", "parallel"]'
    red3 = '["parallel", "parallel", "reduction"]'

    def ew(res, src, src_t, out, out_t, body, in_ty, out_ty):
        return (f"    {res} = linalg.generic {{indexing_maps = [#m3, #m3], iterator_types = {par3}}} "
                f"ins({src} : {src_t}) outs({out} : {out_t}) {{\n"
                f"    ^bb0(%in: {in_ty}, %out: {out_ty}):\n{body}"
                f"    }} -> {out_t}\n")
    ext = "      %v = arith.extf %in : f16 to f32\n      linalg.yield %v : f32\n"
    scal = ("      %c = arith.truncf %cst_s : f64 to f32\n      %v = arith.mulf %in, %c : f32\n"
            "      linalg.yield %v : f32\n")
    return f"""#m3 = affine_map<(d0, d1, d2) -> (d0, d1, d2)>
#m2 = affine_map<(d0, d1, d2) -> (d0, d1)>
#m1 = affine_map<(d0, d1, d2) -> (d0, d1, 0)>
module @module {{
  util.func public @main$async(%arg0: !hal.buffer_view, %arg1: !hal.buffer_view, %arg2: !hal.buffer_view, %arg3: !hal.fence, %arg4: !hal.fence) -> !hal.buffer_view attributes {{iree.abi.model = "coarse-fences", iree.abi.stub}} {{
    %zeros = arith.constant dense<0.000000e+00> : {SS}
    %f0 = arith.constant 0.000000e+00 : f32
    %i0 = arith.constant 0 : i64
    %ninf = arith.constant 0xFF800000 : f32
    %true = arith.constant true
    %ninf64 = arith.constant 0xFFF0000000000000 : f64
    %cst_s = arith.constant {scale_sqrt!r} : f64
    %q = hal.tensor.import wait(%arg3) => %arg0 : !hal.buffer_view -> {Q16}
    %k = hal.tensor.import wait(%arg3) => %arg1 : !hal.buffer_view -> {Q16}
    %v = hal.tensor.import wait(%arg3) => %arg2 : !hal.buffer_view -> {Q16}
    %e3 = tensor.empty() : {Q32}
{ew("%q32", "%q", Q16, "%e3", Q32, ext, "f16", "f32")}{ew("%k32", "%k", Q16, "%e3", Q32, ext, "f16", "f32")}{ew("%v32", "%v", Q16, "%e3", Q32, ext, "f16", "f32")}{ew("%qs", "%q32", Q32, "%e3", Q32, scal, "f32", "f32")}    %ekt = tensor.empty() : {KT}
    %kt = linalg.transpose ins(%k32 : {Q32}) outs(%ekt : {KT}) permutation = [0, 2, 1]
{ew("%kts", "%kt", KT, "%ekt", KT, scal, "f32", "f32")}    %es = tensor.empty() : {SS}
    %zs = linalg.fill ins(%f0 : f32) outs(%es : {SS}) -> {SS}
    %s = linalg.batch_matmul ins(%qs, %kts : {Q32}, {KT}) outs(%zs : {SS}) -> {SS}
    %ei = tensor.empty() : {RI}
    %zi = linalg.fill ins(%i0 : i64) outs(%ei : {RI}) -> {RI}
    %er = tensor.empty() : {R}
    %mi = linalg.fill ins(%ninf : f32) outs(%er : {R}) -> {R}
    %mx:2 = linalg.generic {{indexing_maps = [#m3, #m2, #m2], iterator_types = {red3}}} ins(%s : {SS}) outs(%mi, %zi : {R}, {RI}) {{
    ^bb0(%in: f32, %out: f32, %idx: i64):
      %j = linalg.index 2 : index
      %ji = arith.index_cast %j : index to i64
      %m = arith.maximumf %in, %out : f32
      %gt = arith.cmpf ogt, %in, %out : f32
      %ni = arith.select %gt, %ji, %idx : i64
      linalg.yield %m, %ni : f32, i64
    }} -> ({R}, {RI})
    %mxe = tensor.expand_shape %mx#0 [[0], [1, 2]] output_shape [{BH}, {S}, 1] : {R} into {R1}
    %sub = linalg.generic {{indexing_maps = [#m3, #m1, #m3], iterator_types = {par3}}} ins(%s, %mxe : {SS}, {R1}) outs(%es : {SS}) {{
    ^bb0(%in: f32, %mm: f32, %out: f32):
      %d = arith.subf %in, %mm : f32
      linalg.yield %d : f32
    }} -> {SS}
    %ex = linalg.generic {{indexing_maps = [#m3, #m3], iterator_types = {par3}}} ins(%sub : {SS}) outs(%es : {SS}) {{
    ^bb0(%in: f32, %out: f32):
      %x = math.exp %in : f32
      linalg.yield %x : f32
    }} -> {SS}
    %e1 = tensor.empty() : {R1}
    %z1 = linalg.fill ins(%f0 : f32) outs(%e1 : {R1}) -> {R1}
    %sum = linalg.generic {{indexing_maps = [#m3, #m1], iterator_types = {red3}}} ins(%ex : {SS}) outs(%z1 : {R1}) {{
    ^bb0(%in: f32, %out: f32):
      %a = arith.addf %in, %out : f32
      linalg.yield %a : f32
    }} -> {R1}
    %p = linalg.generic {{indexing_maps = [#m3, #m1, #m3], iterator_types = {par3}}} ins(%ex, %sum : {SS}, {R1}) outs(%es : {SS}) {{
    ^bb0(%in: f32, %t: f32, %out: f32):
      %q2 = arith.divf %in, %t : f32
      linalg.yield %q2 : f32
    }} -> {SS}
    %eb = tensor.empty() : {BB}
    %isinf = linalg.generic {{indexing_maps = [#m3, #m3], iterator_types = {par3}}} ins(%s : {SS}) outs(%eb : {BB}) {{
    ^bb0(%in: f32, %out: i1):
      %w = arith.extf %in : f32 to f64
      %c2 = arith.cmpf oeq, %w, %ninf64 : f64
      linalg.yield %c2 : i1
    }} -> {BB}
    %eb1 = tensor.empty() : {B1}
    %t1 = linalg.fill ins(%true : i1) outs(%eb1 : {B1}) -> {B1}
    %all = linalg.generic {{indexing_maps = [#m3, #m1], iterator_types = {red3}}} ins(%isinf : {BB}) outs(%t1 : {B1}) {{
    ^bb0(%in: i1, %out: i1):
      %n = arith.andi %in, %out : i1
      linalg.yield %n : i1
    }} -> {B1}
    %pm = linalg.generic {{indexing_maps = [#m1, #m3, #m3, #m3], iterator_types = {par3}}} ins(%all, %zeros, %p : {B1}, {SS}, {SS}) outs(%es : {SS}) {{
    ^bb0(%c3: i1, %z: f32, %pp: f32, %out: f32):
      %sel = arith.select %c3, %z, %pp : f32
      linalg.yield %sel : f32
    }} -> {SS}
    %zo = linalg.fill ins(%f0 : f32) outs(%e3 : {Q32}) -> {Q32}
    %o32 = linalg.batch_matmul ins(%pm, %v32 : {SS}, {Q32}) outs(%zo : {Q32}) -> {Q32}
    %e16 = tensor.empty() : {Q16}
{ew("%o", "%o32", Q32, "%e16", Q16, "      %h = arith.truncf %in : f32 to f16\n      linalg.yield %h : f16\n", "f32", "f16")}    %ob = hal.tensor.barrier join(%o : {Q16}) => %arg4 : !hal.fence
    %ov = hal.tensor.export %ob : {Q16} -> !hal.buffer_view
    util.return %ov : !hal.buffer_view
  }}
  util.func public @main(%arg0: !hal.buffer_view, %arg1: !hal.buffer_view, %arg2: !hal.buffer_view) -> !hal.buffer_view attributes {{iree.abi.stub}} {{
    %0 = util.null : !hal.fence
    %c0 = arith.constant 0 : index
    %dev = hal.devices.get %c0 : !hal.device
    %fence = hal.fence.create device(%dev : !hal.device) flags("None") : !hal.fence
    %r = util.call @main$async(%arg0, %arg1, %arg2, %0, %fence) : (!hal.buffer_view, !hal.buffer_view, !hal.buffer_view, !hal.fence, !hal.fence) -> !hal.buffer_view
    util.return %r : !hal.buffer_view
  }}
}}
"""


def dispatch_matmul(M, N, K, *, out="f32", dialect="iree_tensor_ext") -> str:
    """One matmul in the dispatch form a target backend receives inside a
    hal.executable.variant: operands through hal.interface.binding.subspan
    and dispatch.tensor.load / store, no function arguments or results."""
    A, B, C = _t([M, K], "f16"), _t([K, N], "f16"), _t([M, N], out)
    dt = f"!{dialect}.dispatch.tensor"
    return f"""#pipeline_layout = #hal.pipeline.layout<bindings = [#hal.pipeline.binding<storage_buffer, "ReadOnly|Indirect">, #hal.pipeline.binding<storage_buffer, "ReadOnly|Indirect">, #hal.pipeline.binding<storage_buffer, Indirect>]>
module {{
  func.func @matmul_dispatch_0_matmul_{M}x{N}x{K}_f16xf16x{out}() {{
    %c0 = arith.constant 0 : index
    %cst = arith.constant 0.000000e+00 : {out}
    %0 = hal.interface.binding.subspan layout(#pipeline_layout) binding(0) alignment(64) offset(%c0) flags("ReadOnly|Indirect") : {dt}<readonly:{A}>
    %1 = hal.interface.binding.subspan layout(#pipeline_layout) binding(1) alignment(64) offset(%c0) flags("ReadOnly|Indirect") : {dt}<readonly:{B}>
    %2 = hal.interface.binding.subspan layout(#pipeline_layout) binding(2) alignment(64) offset(%c0) flags(Indirect) : {dt}<writeonly:{C}>
    %3 = {dialect}.dispatch.tensor.load %0, offsets = [0, 0], sizes = [{M}, {K}], strides = [1, 1] : {dt}<readonly:{A}> -> {A}
    %4 = {dialect}.dispatch.tensor.load %1, offsets = [0, 0], sizes = [{K}, {N}], strides = [1, 1] : {dt}<readonly:{B}> -> {B}
    %5 = tensor.empty() : {C}
    %6 = linalg.fill ins(%cst : {out}) outs(%5 : {C}) -> {C}
    %7 = linalg.matmul ins(%3, %4 : {A}, {B}) outs(%6 : {C}) -> {C}
    {dialect}.dispatch.tensor.store %7, %2, offsets = [0, 0], sizes = [{M}, {N}], strides = [1, 1] : {C} -> {dt}<writeonly:{C}>
    return
  }}
}}
"""
