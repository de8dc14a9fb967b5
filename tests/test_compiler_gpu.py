"""End to end through the compiler half and the runtime half of the drop-in
on the GPU: MLIR text -> hxb_compile_mlir -> executable -> hxb_module_load on
a HAL device -> hxb_module_invoke with device buffers -> results compared
with the oracle. The MLIR has the op structure of the reference's inputs at
their sizes (examples/matmul/matmul.mlir: a 32x32x32 matmul with an f32
result; examples/attention_layer/attention_layer.mlir: the decomposed
attention over [4, 1024, 128]); it is written by tests/mlir_gen.py, since the
reference checkout is not present where these tests run."""
from __future__ import annotations

import numpy as np
import pytest

import mlir_gen
from _support import baseline_check

pytestmark = pytest.mark.gpu


@pytest.fixture()
def device(cuda_pkg):
    dev = cuda_pkg.hal.Device(0)
    yield dev
    dev.close()


def _run(cuda_pkg, device, text, fn, inputs, *, invocations=1):
    """Compiles, loads and invokes `fn`; returns the results of the last
    invocation (each invocation binds freshly allocated buffers)."""
    exe = cuda_pkg.compiler.compile_mlir(text)
    mod = cuda_pkg.compiler.Module(device, exe)
    args_sig, res_sig = mod.signature(fn)
    assert [tuple(x.shape) for x in inputs] == [s for _, s in args_sig]
    done = device.semaphore(0)
    outs = None
    for it in range(invocations):
        args = []
        for x in inputs:
            b = device.allocate(x.nbytes)
            b.write(np.ascontiguousarray(x))
            args.append(b)
        res = [device.allocate(int(np.prod(s)) * np.dtype(dt).itemsize) for dt, s in res_sig]
        mod.invoke(fn, args, res, wait=(done, it), signal=(done, it + 1))
        done.wait(it + 1)
        outs = [np.frombuffer(r.read(), dt).reshape(s) for r, (dt, s) in zip(res, res_sig)]
        for b in args + res:
            b.close()
    n = mod.dispatch_count(fn)
    mod.close()
    done.close()
    return outs, n


@pytest.mark.parametrize("M,N,K", [(32, 32, 32), (1024, 1024, 1024), (70, 90, 111)])
def test_matmul_module(cuda_pkg, oracle, device, M, N, K):
    rng = np.random.default_rng(M + N + K)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    [c], n = _run(cuda_pkg, device, mlir_gen.matmul(M, N, K, out="f32"), "matmul", [a, b])
    assert n == 1
    baseline_check(oracle.matmul_f32(a, b), c, f"compiled matmul {M}x{N}x{K}")


def test_batched_rhs_transposed_torch_form(cuda_pkg, oracle, device):
    rng = np.random.default_rng(3)
    B, M, N, K = 3, 96, 80, 64
    a = rng.uniform(-1, 1, (B, M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (B, N, K)).astype(np.float16)
    text = mlir_gen.matmul(M, N, K, batch=B, transpose_b=True, f32_inputs_from_f16=True)
    [c], n = _run(cuda_pkg, device, text, "matmul", [a, b])
    assert n == B
    for i in range(B):
        baseline_check(oracle.matmul_f32(a[i], b[i], transpose_b=True), c[i], f"batch {i}")


def test_chain_through_a_transient_twice(cuda_pkg, oracle, device):
    """Two dispatches with a transient between them; invoked twice with
    different buffers, so the second invocation re-captures the graph with
    the new binding table."""
    rng = np.random.default_rng(4)
    M, N, K, P = 256, 128, 192, 64
    a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    e = rng.uniform(-0.1, 0.1, (N, P)).astype(np.float16)
    [d], n = _run(cuda_pkg, device, mlir_gen.matmul_chain(M, N, K, P), "chain", [a, b, e],
                  invocations=2)
    assert n == 2
    ab = oracle.matmul_f16(a, b)
    baseline_check(oracle.matmul_f32(ab, e), d.astype(np.float32), "compiled chain")


def test_w8a16_module(cuda_pkg, oracle, device):
    rng = np.random.default_rng(5)
    M, K, N = 300, 512, 1104
    a = rng.standard_normal((M, K)).astype(np.float16)
    w = rng.integers(-127, 128, (K, N), dtype=np.int8)
    s = rng.uniform(0.001, 0.02, N).astype(np.float16)
    [c], n = _run(cuda_pkg, device, mlir_gen.w8a16(M, K, N), "linear", [a, w, s])
    assert n == 1 and c.dtype == np.float16
    baseline_check(oracle.matmul_w8a16_f32(a, w, s), c.astype(np.float32), "compiled w8a16")


def test_attention_layer_module(cuda_pkg, oracle, device):
    """The attention layer at the reference example's size, entered through
    `main` (the synchronous wrapper's name resolves to main$async)."""
    rng = np.random.default_rng(6)
    BH, S, D = 4, 1024, 128
    q, k, v = (rng.standard_normal((BH, S, D)).astype(np.float16) for _ in range(3))
    [o], n = _run(cuda_pkg, device, mlir_gen.sdpa(BH, S, D), "main", [q, k, v])
    assert n == 1
    baseline_check(oracle.attention_f32(q, k, v), o.astype(np.float32), "compiled attention")
