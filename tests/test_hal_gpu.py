"""The HAL-shaped runtime on the GPU: a command buffer of the executable
library's dispatches, recorded once and replayed, ordered by timeline
semaphores, gives the same bits as the direct C-ABI calls of the same
kernels (and the oracle's values)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _support import baseline_check

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture()
def device(cuda_pkg):
    drv = cuda_pkg.hal.Driver()
    assert drv.device_count() >= 1
    dev = drv.create_device(0)
    yield dev
    dev.close()
    drv.close()


def _upload(dev, arr: np.ndarray):
    b = dev.allocate(arr.nbytes)
    b.write(np.ascontiguousarray(arr))
    return b


def test_command_buffer_matches_direct_calls(cuda_pkg, oracle, device):
    hal = cuda_pkg.hal
    rng = np.random.default_rng(11)
    # f16 matmul with a DPS init (f32 out), 320 x 256 x 192
    M, N, K = 320, 256, 192
    a = (rng.random((M, K)) * 2 - 1).astype(np.float16)
    b = (rng.random((K, N)) * 2 - 1).astype(np.float16)
    init = rng.standard_normal((M, N)).astype(np.float32)
    # int8-weight matmul at a decoder shape (stream-K through the device scratch)
    M8, K8, N8 = 512, 4096, 4096
    x8 = rng.standard_normal((M8, K8)).astype(np.float16)
    w8 = rng.integers(-127, 128, (K8, N8), dtype=np.int8)
    s8 = rng.uniform(0.001, 0.02, N8).astype(np.float16)
    # attention [2 heads, 256 queries, 384 keys, 128], causal
    BH, Sq, Skv = 2, 256, 384
    q = rng.standard_normal((BH, Sq, 128)).astype(np.float16)
    k = rng.standard_normal((BH, Skv, 128)).astype(np.float16)
    v = rng.standard_normal((BH, Skv, 128)).astype(np.float16)

    bufs = {n: _upload(device, x) for n, x in
            [("a", a), ("b", b), ("init", init), ("x8", x8), ("w8", w8), ("s8", s8),
             ("q", q), ("k", k), ("v", v)]}
    c = device.allocate(M * N * 4)
    c8 = device.allocate(M8 * N8 * 2)
    o = device.allocate(BH * Sq * 128 * 2)

    cb = device.command_buffer()
    cb.begin()
    cb.dispatch("matmul_f16", [M, N, K, 2], [bufs["a"], bufs["b"], c, bufs["init"]])
    cb.dispatch("matmul_w8a16", [M8, N8, K8], [bufs["x8"], bufs["w8"], bufs["s8"], c8])
    cb.dispatch("attention_f16", [BH, Sq, Skv, 128, 1, 0], [bufs["q"], bufs["k"], bufs["v"], o])
    cb.end()

    done = device.semaphore(0)
    device.execute(cb, signal=(done, 1))
    done.wait(1)
    got_c = np.frombuffer(c.read(), np.float32).reshape(M, N)
    got_c8 = np.frombuffer(c8.read(), np.float16).reshape(M8, N8)
    got_o = np.frombuffer(o.read(), np.float16).reshape(BH, Sq, 128)

    # the same kernels through the direct calls give the same bits
    t = lambda x: torch.from_numpy(x).to(DEV)
    want_c = cuda_pkg.matmul(t(a), t(b), out_dtype=torch.float32, init=t(init))
    want_c8 = cuda_pkg.matmul_w8a16(t(x8), t(w8), t(s8), workspace=cuda_pkg.w8a16_workspace(DEV))
    want_o = cuda_pkg.attention(t(q), t(k), t(v), causal=True)
    torch.cuda.synchronize()
    assert np.array_equal(got_c, want_c.cpu().numpy())
    assert np.array_equal(got_c8, want_c8.cpu().numpy())
    assert np.array_equal(got_o, want_o.cpu().numpy())
    # and the oracle's values
    baseline_check(oracle.matmul_f32(a, b, init=init), got_c, "hal matmul_f16")
    rows = np.array([0, 1, 255, 256, 511])
    baseline_check(oracle.matmul_w8a16_f32(x8[rows], w8, s8), got_c8[rows].astype(np.float32),
                   "hal matmul_w8a16")

    # replay: the captured graph runs again, ordered by the semaphore
    c8.write(np.zeros(M8 * N8, np.float16))
    device.execute(cb, wait=(done, 1), signal=(done, 2))
    done.wait(2)
    assert np.array_equal(np.frombuffer(c8.read(), np.float16).reshape(M8, N8), got_c8)
    assert cuda_pkg.device_status() == 0
    cb.close()
    done.close()
    for buf in list(bufs.values()) + [c, c8, o]:
        buf.close()


def test_queue_waits_for_host_signal(cuda_pkg, device):
    """A submission whose wait value the host has not signalled yet does not
    run until the host signals it."""
    rng = np.random.default_rng(12)
    M = N = K = 256
    a = (rng.random((M, K)) * 2 - 1).astype(np.float16)
    b = (rng.random((K, N)) * 2 - 1).astype(np.float16)
    ab, bb = _upload(device, a), _upload(device, b)
    c = device.allocate(M * N * 2)
    c.write(np.zeros(M * N, np.float16))
    cb = device.command_buffer()
    cb.begin()
    cb.dispatch("matmul_f16", [M, N, K, 0], [ab, bb, c])
    cb.end()
    go, done = device.semaphore(0), device.semaphore(0)
    device.execute(cb, wait=(go, 5), signal=(done, 1))
    with pytest.raises(cuda_pkg.HxbError, match="not reached"):
        done.wait(1, timeout_s=0.2)
    assert done.value == 0
    go.signal(5)
    done.wait(1, timeout_s=10)
    want = cuda_pkg.matmul(torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV))
    torch.cuda.synchronize()
    assert np.array_equal(np.frombuffer(c.read(), np.float16).reshape(M, N),
                          want.cpu().numpy())
    # a host signal below the current value is refused
    with pytest.raises(cuda_pkg.HxbError, match="below"):
        go.signal(4)
    for o in (cb, go, done, ab, bb, c):
        o.close()


def test_decoder_block_dispatch(cuda_pkg, device):
    hal = cuda_pkg.hal
    H, NH, F, S = 1024, 8, 2816, 64
    rng = np.random.default_rng(13)
    w = {
        "attn_norm": np.ones(H, np.float16), "ffn_norm": np.ones(H, np.float16),
        "w_qkv": rng.integers(-127, 128, (H, 3 * H), dtype=np.int8),
        "s_qkv": rng.uniform(1.5e-4, 4e-4, 3 * H).astype(np.float16),
        "w_o": rng.integers(-127, 128, (H, H), dtype=np.int8),
        "s_o": rng.uniform(1.5e-4, 4e-4, H).astype(np.float16),
        "w_gate_up": rng.integers(-127, 128, (H, 2 * F), dtype=np.int8),
        "s_gate_up": rng.uniform(1.5e-4, 4e-4, 2 * F).astype(np.float16),
        "w_down": rng.integers(-127, 128, (F, H), dtype=np.int8),
        "s_down": rng.uniform(1.5e-4, 4e-4, H).astype(np.float16),
    }
    x = rng.standard_normal((S, H)).astype(np.float16)
    t = {n: torch.from_numpy(v).to(DEV) for n, v in w.items()}
    blk = cuda_pkg.DecoderBlockW8(heads=NH, **t)
    want = blk(torch.from_numpy(x).to(DEV))
    torch.cuda.synchronize()
    ws_bytes = blk.workspace_bytes(1, S)
    order = ["attn_norm", "w_qkv", "s_qkv", "w_o", "s_o", "ffn_norm", "w_gate_up", "s_gate_up",
             "w_down", "s_down"]
    xb = _upload(device, x)
    out = device.allocate(S * H * 2)
    wb = [_upload(device, w[n]) for n in order]
    ws = device.allocate(ws_bytes)
    cb = device.command_buffer()
    cb.begin()
    cb.dispatch("decoder_block_w8a16",
                [1, S, 0, H, NH, 128, F, hal.f32_bits(1e-5), hal.f32_bits(1e4)],
                [xb, out] + wb + [ws])
    cb.end()
    done = device.semaphore(0)
    device.execute(cb, signal=(done, 1))
    done.wait(1)
    got = np.frombuffer(out.read(), np.float16).reshape(S, H)
    assert np.array_equal(got, want.cpu().numpy())
    for o in [cb, done, xb, out, ws] + wb:
        o.close()


def test_end_reports_bad_dispatch(cuda_pkg, device):
    a = device.allocate(64 * 64 * 2)
    cb = device.command_buffer()
    cb.begin()
    # C binding too short for 64 x 64 f16
    cb.dispatch("matmul_f16", [64, 64, 64, 0], [a, a, a.ref(0, 1024)])
    with pytest.raises(cuda_pkg.HxbError, match="needs 8192"):
        cb.end()
    # the command buffer can be recorded again after the failure
    cb.begin()
    cb.dispatch("matmul_f16", [64, 64, 64, 0], [a, a, a])
    cb.end()
    cb.close()
    a.close()


def test_gqa_attention_dispatch(cuda_pkg, device):
    """The sliced-cache GQA export gives the direct call's bits."""
    rng = np.random.default_rng(14)
    B, Hq, Hkv, q_len, kv_len, rows, D = 1, 9, 3, 64, 64, 128, 64
    q = rng.standard_normal((B, Hq, q_len, D)).astype(np.float16)
    k = rng.standard_normal((B, Hkv, rows, D)).astype(np.float16)
    v = rng.standard_normal((B, Hkv, rows, D)).astype(np.float16)
    qb, kb, vb = _upload(device, q), _upload(device, k), _upload(device, v)
    o = device.allocate(q.nbytes)
    cb = device.command_buffer()
    cb.begin()
    cb.dispatch("attention_gqa_f16", [B, Hq, Hkv, q_len, 0, kv_len, rows, D, 0, 1, 0],
                [qb, kb, vb, o])
    cb.end()
    done = device.semaphore(0)
    device.execute(cb, signal=(done, 1))
    done.wait(1)
    got = np.frombuffer(o.read(), np.float16).reshape(B, q_len, Hq, D)
    t = lambda x: torch.from_numpy(x).to(DEV)
    want = cuda_pkg.attention_gqa(t(q), t(k), t(v), kv_len=kv_len, out_layout="bshd")
    torch.cuda.synchronize()
    assert np.array_equal(got, want.cpu().numpy())
    for x in (cb, done, qb, kb, vb, o):
        x.close()


def test_repitched_matmul_in_command_buffer(cuda_pkg, oracle, device):
    """K and N whose rows are not 16-byte multiples make the matmul export
    re-pitch through the library's built-in scratch while end() captures the
    command buffer; the device resolved that scratch when it was created.
    Recorded once, executed twice, checked against the oracle each time."""
    rng = np.random.default_rng(15)
    M, N, K = 70, 90, 111
    a = (rng.random((M, K)) * 2 - 1).astype(np.float16)
    b = (rng.random((K, N)) * 2 - 1).astype(np.float16)
    ab, bb = _upload(device, a), _upload(device, b)
    c = device.allocate(M * N * 4)
    cb = device.command_buffer()
    cb.begin()
    cb.dispatch("matmul_f16", [M, N, K, 2], [ab, bb, c])
    cb.end()
    done = device.semaphore(0)
    want = oracle.matmul_f32(a, b)
    for i in (1, 2):
        c.write(np.full(M * N, np.nan, np.float32))
        device.execute(cb, wait=(done, i - 1), signal=(done, i))
        done.wait(i)
        got = np.frombuffer(c.read(), np.float32).reshape(M, N)
        baseline_check(want, got, f"hal re-pitched matmul, execution {i}")
    assert cuda_pkg.device_status() == 0
    for x in (cb, done, ab, bb, c):
        x.close()


def test_binding_table_slots(cuda_pkg, oracle, device):
    """A command buffer recorded against binding-table slots runs with the
    buffers of each submission's table (device.c:977-1012 resolves tables at
    submission too): two tables, then the first again."""
    rng = np.random.default_rng(16)
    M, N, K = 256, 192, 320
    sets = []
    for _ in range(2):
        a = (rng.random((M, K)) * 2 - 1).astype(np.float16)
        b = (rng.random((K, N)) * 2 - 1).astype(np.float16)
        sets.append((a, b, _upload(device, a), _upload(device, b), device.allocate(M * N * 2)))
    hal = cuda_pkg.hal
    cb = device.command_buffer(binding_capacity=3)
    cb.begin()
    cb.dispatch("matmul_f16", [M, N, K, 0],
                [hal.slot(0, 0, M * K * 2), hal.slot(1, 0, K * N * 2), hal.slot(2, 0, M * N * 2)])
    cb.end()
    done = device.semaphore(0)
    step = 0
    for which in (0, 1, 0):
        a, b, ab, bb, cbuf = sets[which]
        cbuf.write(np.zeros(M * N, np.float16))
        step += 1
        device.execute(cb, wait=(done, step - 1), signal=(done, step), bindings=[ab, bb, cbuf])
        done.wait(step)
        got = np.frombuffer(cbuf.read(), np.float16).reshape(M, N)
        baseline_check(oracle.matmul_f32(a, b), got.astype(np.float32), f"table set {which}")
    # a submission without the table it needs is refused on the host
    with pytest.raises(cuda_pkg.HxbError, match="table"):
        device.execute(cb)
    for x in [cb, done] + [o for s in sets for o in s[2:]]:
        x.close()


def test_queue_wait_bound_runs_out(cuda_pkg, oracle):
    """A submission waits on a semaphore nobody signals. The device-side wait
    gives up after the device's bound (50 ms here), sets the timeout bit of
    the device status word and marks the device lost; the submission's signal
    is never written, so a host waiter times out too; later submissions are
    refused; release returns. A new device then computes correctly."""
    hal = cuda_pkg.hal
    cuda_pkg.device_status(clear=True)
    dev = hal.Device(0, queue_wait_timeout_ns=50_000_000)
    M = N = K = 128
    rng = np.random.default_rng(17)
    a = (rng.random((M, K)) * 2 - 1).astype(np.float16)
    b = (rng.random((K, N)) * 2 - 1).astype(np.float16)
    ab, bb, c = _upload(dev, a), _upload(dev, b), dev.allocate(M * N * 2)
    cb = dev.command_buffer()
    cb.begin()
    cb.dispatch("matmul_f16", [M, N, K, 0], [ab, bb, c])
    cb.end()
    never, done = dev.semaphore(0), dev.semaphore(0)
    dev.execute(cb, wait=(never, 1), signal=(done, 1))
    with pytest.raises(cuda_pkg.HxbError, match="DEVICE_TIMEOUT"):
        done.wait(1, timeout_s=2.0)
    torch.cuda.synchronize()
    assert dev.lost
    assert cuda_pkg.device_status(clear=False) & 1
    with pytest.raises(cuda_pkg.HxbError, match="device lost"):
        dev.execute(cb)
    for x in (cb, never, done, ab, bb, c):
        x.close()
    dev.close()
    assert cuda_pkg.device_status(clear=True) & 1
    assert cuda_pkg.device_status(clear=False) == 0
    # a fresh device on the same GPU works
    dev2 = hal.Driver().create_device_by_id(0)
    ab, bb, c = _upload(dev2, a), _upload(dev2, b), dev2.allocate(M * N * 2)
    cb = dev2.command_buffer()
    cb.begin()
    cb.dispatch("matmul_f16", [M, N, K, 0], [ab, bb, c])
    cb.end()
    done = dev2.semaphore(0)
    dev2.execute(cb, signal=(done, 1))
    done.wait(1)
    got = np.frombuffer(c.read(), np.float16).reshape(M, N)
    baseline_check(oracle.matmul_f32(a, b), got.astype(np.float32), "matmul after a lost device")
    for x in (cb, done, ab, bb, c):
        x.close()
    dev2.close()
