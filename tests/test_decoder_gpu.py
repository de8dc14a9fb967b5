"""Parity of the decoder-block dispatches (Llama-style
block with int8-weight linears) with the oracle's restatement of the Hugging
Face Llama modules the reference's decoder models run
(integration_tests/models/meta-llama/Llama-3.2-1B-Instruct/model.py).

Stage tests feed each kernel the same f16 input as the oracle and allow one
f16 ulp (two where two roundings stack). The end-to-end tests run the whole
block and compare every output with the oracle's block, whose intermediates
are rounded to f16 at the same points."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _support import baseline_check, f16_ulp


def _block_check(ref: np.ndarray, got: np.ndarray, what: str) -> None:
    """The BASELINE bar on a whole decoder-block output against the oracle's
    restatement of the Hugging Face modules: |d| <= 1e-2 + one f16 ulp of the
    reference value and relative L2 <= 1e-3 (baseline_check), with the
    measured figures printed for the record."""
    r = ref.astype(np.float64)
    d = np.abs(got.astype(np.float64) - r)
    rel = np.linalg.norm(d) / np.linalg.norm(r)
    worst = float((d / (1e-2 + f16_ulp(ref.astype(np.float32)))).max())
    print(f"{what}: rel-L2 {rel:.3g}, max|d| {d.max():.4g}, "
          f"max |d| / (1e-2 + ulp) {worst:.3g}, max |ref| {float(np.abs(r).max()):.4g}")
    baseline_check(ref.astype(np.float32), got.astype(np.float32), what)

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def _within_ulps(ref, got, ulps, what):
    r = ref.astype(np.float64)
    g = got.astype(np.float64)
    bound = ulps * f16_ulp(ref.astype(np.float32)) + 1e-6
    bad = np.abs(g - r) > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements beyond {ulps} ulp; worst "
                           f"{np.abs(g - r).max():.4g}")


@pytest.mark.parametrize("rows,cols", [
    (1100, 4096),  # one warp per row
    (300, 4096),   # a prefill: one block per row
    (1, 4096),     # decode step
    (7, 1000),     # a few rows, ragged vector count per thread
    (32, 8192),    # the largest rows the block-per-row kernel holds
])
def test_rmsnorm_vs_oracle(cuda_pkg, oracle, rows, cols):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((rows, cols)) * 3).astype(np.float16)
    g = rng.uniform(0.5, 1.5, cols).astype(np.float16)
    got = cuda_pkg.rmsnorm(_t(x), _t(g), 1e-5).cpu().numpy()
    # two f16 roundings (normalised row, then times the weight): a 1-ulp flip of
    # the first, scaled by a weight up to 1.5, can reach 2 ulp of the result
    _within_ulps(oracle.rmsnorm_f16(x, g, 1e-5), got, 2, "rmsnorm")
    ones = np.ones(cols, np.float16)
    got1 = cuda_pkg.rmsnorm(_t(x), _t(ones), 1e-5).cpu().numpy()
    _within_ulps(oracle.rmsnorm_f16(x, ones, 1e-5), got1, 1, "rmsnorm (unit weight)")


def test_rope_vs_oracle(cuda_pkg, oracle):
    rng = np.random.default_rng(2)
    S, H = 200, 4
    x = rng.standard_normal((2 * S, 3 * H * 128)).astype(np.float16)  # batch 2, fused qkv rows
    xd = _t(x)
    cuda_pkg.rope_(xd, heads=2 * H, seq=S, pos0=7)
    got = xd.cpu().numpy()
    want = oracle.rope_f16(x, 2 * H, S, 7)
    # The kernel forms the angle pos * theta^(-2i/128) in f32, as the Hugging
    # Face rotary module does (the oracle uses f64): at positions ~200 that is
    # up to ~1e-4 rad off, i.e. |x| * 1e-4 on the rotated value, on top of the
    # final f16 rounding.
    pair_mag = np.zeros(x.shape, np.float64)
    for h in range(2 * H):
        lo = np.abs(x[:, h * 128:h * 128 + 64].astype(np.float64))
        hi = np.abs(x[:, h * 128 + 64:h * 128 + 128].astype(np.float64))
        m = np.maximum(lo, hi)
        pair_mag[:, h * 128:h * 128 + 64] = m
        pair_mag[:, h * 128 + 64:h * 128 + 128] = m
    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
    bound = f16_ulp(want.astype(np.float32)) + 2e-4 * pair_mag
    assert (d <= bound).all(), f"rope: {int((d > bound).sum())} elements out of bound"
    assert np.array_equal(got[:, 2 * H * 128:], x[:, 2 * H * 128:]), "v block must be untouched"


def test_swiglu_vs_oracle(cuda_pkg, oracle):
    rng = np.random.default_rng(3)
    gu = (rng.standard_normal((64, 2 * 1104)) * 4).astype(np.float16)
    got = cuda_pkg.swiglu(_t(gu)).cpu().numpy()
    _within_ulps(oracle.swiglu_f16(gu), got, 1, "swiglu")


@pytest.mark.parametrize("M", [1, 16, 300])
def test_w8a16_residual_vs_oracle(cuda_pkg, oracle, M):
    rng = np.random.default_rng(M)
    K, N = 1024, 1104
    a = rng.standard_normal((M, K)).astype(np.float16)
    w = rng.integers(-127, 128, (K, N), dtype=np.int8)
    s = rng.uniform(0.001, 0.02, N).astype(np.float16)
    r = (rng.standard_normal((M, N)) * 8).astype(np.float16)
    got = cuda_pkg.matmul_w8a16(_t(a), _t(w), _t(s), residual=_t(r)).float().cpu().numpy()
    want = oracle.matmul_w8a16_f32(a, w, s) + r.astype(np.float32)
    baseline_check(want, got, f"w8 residual M={M}")


@pytest.mark.parametrize("batch,S,H", [(1, 512, 4), (2, 200, 3), (1, 77, 2)])
def test_attention_bshd_fused_qkv_vs_oracle(cuda_pkg, oracle, batch, S, H):
    rng = np.random.default_rng(S + H)
    qkv = rng.standard_normal((batch * S, 3 * H * 128)).astype(np.float16)
    d = _t(qkv)
    HD = H * 128
    got = cuda_pkg.attention_bshd(d[:, :HD], d[:, HD:2 * HD], d[:, 2 * HD:], batch=batch,
                                  heads=H, causal=True).float().cpu().numpy()
    want = oracle.attention_bshd_f16(qkv, heads=H, seq=S, batch=batch).astype(np.float32)
    baseline_check(want, got, f"attention bshd {batch}x{S}x{H}")


def _weights(rng, hidden, ffn, scale_lo, scale_hi, gamma_random):
    def s(n):
        return rng.uniform(scale_lo, scale_hi, n).astype(np.float16)

    def g():
        return (rng.uniform(0.5, 1.5, hidden) if gamma_random else np.ones(hidden)).astype(np.float16)
    return {
        "attn_norm": g(), "ffn_norm": g(),
        "w_qkv": rng.integers(-127, 128, (hidden, 3 * hidden), dtype=np.int8), "s_qkv": s(3 * hidden),
        "w_o": rng.integers(-127, 128, (hidden, hidden), dtype=np.int8), "s_o": s(hidden),
        "w_gate_up": rng.integers(-127, 128, (hidden, 2 * ffn), dtype=np.int8),
        "s_gate_up": s(2 * ffn),
        "w_down": rng.integers(-127, 128, (ffn, hidden), dtype=np.int8), "s_down": s(hidden),
    }


def _run_block(cuda_pkg, x, wt, heads, batch):
    blk = cuda_pkg.DecoderBlockW8(heads=heads, **{k: _t(v) for k, v in wt.items()})
    out = blk(_t(x), batch=batch)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("batch,S,hidden,heads,ffn", [(1, 128, 512, 4, 1376), (2, 200, 1024, 8, 2752)])
def test_decoder_block_well_conditioned(cuda_pkg, oracle, batch, S, hidden, heads, ffn):
    """Small weight scales keep activations O(1) and the softmax soft, so the
    block is well conditioned and every output is compared."""
    rng = np.random.default_rng(hidden + S)
    wt = _weights(rng, hidden, ffn, 2e-4, 8e-4, gamma_random=True)
    x = rng.standard_normal((batch * S, hidden)).astype(np.float16)
    got = _run_block(cuda_pkg, x, wt, heads, batch)
    ref = oracle.decoder_block_w8(x, wt, heads=heads, batch=batch)["out"]
    assert np.isfinite(got).all()
    _block_check(ref, got, f"block {batch}x{S}x{hidden}")
    assert cuda_pkg.device_status() == 0


def test_decoder_block_baseline_config4(cuda_pkg, oracle):
    """BASELINE configuration 4 at full size: hidden 4096, 32 heads x 128, ffn
    11008, batch 1, seq 512, RMSNorm weight 1, RoPE theta 1e4, causal,
    x ~ N(0, 1), int8 weights U{-127..127}. Configuration 4 leaves the
    per-channel scales open; they are U[1.5e-4, 4e-4], i.e. the int8
    quantisation of a random init with standard deviation 0.02 (the
    Hugging Face Llama initializer range). (Configuration 2's U[0.001, 0.02]
    scales would drive the FFN output to ~1e5, past the f16 range, in the
    oracle and the GPU alike.) Every output is compared."""
    rng = np.random.default_rng(4)
    hidden, heads, ffn, S = 4096, 32, 11008, 512
    wt = _weights(rng, hidden, ffn, 1.5e-4, 4e-4, gamma_random=False)
    x = rng.standard_normal((S, hidden)).astype(np.float16)
    got = _run_block(cuda_pkg, x, wt, heads, 1)
    ref = oracle.decoder_block_w8(x, wt, heads=heads)["out"]
    assert np.isfinite(ref).all() and np.isfinite(got).all()
    _block_check(ref, got, "cfg 4 block")


# ------------------------------------------------------------- KV cache
def test_kv_cache_write(cuda_pkg, oracle):
    """SliceUpdateKvCache.update: the K and V column blocks of fused QKV rows
    land in the caches at rows [begin, begin + n) of every batch and head;
    every other row is untouched (bit-exact copy)."""
    rng = np.random.default_rng(21)
    batch, n, heads, rows, begin = 2, 37, 3, 96, 50
    qkv = rng.standard_normal((batch * n, 3 * heads * 128)).astype(np.float16)
    kc = rng.standard_normal((batch, heads, rows, 128)).astype(np.float16)
    vc = rng.standard_normal((batch, heads, rows, 128)).astype(np.float16)
    d, kd, vd = _t(qkv), _t(kc), _t(vc)
    HD = heads * 128
    cuda_pkg.kv_cache_write(d[:, HD:2 * HD], d[:, 2 * HD:], kd, vd, begin=begin, batch=batch)
    oracle.kv_cache_write(qkv[:, HD:2 * HD], qkv[:, 2 * HD:], kc, vc, begin=begin, batch=batch)
    torch.cuda.synchronize()
    assert np.array_equal(kd.cpu().numpy(), kc) and np.array_equal(vd.cpu().numpy(), vc)
    with pytest.raises(cuda_pkg.HxbError, match="exceed"):
        cuda_pkg.kv_cache_write(d[:, HD:2 * HD], d[:, 2 * HD:], kd, vd, begin=60, batch=batch)


def _block(cuda_pkg, wt, heads):
    return cuda_pkg.DecoderBlockW8(heads=heads, **{k: _t(v) for k, v in wt.items()})


@pytest.mark.parametrize("batch,S", [(1, 160), (2, 300)])
def test_cached_prefill_equals_block(cuda_pkg, oracle, batch, S):
    """A prefill through the KV cache (pos0 = 0, the whole prompt) gives the
    uncached block's bits (the same GEMMs; attention reads the same K/V
    values from the cache), and leaves the prompt's rotated K and V in it."""
    rng = np.random.default_rng(22 + S)
    hidden, heads, ffn, rows = 512, 4, 1376, 512
    wt = _weights(rng, hidden, ffn, 2e-4, 8e-4, gamma_random=True)
    x = rng.standard_normal((batch * S, hidden)).astype(np.float16)
    blk = _block(cuda_pkg, wt, heads)
    want = blk(_t(x), batch=batch)
    kc, vc = blk.new_cache(batch, rows)
    got = blk.step(_t(x), kc, vc, pos0=0, batch=batch)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), want.cpu().numpy())
    ref = oracle.decoder_block_w8(x, wt, heads=heads, batch=batch)
    HD = heads * 128
    k_ref = ref["qkv"][:, HD:2 * HD].reshape(batch, S, heads, 128).transpose(0, 2, 1, 3)
    v_ref = ref["qkv"][:, 2 * HD:].reshape(batch, S, heads, 128).transpose(0, 2, 1, 3)
    kg, vg = kc.cpu().numpy(), vc.cpu().numpy()
    assert not kg[:, :, S:].any() and not vg[:, :, S:].any()
    # rotated K within the RoPE kernel's angle error, V within the GEMM's
    assert np.abs(kg[:, :, :S].astype(np.float32) - k_ref).max() < 3e-2
    assert np.abs(vg[:, :, :S].astype(np.float32) - v_ref).max() < 3e-2
    assert cuda_pkg.device_status() == 0


@pytest.mark.parametrize("batch,prompt,steps,hidden,heads,ffn",
                         [(1, 300, 3, 512, 4, 1376), (2, 257, 2, 1024, 8, 2752)])
def test_cached_decode_steps_vs_oracle(cuda_pkg, oracle, batch, prompt, steps, hidden, heads,
                                       ffn):
    """Prefill, then single-row decode steps against the cache (the keys
    split across SMs), each compared with the oracle's cached block run on
    its own copy of the cache."""
    rng = np.random.default_rng(23 + prompt)
    wt = _weights(rng, hidden, ffn, 2e-4, 8e-4, gamma_random=True)
    rows = prompt + steps + 5
    blk = _block(cuda_pkg, wt, heads)
    kc, vc = blk.new_cache(batch, rows)
    k_ref = np.zeros((batch, heads, rows, 128), np.float16)
    v_ref = np.zeros_like(k_ref)
    x = rng.standard_normal((batch * prompt, hidden)).astype(np.float16)
    blk.step(_t(x), kc, vc, pos0=0, batch=batch)
    oracle.decoder_block_w8(x, wt, heads=heads, batch=batch, k_cache=k_ref, v_cache=v_ref)
    for i in range(steps):
        xt = rng.standard_normal((batch, hidden)).astype(np.float16)
        got = blk.step(_t(xt), kc, vc, pos0=prompt + i, batch=batch)
        torch.cuda.synchronize()
        ref = oracle.decoder_block_w8(xt, wt, heads=heads, batch=batch, pos0=prompt + i,
                                      k_cache=k_ref, v_cache=v_ref)["out"]
        g = got.cpu().numpy()
        assert np.isfinite(g.astype(np.float32)).all()
        _block_check(ref, g, f"decode step {i}")
    # the caches hold every row written so far and nothing past it
    n = prompt + steps
    assert not kc[:, :, n:].any() and not vc[:, :, n:].any()
    assert np.abs(kc[:, :, :n].float().cpu().numpy() - k_ref[:, :, :n]).max() < 3e-2
    assert cuda_pkg.device_status() == 0
