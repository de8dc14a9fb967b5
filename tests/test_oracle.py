"""Pins the CPU oracle before it is trusted as the checker (no GPU needed).

Anchors, all from the reference:
  * the HMX simulator known answers (plugins/runtime/hexagon/dsp/ukernel/hmx/
    test/accumulator_test.c:14-42, test_support.c:242-260): bit-exact;
  * the VTCM tile-search lit test (plugins/compiler/hexagon/test/codegen/
    strategy/hexagon_vtcm_planning_hmx.mlir:44,64,84,104,123,142);
  * the golden outputs of the reference's own micro models run eagerly
    (tests/golden/, made by tests/golden/make_golden.py), within each model's
    own tolerances from its model.yaml.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from _support import compare, golden_expected, golden_inputs, golden_manifest, select_rows


def test_hmx_known_answer_single_and_accumulating(oracle):
    a, w, expected1 = oracle.hmx_known_answer(1)
    # independent closed form: W = I + 0.5 * cyclic super-diagonal
    closed = a.astype(np.float32) + 0.5 * np.roll(a.astype(np.float32), 1, axis=1)
    assert np.array_equal(expected1, closed.astype(np.float16))
    assert np.array_equal(oracle.matmul_f16(a, w), expected1)
    _, _, expected2 = oracle.hmx_known_answer(2)
    # two MMAs without a clear accumulate (accumulator_test.c:61-72)
    twice = oracle.matmul_f16(a, w, init=oracle.matmul_f32(a, w))
    assert np.array_equal(twice, expected2)


@pytest.mark.parametrize("shape,rhs_t,out_bytes,expected", [
    ((52, 896, 7680), True, 4, [52, 32, 7680]),     # planning_hmx.mlir:44
    ((128, 2560, 9728), True, 2, [128, 32, 9728]),  # :64 (over budget, <= 2x)
    ((64, 64, 32768), True, 2, None),               # :84 cap -> hexagon-mlir fallback
    ((32, 32, 128), False, 4, [32, 32, 128]),       # :104 dynamic K <= 128
    ((1024, 1024, 2048), False, 4, [64, 128, 2048]),  # :123 dynamic M <= 1024
    ((1024, 1024, 2048), False, 4, [64, 128, 2048]),  # :142 dynamic N <= 1024
])
def test_vtcm_tile_search_pins(oracle, shape, rhs_t, out_bytes, expected):
    assert oracle.hmx_vtcm_tile_search(*shape, rhs_transposed=rhs_t,
                                       out_bytes=out_bytes) == expected


def test_tile_candidates(oracle):
    assert oracle.hmx_tile_candidates(52) == [52]
    assert oracle.hmx_tile_candidates(96) == [32, 96]
    assert oracle.hmx_tile_candidates(128) == [32, 64, 128]


def _golden_matmul_keys():
    return [k for k, e in golden_manifest().items() if "matmul" in e["model"]]


@pytest.mark.parametrize("key", _golden_matmul_keys())
def test_oracle_matches_reference_golden_matmul(oracle, key):
    entry = golden_manifest()[key]
    a, b = golden_inputs(key)
    a, b = a.numpy(), b.numpy()
    transposed = "rhs-transposed" in key
    if a.ndim == 3:  # batch matmul: one oracle call per batch
        got = np.stack([oracle.matmul_f32(a[i], b[i]) for i in range(a.shape[0])])
    else:
        got = oracle.matmul_f32(a, b, transpose_b=transposed)
    if entry["out_dtype"] == "float16":
        got = got.astype(np.float16)
    exp, rows = golden_expected(key)
    tol = entry["tolerances"]
    c = compare(exp, select_rows(got, rows), tol["atol"], tol["rtol"])
    assert c.close, f"{key}: {c}"
    assert c.rel_l2_percent <= tol["relative_l2_percent"], f"{key}: {c}"
    assert math.isclose(float(got.astype(np.float64).sum()), entry["out_sum"],
                        rel_tol=1e-3, abs_tol=1.0)


def test_oracle_matches_reference_golden_attention(oracle):
    key = "micro__attention-4x1024x128-f16"
    entry = golden_manifest()[key]
    q, k, v = (t.numpy() for t in golden_inputs(key))
    got = oracle.attention_f32(q, k, v).astype(np.float16)
    exp, rows = golden_expected(key)
    tol = entry["tolerances"]
    c = compare(exp, select_rows(got, rows), tol["atol"], tol["rtol"])
    assert c.close and c.rel_l2_percent <= tol["relative_l2_percent"], str(c)


def test_oracle_matches_reference_golden_gqa_attention(oracle):
    """integration_tests/models/micro/attention-cache-slice-f16: 9 query heads
    over 3 KV heads, the first 64 of 128 cache rows, output permuted to
    [batch, q_len, heads, D]."""
    key = "micro__attention-cache-slice-f16"
    entry = golden_manifest()[key]
    q, k, v = (t.numpy() for t in golden_inputs(key))
    got = oracle.attention_gqa_f32(q, k, v, kv_len=64, out_layout="bshd").astype(np.float16)
    exp, rows = golden_expected(key)
    assert rows is None and exp.shape == got.shape == (1, 64, 9, 64)
    tol = entry["tolerances"]
    c = compare(exp, got, tol["atol"], tol["rtol"])
    assert c.close and c.rel_l2_percent <= tol["relative_l2_percent"], str(c)
    # the restatement follows the model's roundings: nearly every element is
    # bit-identical to the eager output, the rest differ by accumulation order
    # (100x inside the model's atol)
    assert (got == exp).mean() > 0.99
    assert np.abs(got.astype(np.float32) - exp.astype(np.float32)).max() <= 5e-4


@pytest.mark.parametrize("causal", [False, True])
def test_oracle_gqa_equals_attention_on_repeated_heads(oracle, causal):
    """GQA over a cache slice is plain attention with each KV head repeated
    for its query heads (up to the f16 rounding of the scores that the
    sliced-cache model does and the attention layer does not)."""
    rng = np.random.default_rng(3)
    B, Hq, Hkv, q_len, kv_len, rows, D = 2, 6, 2, 20, 45, 64, 64
    q = rng.standard_normal((B, Hq, q_len, D)).astype(np.float16)
    k = rng.standard_normal((B, Hkv, rows, D)).astype(np.float16)
    v = rng.standard_normal((B, Hkv, rows, D)).astype(np.float16)
    got = oracle.attention_gqa_f32(q, k, v, kv_len=kv_len, causal=causal)
    rep = lambda t: np.repeat(t[:, :, :kv_len], Hq // Hkv, axis=1).reshape(B * Hq, kv_len, D)
    want = oracle.attention_f32(q.reshape(B * Hq, q_len, D), rep(k), rep(v), causal=causal)
    assert np.abs(got.reshape(want.shape) - want).max() < 5e-3
    bshd = oracle.attention_gqa_f32(q, k, v, kv_len=kv_len, causal=causal, out_layout="bshd")
    assert np.array_equal(bshd, got.transpose(0, 2, 1, 3))
    # with f32 scores only the f16 weights (model.py:27) remain as a difference
    exact = oracle.attention_gqa_f32(q, k, v, kv_len=kv_len, causal=causal, round_scores=False)
    assert np.abs(exact.reshape(want.shape) - want).max() < 1e-3


def test_oracle_gqa_padded_prefill_mask(oracle):
    """q_pos0 = 0 with kv_len cut at the last real token: the prefill mask of
    integration_tests/models/kv_cache.py:160-171 (causal, and no key past
    input_length), against a direct additive-mask softmax."""
    rng = np.random.default_rng(4)
    B, Hq, Hkv, n, last, D = 1, 4, 2, 12, 8, 64
    q = rng.standard_normal((B, Hq, n, D)).astype(np.float16)
    k = rng.standard_normal((B, Hkv, 16, D)).astype(np.float16)
    v = rng.standard_normal((B, Hkv, 16, D)).astype(np.float16)
    got = oracle.attention_gqa_f32(q, k, v, kv_len=last + 1, causal=True, q_pos0=0,
                                   round_scores=False)
    kk = np.repeat(k[:, :, :n], 2, axis=1).astype(np.float64)
    vv = np.repeat(v[:, :, :n], 2, axis=1).astype(np.float64)
    s = q.astype(np.float64) @ kk.transpose(0, 1, 3, 2) * D ** -0.5
    i, j = np.arange(n)[:, None], np.arange(n)[None, :]
    s = s + np.where((j <= i) & (j <= last), 0.0, -np.inf)
    w = np.exp(s - s.max(-1, keepdims=True))
    w = (w / w.sum(-1, keepdims=True)).astype(np.float16).astype(np.float64)
    assert np.abs(got - w @ vv).max() < 1e-4


def test_attention_split_scale_constant(oracle):
    # attention_layer.mlir:12 holds s = 0.29730177875068026 for head_dim 128
    assert oracle.split_scale(128 ** -0.5) == float(np.float32(0.29730177875068026))


@pytest.mark.parametrize("causal", [False, True])
def test_oracle_attention_vs_float64(oracle, causal):
    rng = np.random.default_rng(3)
    BH, Sq, Skv, D = 3, 37, 53, 128
    q = rng.standard_normal((BH, Sq, D)).astype(np.float16)
    k = rng.standard_normal((BH, Skv, D)).astype(np.float16)
    v = rng.standard_normal((BH, Skv, D)).astype(np.float16)
    got = oracle.attention_f32(q, k, v, causal=causal)
    s = q.astype(np.float64) @ np.swapaxes(k.astype(np.float64), 1, 2) / math.sqrt(D)
    if causal:
        i = np.arange(Sq)[:, None]
        j = np.arange(Skv)[None, :]
        s = np.where(j > i + (Skv - Sq), -np.inf, s)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    want = p @ v.astype(np.float64)
    assert np.abs(got - want).max() < 2e-5


def test_oracle_attention_vs_torch_sdpa(oracle):
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(2, 64, 128, generator=g).half() for _ in range(3))
    want = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float(), v.float(), is_causal=True).numpy()
    got = oracle.attention_f32(q.numpy(), k.numpy(), v.numpy(), causal=True)
    assert np.abs(got - want).max() < 1e-5


def test_fully_masked_rows_are_zero(oracle):
    # attention_layer.mlir:86-103: a row whose scores are all -inf selects 0
    q = np.zeros((1, 2, 128), np.float16)
    k = np.zeros((1, 3, 128), np.float16)
    k[0, :, 0] = -np.inf
    q[0, 0, 0] = 1.0
    v = np.ones((1, 3, 128), np.float16)
    out = oracle.attention_f32(q, k, v)
    assert np.array_equal(out[0, 0], np.zeros(128, np.float32))


def test_oracle_matmul_vs_float64_ragged(oracle):
    rng = np.random.default_rng(11)
    for (M, N, K) in [(1, 1, 1), (3, 5, 7), (17, 19, 23), (130, 70, 300)]:
        a = rng.uniform(-1, 1, (M, K)).astype(np.float16)
        b = rng.uniform(-1, 1, (K, N)).astype(np.float16)
        init = rng.standard_normal((M, N)).astype(np.float32)
        got = oracle.matmul_f32(a, b, init=init)
        want = init + a.astype(np.float64) @ b.astype(np.float64)
        assert np.abs(got - want).max() < 1e-4 * max(1, K ** 0.5)
        gt = oracle.matmul_f32(a, np.ascontiguousarray(b.T), transpose_b=True)
        assert np.array_equal(gt, oracle.matmul_f32(a, b))


def test_oracle_w8a16_vs_float64(oracle):
    rng = np.random.default_rng(5)
    M, K, N = 9, 200, 77
    a = rng.standard_normal((M, K)).astype(np.float16)
    w = rng.integers(-127, 128, (K, N), dtype=np.int8)
    s = rng.uniform(0.001, 0.02, N).astype(np.float16)
    got = oracle.matmul_w8a16_f32(a, w, s)
    want = a.astype(np.float64) @ (w.astype(np.float64) * s.astype(np.float64))
    assert np.abs(got - want).max() < 1e-3


def test_oracle_cached_decoder_matches_uncached(oracle):
    """The oracle's KV-cache block: a prefill of S rows then a decode step at
    position S give the bits of the uncached block on S + 1 rows (the linears
    and RoPE are row-wise, the attention row sees the same keys)."""
    rng = np.random.default_rng(5)
    hidden, heads, ffn, S = 256, 2, 512, 20

    def s(n):
        return rng.uniform(2e-4, 8e-4, n).astype(np.float16)
    wt = {"attn_norm": np.ones(hidden, np.float16), "ffn_norm": np.ones(hidden, np.float16),
          "w_qkv": rng.integers(-127, 128, (hidden, 3 * hidden), dtype=np.int8),
          "s_qkv": s(3 * hidden),
          "w_o": rng.integers(-127, 128, (hidden, hidden), dtype=np.int8), "s_o": s(hidden),
          "w_gate_up": rng.integers(-127, 128, (hidden, 2 * ffn), dtype=np.int8),
          "s_gate_up": s(2 * ffn),
          "w_down": rng.integers(-127, 128, (ffn, hidden), dtype=np.int8), "s_down": s(hidden)}
    x = rng.standard_normal((S + 1, hidden)).astype(np.float16)
    full = oracle.decoder_block_w8(x, wt, heads=heads)["out"]
    kc = np.zeros((1, heads, S + 4, 128), np.float16)
    vc = np.zeros_like(kc)
    pre = oracle.decoder_block_w8(x[:S], wt, heads=heads, k_cache=kc, v_cache=vc)["out"]
    assert np.array_equal(pre, oracle.decoder_block_w8(x[:S], wt, heads=heads)["out"])
    step = oracle.decoder_block_w8(x[S:], wt, heads=heads, pos0=S, k_cache=kc, v_cache=vc)["out"]
    assert np.array_equal(step, full[S:])
    assert not kc[:, :, S + 1:].any()
