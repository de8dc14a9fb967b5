"""Parity of the fused tcgen05 attention dispatch (through the C ABI) with the
oracle's restatement of examples/attention_layer/attention_layer.mlir:17-111
and with the reference's golden micro model
(integration_tests/models/micro/attention-4x1024x128-f16)."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from _support import (baseline_check, compare, golden_expected, golden_inputs,
                      golden_manifest, select_rows)

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _qkv(BH, Sq, Skv, seed, D=128):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((BH, Sq, D)).astype(np.float16)
    k = rng.standard_normal((BH, Skv, D)).astype(np.float16)
    v = rng.standard_normal((BH, Skv, D)).astype(np.float16)
    return q, k, v


def _run(pkg, q, k, v, causal=False, scale=None):
    qd, kd, vd = (torch.from_numpy(x).to(DEV) for x in (q, k, v))
    out = pkg.attention(qd, kd, vd, causal=causal, scale=scale)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("BH,Sq,Skv", [(2, 256, 256), (3, 128, 512), (1, 512, 128),
                                       (2, 200, 333), (1, 1, 1), (1, 17, 300),
                                       (5, 300, 129)])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_vs_oracle(cuda_pkg, oracle, BH, Sq, Skv, causal):
    q, k, v = _qkv(BH, Sq, Skv, seed=BH * 1000 + Sq + Skv)
    got = _run(cuda_pkg, q, k, v, causal=causal)
    want = oracle.attention_f32(q, k, v, causal=causal)
    baseline_check(want, got, f"attention {BH}x{Sq}x{Skv} causal={causal}")
    assert cuda_pkg.device_status() == 0


def test_attention_fully_masked_rows_are_zero(cuda_pkg, oracle):
    """Causal with Sq > Skv: the first Sq - Skv query rows see no key at all;
    attention_layer.mlir:86-103 selects 0 for them."""
    q, k, v = _qkv(2, 300, 100, seed=5)
    got = _run(cuda_pkg, q, k, v, causal=True)
    assert np.array_equal(got[:, :200], np.zeros_like(got[:, :200]))
    baseline_check(oracle.attention_f32(q, k, v, causal=True), got, "masked rows")


def test_attention_large_scores_rescale(cuda_pkg, oracle):
    """Keys whose scores grow block after block force the running maximum to
    move by more than the rescale threshold several times."""
    BH, S = 2, 1024
    q, k, v = _qkv(BH, S, S, seed=9)
    ramp = np.linspace(0.2, 3.0, S, dtype=np.float32)[None, :, None]
    k = (k.astype(np.float32) * ramp).astype(np.float16)
    got = _run(cuda_pkg, q, k, v)
    baseline_check(oracle.attention_f32(q, k, v), got, "rescale")


def test_attention_custom_scale(cuda_pkg, oracle):
    q, k, v = _qkv(2, 256, 384, seed=13)
    got = _run(cuda_pkg, q, k, v, scale=0.3)
    baseline_check(oracle.attention_f32(q, k, v, scale=0.3), got, "scale=0.3")


def test_attention_vs_reference_golden(cuda_pkg, oracle):
    """integration_tests/models/micro/attention-4x1024x128-f16: the reference's
    own torch-eager output under its model.yaml tolerances."""
    key = "micro__attention-4x1024x128-f16"
    entry = golden_manifest()[key]
    q, k, v = (t.numpy() for t in golden_inputs(key))
    got = _run(cuda_pkg, q, k, v).astype(np.float16)
    exp, rows = golden_expected(key)
    tol = entry["tolerances"]
    c = compare(exp, select_rows(got, rows), tol["atol"], tol["rtol"])
    assert c.close and c.rel_l2_percent <= tol["relative_l2_percent"], str(c)
    assert math.isclose(float(got.astype(np.float64).sum()), entry["out_sum"],
                        rel_tol=1e-3, abs_tol=1.0)
    baseline_check(oracle.attention_f32(q, k, v), got.astype(np.float32), key)


def test_attention_baseline_config_heads(cuda_pkg, oracle):
    """BASELINE configuration 3 ([4, 32, 2048, 128], scale 1/sqrt(128)) at full
    size on the GPU; a sample of heads is checked against the oracle, and
    every output row is a convex combination of V rows (bounded by V's range)."""
    B, H, S, D = 4, 32, 2048, 128
    g = torch.Generator(device=DEV).manual_seed(0)
    q, k, v = (torch.randn(B, H, S, D, device=DEV, generator=g).half() for _ in range(3))
    out = cuda_pkg.attention(q, k, v)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    vmax = v.float().amax(dim=2, keepdim=True)
    vmin = v.float().amin(dim=2, keepdim=True)
    o = out.float()
    assert bool(((o <= vmax + 1e-2) & (o >= vmin - 1e-2)).all())
    for b, h in [(0, 0), (1, 17), (3, 31)]:
        want = oracle.attention_f32(q[b, h].cpu().numpy()[None], k[b, h].cpu().numpy()[None],
                                    v[b, h].cpu().numpy()[None])
        baseline_check(want[0], o[b, h].cpu().numpy(), f"cfg3 head ({b},{h})")


def test_attention_rejects_unsupported_head_dim(cuda_pkg):
    q = torch.zeros(1, 16, 96, dtype=torch.float16, device=DEV)
    with pytest.raises(cuda_pkg.HxbError, match="head dim"):
        cuda_pkg.attention(q, q, q)


@pytest.mark.parametrize("BH,Sq,Skv,causal", [(3, 256, 256, False), (2, 200, 333, True),
                                              (1, 1, 700, False), (4, 513, 129, True)])
def test_attention_head_dim_64(cuda_pkg, oracle, BH, Sq, Skv, causal):
    q, k, v = _qkv(BH, Sq, Skv, seed=64 + Sq + Skv, D=64)
    got = _run(cuda_pkg, q, k, v, causal=causal)
    baseline_check(oracle.attention_f32(q, k, v, causal=causal), got,
                   f"attention D=64 {BH}x{Sq}x{Skv} causal={causal}")


# ----------------------------------------------- grouped-query, sliced cache
def _gqa_inputs(B, Hq, Hkv, q_len, rows, D, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, Hq, q_len, D)).astype(np.float16)
    k = rng.standard_normal((B, Hkv, rows, D)).astype(np.float16)
    v = rng.standard_normal((B, Hkv, rows, D)).astype(np.float16)
    return q, k, v


@pytest.mark.parametrize("B,Hq,Hkv,q_len,q_pos0,kv_len,rows,D,causal,layout", [
    (1, 9, 3, 64, None, 64, 128, 64, False, "bshd"),   # the sliced-cache micro model
    (2, 8, 2, 1, None, 300, 512, 128, False, "bhsd"),  # decode, group 4
    (1, 32, 8, 1, None, 1000, 1024, 64, True, "bshd"), # decode against a long cache
    (2, 12, 4, 100, None, 250, 256, 64, True, "bhsd"), # a group spans two CTAs
    (1, 4, 4, 130, None, 130, 200, 128, True, "bshd"), # no grouping, cache rows > kv_len
    (3, 6, 1, 50, None, 77, 77, 64, False, "bhsd"),    # one KV head for all (MQA)
    (1, 16, 2, 40, None, 30, 64, 128, True, "bhsd"),   # q_len > kv_len: masked rows
    (1, 9, 3, 96, 0, 70, 128, 64, True, "bshd"),       # padded prefill: keys cut at 70
    (2, 15, 5, 32, 200, 232, 256, 64, True, "bshd"),   # chunked prefill after 200 tokens
    (2, 16, 4, 4, 100, 180, 256, 128, True, "bshd"),   # 16 rows per KV head, from position 100
    (1, 6, 3, 1, None, 129, 200, 128, False, "bhsd"),  # 2 rows per KV head, a ragged key block
])
def test_attention_gqa_vs_oracle(cuda_pkg, oracle, B, Hq, Hkv, q_len, q_pos0, kv_len, rows, D,
                                 causal, layout):
    q, k, v = _gqa_inputs(B, Hq, Hkv, q_len, rows, D, seed=Hq * 100 + q_len + kv_len)
    qd, kd, vd = (torch.from_numpy(x).to(DEV) for x in (q, k, v))
    got = cuda_pkg.attention_gqa(qd, kd, vd, kv_len=kv_len, causal=causal, q_pos0=q_pos0,
                                 out_layout=layout)
    torch.cuda.synchronize()
    got = got.float().cpu().numpy()
    kw = dict(kv_len=kv_len, causal=causal, q_pos0=q_pos0, out_layout=layout)
    # the fused arithmetic (f32 scores) within the baseline bar
    want = oracle.attention_gqa_f32(q, k, v, round_scores=False, **kw)
    what = f"gqa {B}x{Hq}/{Hkv}x{q_len}@{q_pos0}x{kv_len}/{rows}x{D} {causal} {layout}"
    baseline_check(want, got, what)
    if causal and q_pos0 is None and q_len > kv_len:
        dead = q_len - kv_len  # positions that see no key
        assert not got.reshape(B, Hq, q_len, D)[:, :, :dead].any()
    # and the model's own roundings within its tolerance
    c = compare(oracle.attention_gqa_f32(q, k, v, **kw), got, 5e-2, 5e-2)
    assert c.close and c.rel_l2_percent <= 1.0, str(c)
    assert cuda_pkg.device_status() == 0


def test_attention_gqa_vs_reference_golden(cuda_pkg, oracle):
    """integration_tests/models/micro/attention-cache-slice-f16: the
    reference's own torch-eager output of SlicedCacheAttention(context=64)
    under its model.yaml tolerances."""
    key = "micro__attention-cache-slice-f16"
    entry = golden_manifest()[key]
    q, k, v = (t.to(DEV) for t in golden_inputs(key))
    got = cuda_pkg.attention_gqa(q, k, v, kv_len=64, out_layout="bshd")
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    exp, rows = golden_expected(key)
    tol = entry["tolerances"]
    c = compare(exp, got, tol["atol"], tol["rtol"])
    assert c.close and c.rel_l2_percent <= tol["relative_l2_percent"], str(c)
    assert math.isclose(float(got.astype(np.float64).sum()), entry["out_sum"],
                        rel_tol=1e-2, abs_tol=0.5)


def test_attention_gqa_rejects_bad_layouts(cuda_pkg):
    q = torch.zeros(1, 9, 8, 64, dtype=torch.float16, device=DEV)
    kv = torch.zeros(1, 2, 16, 64, dtype=torch.float16, device=DEV)
    with pytest.raises(cuda_pkg.HxbError, match="multiple"):
        cuda_pkg.attention_gqa(q, kv, kv)            # 9 query heads over 2 KV heads
    kv = torch.zeros(1, 3, 16, 64, dtype=torch.float16, device=DEV)
    with pytest.raises(cuda_pkg.HxbError, match="exceeds"):
        cuda_pkg.attention_gqa(q, kv, kv, kv_len=17)  # more keys than cache rows


@pytest.mark.parametrize("B,Hq,Hkv,q_len,q_pos0,kv_len,rows,D,causal", [
    (1, 32, 8, 1, None, 4000, 4096, 128, False),  # decode, long cache: 8 heads x 16 splits
    (4, 32, 8, 1, None, 8192, 8192, 128, True),   # batched decode
    (1, 9, 3, 1, None, 700, 1024, 64, True),      # SmolLM2-like heads, D = 64
    (1, 8, 8, 100, 0, 1000, 1024, 128, True),     # most splits see no visible key
    (2, 28, 4, 4, None, 1500, 2048, 128, True),   # a 4-token step, group 7
    (1, 8, 2, 4, None, 600, 1024, 128, True),     # 16 rows per KV head, causal
    (3, 16, 8, 1, None, 2000, 2048, 128, False),  # group 2
])
def test_attention_gqa_split_keys(cuda_pkg, oracle, B, Hq, Hkv, q_len, q_pos0, kv_len, rows, D,
                                  causal):
    """Short queries against a long cache split the keys across SMs; the
    merged result matches the oracle and the unsplit kernel."""
    n = cuda_pkg.attention_gqa_workspace_bytes(B, Hq, Hkv, q_len, kv_len, D)
    assert n > 0, "this shape is expected to split"
    q, k, v = _gqa_inputs(B, Hq, Hkv, q_len, rows, D, seed=kv_len + q_len)
    qd, kd, vd = (torch.from_numpy(x).to(DEV) for x in (q, k, v))
    kw = dict(kv_len=kv_len, causal=causal, q_pos0=q_pos0)
    ws = torch.empty(n, dtype=torch.uint8, device=DEV)
    split = cuda_pkg.attention_gqa(qd, kd, vd, workspace=ws, **kw)
    whole = cuda_pkg.attention_gqa(qd, kd, vd, workspace=None, **kw)
    torch.cuda.synchronize()
    split, whole = split.float().cpu().numpy(), whole.float().cpu().numpy()
    want = oracle.attention_gqa_f32(q, k, v, round_scores=False, **kw)
    baseline_check(want, split, f"split gqa {B}x{Hq}/{Hkv}x{q_len}x{kv_len}")
    baseline_check(want, whole, f"unsplit gqa {B}x{Hq}/{Hkv}x{q_len}x{kv_len}")
    assert np.abs(split - whole).max() < 4e-3
    assert cuda_pkg.device_status() == 0


def test_attention_gqa_workspace_query(cuda_pkg):
    # long prefill fills the SMs by itself: no split, no workspace
    assert cuda_pkg.attention_gqa_workspace_bytes(4, 32, 8, 2048, 2048, 128) == 0
    # a single key block cannot split
    assert cuda_pkg.attention_gqa_workspace_bytes(1, 32, 8, 1, 100, 128) == 0
    assert cuda_pkg.attention_gqa_workspace_bytes(1, 9, 2, 1, 100, 64) == 0  # invalid heads
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    n = cuda_pkg.attention_gqa_workspace_bytes(1, 32, 8, 1, 4096, 128)
    # 4 rows per KV head on the decode kernel: at most two CTAs per SM
    assert 0 < n <= (2 * sms * 4 * 129 * 4 + 16)
