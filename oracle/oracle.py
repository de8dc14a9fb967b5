"""numpy front end of the CPU oracle (test infrastructure, not product).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module. It restates the reference's semantics for the hot path; see the
header of hxb_oracle.c for the file:line each function follows. The reference
itself cannot be built here (un-vendored IREE/LLVM/hexagon-mlir submodules,
no network); the restatement is pinned instead against the reference's own
known-answer tests (the HMX simulator test vectors, the VTCM tile-search lit
test) and the golden fixtures under tests/golden/.
"""
from __future__ import annotations

import ctypes
import math
from pathlib import Path

import numpy as np

from . import build as _build

_lib = None


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(_build.build()))
        vp, i64, c_int, c_f = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        lib.hxo_matmul_f16.argtypes = [vp, i64, vp, i64, c_int, vp, i64, vp, i64, i64, i64, i64]
        lib.hxo_matmul_w8a16.argtypes = [vp, i64, vp, i64, vp, vp, i64, i64, i64, i64]
        lib.hxo_attention.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, c_f, c_int]
        lib.hxo_hmx_known_answer.argtypes = [vp, vp, vp, ctypes.c_uint32]
        for f in (lib.hxo_matmul_f16, lib.hxo_matmul_w8a16, lib.hxo_attention,
                  lib.hxo_hmx_known_answer):
            f.restype = None
        _lib = lib
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def matmul_f32(a: np.ndarray, b: np.ndarray, *, transpose_b: bool = False,
               init: np.ndarray | None = None) -> np.ndarray:
    """f32 result of linalg.matmul(f16 a, f16 b) accumulating into init (or 0)."""
    a = np.ascontiguousarray(a, dtype=np.float16)
    b = np.ascontiguousarray(b, dtype=np.float16)
    M, K = a.shape
    N = b.shape[0] if transpose_b else b.shape[1]
    c = np.empty((M, N), dtype=np.float32)
    ip = None
    if init is not None:
        init = np.ascontiguousarray(init, dtype=np.float32)
        ip = _ptr(init)
    _load().hxo_matmul_f16(_ptr(a), K, _ptr(b), b.shape[1], int(transpose_b), ip, N,
                           _ptr(c), N, M, N, K)
    return c


def matmul_f16(a, b, *, transpose_b=False, init=None) -> np.ndarray:
    """f16 result: the f32 contraction truncated to f16 (arith.truncf)."""
    return matmul_f32(a, b, transpose_b=transpose_b, init=init).astype(np.float16)


def matmul_w8a16_f32(a: np.ndarray, w: np.ndarray, scale: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float16)
    w = np.ascontiguousarray(w, dtype=np.int8)
    scale = np.ascontiguousarray(scale, dtype=np.float16)
    M, K = a.shape
    N = w.shape[1]
    c = np.empty((M, N), dtype=np.float32)
    _load().hxo_matmul_w8a16(_ptr(a), K, _ptr(w), N, _ptr(scale), _ptr(c), N, M, N, K)
    return c


def split_scale(scale: float) -> float:
    """The per-operand factor the attention MLIR applies to Q and to K^T: the
    square root of the softmax scale, rounded to f32 (attention_layer.mlir:12
    holds 0.29730177875068026 = 128**-0.25 as an f64 constant)."""
    return float(np.float32(math.sqrt(scale)))


def attention_f32(q: np.ndarray, k: np.ndarray, v: np.ndarray, *,
                  scale: float | None = None, causal: bool = False) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float16)
    k = np.ascontiguousarray(k, dtype=np.float16)
    v = np.ascontiguousarray(v, dtype=np.float16)
    D = q.shape[-1]
    Sq, Skv = q.shape[-2], k.shape[-2]
    BH = q.size // (Sq * D)
    if D > 512:
        raise ValueError("oracle attention supports D <= 512")
    if scale is None:
        scale = D ** -0.5
    o = np.empty(q.shape, dtype=np.float32)
    _load().hxo_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(o), BH, Sq, Skv, D,
                          split_scale(scale), int(causal))
    return o


def attention_gqa_f32(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, *,
                      kv_len: int | None = None, scale: float | None = None,
                      causal: bool = False, q_pos0: int | None = None,
                      out_layout: str = "bhsd", round_scores: bool = True) -> np.ndarray:
    """Grouped-query attention over the first kv_len rows of a KV cache,
    restating SlicedCacheAttention.forward
    (integration_tests/models/micro/attention-cache-slice-f16/model.py:17-31):
    the `group` query heads of one KV head are the rows of one f16 matmul
    (:24-25), whose f16 result is widened and scaled in f32 (:26), softmax in
    f32, weights rounded to f16 (:27), weights . V (:28), output
    [B, Hq, q_len, D] ("bhsd") or permuted to [B, q_len, Hq, D] ("bshd",
    :29-30). q [B, Hq, q_len, D], caches [B, Hkv, rows, D], all f16. The f16
    matmuls accumulate in f64 and round once. causal (not in the sliced-cache
    model; the additive causal mask of the KV-cache LMs,
    integration_tests/models/kv_cache.py:72-79) masks key j > q_pos0 + i for
    query i, q_pos0 defaulting to kv_len - q_len; a row with every key masked
    is 0. round_scores=False keeps the scores in f32 (the arithmetic of a fused
    kernel that never materialises them). Returns f32 (the model's last matmul
    output before its f16 rounding)."""
    B, Hq, q_len, D = q.shape
    Hkv, rows = k_cache.shape[1], k_cache.shape[2]
    kv_len = rows if kv_len is None else kv_len
    group = Hq // Hkv
    if scale is None:
        scale = D ** -0.5
    k = k_cache[:, :, :kv_len].astype(np.float64)
    v = v_cache[:, :, :kv_len].astype(np.float64)
    qg = q.reshape(B, Hkv, group * q_len, D).astype(np.float64)
    s = np.matmul(qg, k.transpose(0, 1, 3, 2))
    s = (s.astype(np.float16) if round_scores else s).astype(np.float32) * np.float32(scale)
    if causal:
        q_pos0 = kv_len - q_len if q_pos0 is None else q_pos0
        pos = np.arange(group * q_len) % q_len
        masked = np.arange(kv_len)[None, :] > pos[:, None] + q_pos0
        s = np.where(masked[None, None], np.float32(-np.inf), s)
    m = s.max(axis=-1, keepdims=True)
    dead = ~np.isfinite(m)
    e = np.exp(s - np.where(dead, np.float32(0), m), dtype=np.float32)
    with np.errstate(invalid="ignore"):
        w = e / e.sum(axis=-1, keepdims=True, dtype=np.float32)
    w = np.where(dead, np.float32(0), w).astype(np.float16).astype(np.float64)
    o = np.matmul(w, v).astype(np.float32).reshape(B, Hkv, group, q_len, D)
    if out_layout == "bshd":
        return np.ascontiguousarray(o.transpose(0, 3, 1, 2, 4).reshape(B, q_len, Hq, D))
    return np.ascontiguousarray(o.reshape(B, Hq, q_len, D))


def hmx_known_answer(accumulations: int = 1):
    """(activation, weight, expected) of the reference's HMX accumulator test."""
    act = np.empty((32, 32), dtype=np.float16)
    wt = np.empty((32, 32), dtype=np.float16)
    out = np.empty((32, 32), dtype=np.float16)
    _load().hxo_hmx_known_answer(_ptr(act), _ptr(wt), _ptr(out), accumulations)
    return act, wt, out


# ---------------------------------------------------------------- tile search
def hmx_tile_candidates(extent: int, hmx_tile: int = 32) -> list[int]:
    """VTCMPlanning.cpp:156-165: HMX-aligned divisors of extent, else extent."""
    c = [t for t in range(hmx_tile, extent + 1, hmx_tile) if extent % t == 0]
    return c or [extent]


def hmx_vtcm_tile_search(M: int, N: int, K: int, *, lhs_bytes: int = 2,
                         rhs_bytes: int = 2, out_bytes: int = 4,
                         rhs_transposed: bool = False,
                         budget_bytes: int = 2 * 1024 * 1024,
                         double_buffering: bool = True,
                         hmx_tile: int = 32):
    """Restatement of selectHmxTileSizes (VTCMPlanning.cpp:186-260) for a
    matmul with one M, N and K dimension: returns [mTile, nTile, K] or None
    (the reference then falls back to hexagon-mlir's own search, which is not
    restated). budget_bytes is the --iree-hexagon-vtcm-tile-budget-bytes flag
    (2 MiB); KernelDispatch.cpp:22-23 halves it for double buffering and the
    search doubles it back (VTCMPlanning.cpp:206-208)."""
    opt_budget = budget_bytes // 2 if double_buffering else budget_bytes
    budget = opt_budget * (2 if double_buffering else 1)
    max_overrun = 2
    ranges = {"m": M, "n": N, "k": K}
    # operand -> (dims it reads, element bytes)
    operands = [(("m", "k"), lhs_bytes),
                (("n", "k") if rhs_transposed else ("k", "n"), rhs_bytes),
                (("m", "n"), out_bytes)]
    best, best_rank = None, None
    for mt in hmx_tile_candidates(M, hmx_tile):
        for nt in hmx_tile_candidates(N, hmx_tile):
            tiles = {"m": mt, "n": nt, "k": K}
            num_tiles = 1
            for d in ("m", "n", "k"):
                num_tiles *= ranges[d] // tiles[d]
            vtcm = traffic = 0
            for dims, eb in operands:
                b = eb
                for d in dims:
                    b *= tiles[d]
                invariant = all(tiles[d] == ranges[d] for d in dims)
                vtcm += 2 * b if (double_buffering and not invariant) else b
                traffic += b if invariant else b * num_tiles
            if vtcm > max_overrun * budget:
                continue
            rank = (vtcm > budget, traffic, num_tiles, -nt)
            if best is not None and rank >= best_rank:
                continue
            best, best_rank = [mt, nt, K], rank
    return best


# ------------------------------------------------------------ decoder block
# The reference has no decoder kernels; its decoder models are Hugging Face
# Llama modules run by torch (integration_tests/models/meta-llama/
# Llama-3.2-1B-Instruct/model.py:8-16 loads a Llama checkpoint with transformers'
# AutoModelForCausalLM). These
# restate the arithmetic of those modules for an f16 model: statistics in f32,
# every intermediate tensor rounded to f16 where the f16 model stores one.

def rmsnorm_f16(x: np.ndarray, gamma: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """LlamaRMSNorm: f32 mean of squares, x * rsqrt(var + eps) rounded to f16,
    times the f16 weight (one f16 rounding of the product)."""
    x32 = x.astype(np.float32)
    var = np.mean(x32.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    y = (x32 * (1.0 / np.sqrt(var + np.float32(eps))).astype(np.float32)).astype(np.float16)
    return (y.astype(np.float32) * gamma.astype(np.float32)).astype(np.float16)


def rope_f16(x: np.ndarray, heads: int, seq: int, pos0: int = 0,
             theta: float = 10000.0) -> np.ndarray:
    """Llama rotary embedding (rotate_half convention) applied to the first
    `heads` 128-wide heads of every row; row r has position pos0 + r % seq."""
    out = x.copy()
    rows = x.shape[0]
    i = np.arange(64, dtype=np.float64)
    inv_freq = theta ** (-2.0 * i / 128.0)
    pos = (pos0 + np.arange(rows) % seq).astype(np.float64)
    ang = pos[:, None] * inv_freq[None, :]
    cs, sn = np.cos(ang), np.sin(ang)
    for h in range(heads):
        a = x[:, h * 128:h * 128 + 64].astype(np.float64)
        b = x[:, h * 128 + 64:h * 128 + 128].astype(np.float64)
        out[:, h * 128:h * 128 + 64] = (a * cs - b * sn).astype(np.float16)
        out[:, h * 128 + 64:h * 128 + 128] = (b * cs + a * sn).astype(np.float16)
    return out


def swiglu_f16(gu: np.ndarray) -> np.ndarray:
    """LlamaMLP activation: silu(gate) * up on a fused [rows, 2F] gate/up output."""
    F = gu.shape[1] // 2
    g = gu[:, :F].astype(np.float64)
    u = gu[:, F:].astype(np.float64)
    return (g / (1.0 + np.exp(-g)) * u).astype(np.float16)


def linear_w8_f16(a: np.ndarray, w: np.ndarray, s: np.ndarray,
                  residual: np.ndarray | None = None) -> np.ndarray:
    """f16(a . w * s [+ residual]) with the contraction in f32 (one rounding)."""
    c = matmul_w8a16_f32(a, w, s)
    if residual is not None:
        c = c + residual.astype(np.float32)
    return c.astype(np.float16)


def attention_bshd_f16(qkv_or_q: np.ndarray, *, heads: int, seq: int, batch: int = 1,
                       k: np.ndarray | None = None, v: np.ndarray | None = None,
                       causal: bool = True) -> np.ndarray:
    """Attention over [batch*seq, heads*128] q/k/v matrices (or the q, k, v
    column blocks of one fused [rows, 3*heads*128] matrix), output in the same
    [batch*seq, heads*128] order, rounded to f16."""
    HD = heads * 128
    if k is None:
        q, k, v = qkv_or_q[:, :HD], qkv_or_q[:, HD:2 * HD], qkv_or_q[:, 2 * HD:3 * HD]
    else:
        q = qkv_or_q

    def to_bh(t):
        return np.ascontiguousarray(
            t.reshape(batch, seq, heads, 128).transpose(0, 2, 1, 3).reshape(batch * heads, seq, 128))
    o = attention_f32(to_bh(q), to_bh(k), to_bh(v), causal=causal).astype(np.float16)
    return np.ascontiguousarray(o.reshape(batch, heads, seq, 128).transpose(0, 2, 1, 3)
                                .reshape(batch * seq, HD))


def kv_cache_write(k_src: np.ndarray, v_src: np.ndarray, k_cache: np.ndarray,
                   v_cache: np.ndarray, *, begin: int, batch: int = 1) -> None:
    """SliceUpdateKvCache.update (integration_tests/models/kv_cache.py:101-112)
    on [batch * n, heads * D] source rows: cache[b, h, begin + t] = the head-h
    columns of row b * n + t. Updates the caches in place."""
    B, H, rows, D = k_cache.shape
    n = k_src.shape[0] // batch
    for src, cache in ((k_src, k_cache), (v_src, v_cache)):
        cache[:, :, begin:begin + n] = (src[:, :H * D].reshape(batch, n, H, D)
                                        .transpose(0, 2, 1, 3))


def decoder_block_w8(x: np.ndarray, wt: dict, *, heads: int, batch: int = 1, pos0: int = 0,
                     eps: float = 1e-5, theta: float = 10000.0,
                     k_cache: np.ndarray | None = None,
                     v_cache: np.ndarray | None = None) -> dict:
    """Every intermediate of the decoder block for
    x [batch*seq, hidden] f16; wt holds attn_norm, w_qkv, s_qkv, w_o, s_o,
    ffn_norm, w_gate_up, s_gate_up, w_down, s_down as numpy arrays. With
    k_cache / v_cache ([batch, heads, rows, 128] f16, updated in place) the
    rotated K and V of the new rows are written at rows pos0 .. and attention
    reads keys [0, pos0 + seq) from the caches (kv_cache.py:101-112,
    grouped_query_attention :46-86 with one query head per KV head)."""
    seq = x.shape[0] // batch
    r = {}
    r["h"] = rmsnorm_f16(x, wt["attn_norm"], eps)
    r["qkv_raw"] = linear_w8_f16(r["h"], wt["w_qkv"], wt["s_qkv"])
    r["qkv"] = rope_f16(r["qkv_raw"], 2 * heads, seq, pos0, theta)
    if k_cache is None:
        r["att"] = attention_bshd_f16(r["qkv"], heads=heads, seq=seq, batch=batch)
    else:
        HD = heads * 128
        kv_cache_write(r["qkv"][:, HD:2 * HD], r["qkv"][:, 2 * HD:], k_cache, v_cache,
                       begin=pos0, batch=batch)
        kv_len = pos0 + seq
        q = np.ascontiguousarray(r["qkv"][:, :HD].reshape(batch, seq, heads, 128)
                                 .transpose(0, 2, 1, 3).reshape(batch * heads, seq, 128))
        kk = np.ascontiguousarray(k_cache[:, :, :kv_len]).reshape(batch * heads, kv_len, 128)
        vv = np.ascontiguousarray(v_cache[:, :, :kv_len]).reshape(batch * heads, kv_len, 128)
        o = attention_f32(q, kk, vv, causal=True).astype(np.float16)
        r["att"] = np.ascontiguousarray(o.reshape(batch, heads, seq, 128).transpose(0, 2, 1, 3)
                                        .reshape(batch * seq, HD))
    r["h2"] = linear_w8_f16(r["att"], wt["w_o"], wt["s_o"], residual=x)
    r["n2"] = rmsnorm_f16(r["h2"], wt["ffn_norm"], eps)
    r["gu"] = linear_w8_f16(r["n2"], wt["w_gate_up"], wt["s_gate_up"])
    r["a"] = swiglu_f16(r["gu"])
    r["out"] = linear_w8_f16(r["a"], wt["w_down"], wt["s_down"], residual=r["h2"])
    return r
