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
