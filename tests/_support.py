"""Test helpers: golden-fixture access and the accuracy metrics.

compare() restates the reference harness's metrics
(integration_tests/stages/checking.py:46-83): comparison in float64,
relative L2 error in percent, max abs difference and
np.allclose(atol, rtol). baseline_check() adds BASELINE.json's bar for the
B200 path against the f32 oracle: elementwise |got - ref| <= 1e-2 + one f16
ulp of |ref| (f16 rounding alone can exceed 1e-2 once |ref| >= 8, so the
ulp term is written into the bound) and relative L2 <= 1e-3.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


@dataclass
class Comparison:
    rel_l2_percent: float
    max_abs: float
    close: bool

    def __str__(self):
        return (f"rel-L2 {self.rel_l2_percent:.5f}% max|d| {self.max_abs:.4g} "
                f"allclose={self.close}")


def compare(ref: np.ndarray, act: np.ndarray, atol: float, rtol: float) -> Comparison:
    assert ref.shape == act.shape, (ref.shape, act.shape)
    r = ref.astype(np.float64)
    a = act.astype(np.float64)
    rn = float(np.linalg.norm(r))
    en = float(np.linalg.norm(a - r))
    rel = en / rn * 100.0 if rn > 0 else 100.0
    return Comparison(rel, float(np.abs(a - r).max()) if r.size else 0.0,
                      bool(np.allclose(a, r, atol=atol, rtol=rtol, equal_nan=False)))


def f16_ulp(x: np.ndarray) -> np.ndarray:
    x = np.abs(x.astype(np.float32)).astype(np.float16)
    return (np.spacing(x).astype(np.float64))


def baseline_check(ref_f32: np.ndarray, got: np.ndarray, what: str = "") -> Comparison:
    """BASELINE.json tolerance against the f32 oracle (see module doc)."""
    r = ref_f32.astype(np.float64)
    g = got.astype(np.float64)
    assert np.isfinite(g).all(), f"{what}: non-finite output"
    bound = 1e-2 + f16_ulp(ref_f32)
    diff = np.abs(g - r)
    worst = int(np.argmax(diff - bound)) if diff.size else 0
    c = compare(ref_f32, got, atol=1e-2, rtol=0.0)
    assert (diff <= bound).all(), (
        f"{what}: |d| {diff.flat[worst]:.4g} > bound {bound.flat[worst]:.4g} at flat index "
        f"{worst} (ref {r.flat[worst]:.6g}, got {g.flat[worst]:.6g}); {c}")
    assert c.rel_l2_percent <= 0.1, f"{what}: relative L2 {c.rel_l2_percent / 100:.3g} > 1e-3"
    return c


# --------------------------------------------------------------- golden data
_manifest = None
_arrays = None


def golden_manifest() -> dict:
    global _manifest
    if _manifest is None:
        _manifest = json.loads((GOLDEN / "micro_models.json").read_text())["models"]
    return _manifest


def golden_arrays():
    global _arrays
    if _arrays is None:
        _arrays = dict(np.load(GOLDEN / "micro_models.npz"))
    return _arrays


def golden_inputs(key: str) -> list[torch.Tensor]:
    """Inputs of a golden micro model, rebuilt with the reference harness's
    rule (integration_tests/stages/importing.py:218-241) and checked against
    the checksums recorded when the fixture was made."""
    entry = golden_manifest()[key]
    out = []
    for inp, ck in zip(entry["inputs"], entry["input_checksums"]):
        g = torch.Generator().manual_seed(int(inp["seed"]))
        dt = {"float16": torch.float16, "float32": torch.float32}[inp["dtype"]]
        t = torch.randn(inp["shape"], generator=g, dtype=torch.float32).to(dt)
        got = int(t.contiguous().view(torch.int16).to(torch.int64).sum())
        assert got == ck, f"{key}: regenerated input checksum {got} != {ck}"
        out.append(t)
    return out


def golden_expected(key: str):
    """(expected rows, row indices or None) of a golden micro model."""
    arrs = golden_arrays()
    rows = arrs.get(key + "__rows")
    return arrs[key], rows


def select_rows(full: np.ndarray, rows) -> np.ndarray:
    flat = full.reshape(-1, full.shape[-1])
    return flat if rows is None else flat[rows]
