"""Generates the golden fixtures under tests/golden/ from the reference itself.

Run in a container where the reference checkout is mounted (it is not needed
at test time):

    python tests/golden/make_golden.py /path/to/iree-hexagon-plugins

or with the checkout's path in HXB_REFERENCE_ROOT and no argument.

For every single-op micro model the reference's integration suite runs on the
hot path (integration_tests/models/micro/{matmul-*,hmx/*,attention-*}) this
  * reads the model's model.yaml (input shapes, dtypes, seeds, tolerances),
  * builds the inputs the way the reference's harness does
    (integration_tests/stages/importing.py:218-241: one
    torch.Generator().manual_seed(seed) per input, torch.randn in f32, cast
    to the input dtype),
  * imports the reference's own model.py and runs it eagerly on the CPU, which
    is exactly the reference's correctness oracle
    (integration_tests/stages/importing.py:293-301),
and stores the expected outputs. Inputs are not stored: tests regenerate them
with the same rule and check them against the stored input checksums. Large
outputs are stored as a fixed row sample plus whole-array sum and L2 norm.
"""
from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch
import yaml

HERE = Path(__file__).resolve().parent
OUT_NPZ = HERE / "micro_models.npz"
OUT_JSON = HERE / "micro_models.json"

MODELS = [
    "micro/matmul-1024x1024x1024-f16",
    "micro/attention-4x1024x128-f16",
    "micro/attention-cache-slice-f16",
    "micro/hmx/matmul-small-prime-17x19x23-f16",
    "micro/hmx/matmul-square-32x32x32-f16",
    "micro/hmx/matmul-ragged-k-64x64x65-f16",
    "micro/hmx/matmul-ragged-m-65x64x64-f16",
    "micro/hmx/matmul-ragged-n-64x65x64-f16",
    "micro/hmx/matmul-skinny-m-1x1024x1024-f16",
    "micro/hmx/matmul-tall-m-4096x32x256-f16",
    "micro/hmx/matmul-wide-n-32x4096x256-f16",
    "micro/hmx/matmul-deep-k-32x32x4096-f16",
    "micro/hmx/matmul-ragged-1537x1539x257-f16",
    "micro/hmx/matmul-rhs-transposed-1024x1024x1024-f16",
    "micro/hmx/batch-matmul-4x1024x1024x128-f16",
    "micro/hmx/matmul-square-512x512x512-f16",
]

FULL_LIMIT = 70_000   # outputs up to this many elements are stored whole
SAMPLE_ROWS = 24


def _dtype(name: str) -> torch.dtype:
    return {"float16": torch.float16, "float32": torch.float32}[name]


def generate_inputs(spec: dict) -> list[torch.Tensor]:
    """The reference harness's rule for `generator: normal` inputs."""
    out = []
    for inp in spec["inputs"]:
        assert inp["generator"] == "normal", inp
        g = torch.Generator().manual_seed(int(inp["seed"]))
        out.append(torch.randn(inp["shape"], generator=g, dtype=torch.float32)
                   .to(_dtype(inp["dtype"])))
    return out


def input_checksum(t: torch.Tensor) -> int:
    """Sum of the raw 16-bit patterns: detects any generator drift."""
    return int(t.contiguous().view(torch.int16).to(torch.int64).sum())


def sample_rows(n_rows: int) -> np.ndarray:
    rng = np.random.default_rng(1234)
    rows = np.unique(np.concatenate([[0, n_rows - 1], rng.integers(0, n_rows, SAMPLE_ROWS)]))
    return rows.astype(np.int64)


def main(ref_root: Path) -> None:
    models_root = ref_root / "integration_tests" / "models"
    arrays: dict[str, np.ndarray] = {}
    manifest = {}
    for name in MODELS:
        d = models_root / name
        spec = yaml.safe_load((d / "model.yaml").read_text())
        mspec = importlib.util.spec_from_file_location(f"refmodel_{len(manifest)}", d / "model.py")
        mod = importlib.util.module_from_spec(mspec)
        mspec.loader.exec_module(mod)
        model = mod.get_model()
        inputs = generate_inputs(spec)
        with torch.no_grad():
            out = model(*inputs)
        out_np = out.detach().cpu().numpy()
        key = name.replace("/", "__")
        entry = {
            "model": name,
            "inputs": spec["inputs"],
            "input_checksums": [input_checksum(t) for t in inputs],
            "tolerances": spec["tolerances"],
            "out_shape": list(out_np.shape),
            "out_dtype": str(out_np.dtype),
            "out_sum": float(out_np.astype(np.float64).sum()),
            "out_l2": float(np.linalg.norm(out_np.astype(np.float64))),
        }
        flat_rows = out_np.reshape(-1, out_np.shape[-1])
        if out_np.size <= FULL_LIMIT:
            arrays[key] = out_np
            entry["stored"] = "full"
        else:
            rows = sample_rows(flat_rows.shape[0])
            arrays[key + "__rows"] = rows
            arrays[key] = flat_rows[rows]
            entry["stored"] = "rows"
        manifest[key] = entry
        print(f"{name}: out {out_np.shape} {out_np.dtype} stored {entry['stored']}")
    np.savez_compressed(OUT_NPZ, **arrays)
    OUT_JSON.write_text(json.dumps({"torch": torch.__version__, "models": manifest}, indent=1))
    print(f"wrote {OUT_NPZ} ({OUT_NPZ.stat().st_size} bytes) and {OUT_JSON}")


if __name__ == "__main__":
    import os
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HXB_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py <reference checkout> (or set HXB_REFERENCE_ROOT)")
    main(Path(root))
