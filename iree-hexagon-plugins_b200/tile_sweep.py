"""Offline tile search for the f16 matmul dispatch (run on a B200).

The B200 counterpart of the reference's HMX tile search
(plugins/compiler/hexagon/CodeGen/Strategy/Planning/VTCMPlanning.cpp:186-260,
selectHmxTileSizes): where the reference ranks HMX-aligned tilings of each
matmul by a static cost (VTCM budget, DDR traffic, tile count), this sweep
MEASURES every tile plan the tcgen05 kernel offers -- the N extent of a
128-row output tile (64, 128, 256) and the L2 raster group -- on each shape
and keeps the fastest. The winners are written as the C table
csrc/tile_table.inc, which is compiled into libhxb200.so and consulted by the
planner before its cost model (planner.h), i.e. the search result is baked
into the executable, keyed by dispatch shape.

Default shapes: BASELINE configuration 5b, M, N, K in {128, 512, 2048, 8192}
(64 shapes, row-major B). Usage (on the GPU box):

    python iree-hexagon-plugins_b200/tile_sweep.py --out tile_table.inc --json sweep.json
"""
from __future__ import annotations

import argparse
import ctypes
import itertools
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))


def _time_graph(fn, iters: int) -> float:
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b) / iters)
    return best


def sweep(shapes, *, group_choices=(1, 4, 8, 16)) -> list[dict]:
    import torch
    import __graft_entry__ as ge
    pkg = ge.load_package()
    lib = pkg._native.load()
    dev = torch.device("cuda", 0)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    results = []
    for M, N, K in shapes:
        a = (torch.rand(M, K, device=dev) * 2 - 1).half()
        b = (torch.rand(K, N, device=dev) * 2 - 1).half()
        c = torch.empty(M, N, dtype=torch.float16, device=dev)
        flop = 2.0 * M * N * K
        iters = max(3, min(200, int(2e11 / flop)))
        tiles_m = (M + 127) // 128
        cands = []
        for bn in (64, 128, 256):
            for gm in sorted({min(g, tiles_m) for g in group_choices}):
                def run(bn=bn, gm=gm):
                    pkg._native.check(lib.hxb_matmul_f16_tiled(
                        a.data_ptr(), K, b.data_ptr(), N, 0, c.data_ptr(), N, 0, M, N, K, bn, gm,
                        torch.cuda.current_stream().cuda_stream))
                ms = _time_graph(run, iters)
                cands.append({"block_n": bn, "group_m": gm, "us": ms * 1e3,
                              "tflops": flop / ms / 1e9})
        best = min(cands, key=lambda r: r["us"])
        pbn, pgm = ctypes.c_int(0), ctypes.c_int(0)
        pkg._native.check(lib.hxb_plan_matmul_f16(M, N, K, 0, sms, ctypes.byref(pbn),
                                                  ctypes.byref(pgm)))
        planned = next(r for r in cands if r["block_n"] == pbn.value and
                       r["group_m"] == min(max(pgm.value, 1), tiles_m)) if any(
            r["block_n"] == pbn.value for r in cands) else None
        results.append({"M": M, "N": N, "K": K, "best": best, "candidates": cands,
                        "cost_model": planned})
        print(f"{M:5d} {N:5d} {K:5d}  best bn={best['block_n']:3d} gm={best['group_m']:2d} "
              f"{best['tflops']:7.1f} TF/s", flush=True)
    return results


def write_table(results, path: Path) -> None:
    lines = ["// {M, N, K, bmode, block_n, group_m} -- written by tile_sweep.py "
             "(measured on a B200; row-major B, bmode 0)"]
    for r in results:
        b = r["best"]
        lines.append(f"{{{r['M']}, {r['N']}, {r['K']}, 0, {b['block_n']}, {b['group_m']}}},")
    path.write_text("\n".join(lines) + "\n")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", type=Path, required=True, help="tile_table.inc to write")
    ap.add_argument("--json", type=Path, default=None)
    ap.add_argument("--sizes", type=int, nargs="+", default=[128, 512, 2048, 8192])
    args = ap.parse_args()
    shapes = list(itertools.product(args.sizes, args.sizes, args.sizes))
    results = sweep(shapes)
    write_table(results, args.out)
    if args.json:
        args.json.write_text(json.dumps(results, indent=1))


if __name__ == "__main__":
    main()
