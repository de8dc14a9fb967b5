"""Offline tile search for the f16 matmul dispatch (run on a B200).

The B200 counterpart of the reference's HMX tile search
(plugins/compiler/hexagon/CodeGen/Strategy/Planning/VTCMPlanning.cpp:186-260,
selectHmxTileSizes): where the reference ranks HMX-aligned tilings of each
matmul by a static cost (VTCM budget, DDR traffic, tile count), this sweep
MEASURES every tile plan the tcgen05 kernels offer -- the N extent of a
128-row output tile (64, 128, 256), the L2 raster group of the persistent
kernel, the K split over a thread-block cluster (2, 4, 8 CTAs per tile,
partials summed in distributed shared memory) and the CTA pair (256-row
tiles computed by cta_group::2 MMAs on two SMs, each loading half of the
operands; block_n 512 as two 256-column MMA chunks per A stage with one TMEM
accumulator) -- on each shape and keeps the fastest. The winners are written as the C table
csrc/tile_table.inc, which is compiled into libhxb200.so and consulted by the
planner before its cost model (planner.h), i.e. the search result is baked
into the executable, keyed by dispatch shape.

Default shapes: BASELINE configuration 5b, M, N, K in {128, 512, 2048, 8192}
(64 shapes, row-major B), plus configuration 1 (1024^3). Usage (on the GPU
box):

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
        # rotating input sets, together larger than the 126 MB L2, as the
        # bench times its dispatches: every dispatch reads its operands from
        # HBM
        per_set = 2 * (M * K + K * N + M * N)
        sets = max(2, min(64, -(-260_000_000 // per_set)))
        a = [(torch.rand(M, K, device=dev) * 2 - 1).half() for _ in range(sets)]
        b = [(torch.rand(K, N, device=dev) * 2 - 1).half() for _ in range(sets)]
        c = [torch.empty(M, N, dtype=torch.float16, device=dev) for _ in range(sets)]
        flop = 2.0 * M * N * K
        iters = max(3 * sets, min(200, int(2e11 / flop)))
        tiles_m = (M + 127) // 128
        kb = (K + 63) // 64
        cands = []
        for bn in (64, 128, 256, 512):
            tiles = tiles_m * ((N + bn - 1) // bn)
            plans = []
            if bn <= 256:
                plans += [(gm, 1, 1) for gm in sorted({min(g, tiles_m) for g in group_choices})]
                # split-K: clusters of 2, 4, 8 CTAs per tile, one wave, >= 2 K-blocks each
                plans += [(1, sk, 1) for sk in (2, 4, 8) if kb >= 2 * sk and tiles * sk <= sms]
            # CTA pairs: 256-row tiles on two SMs (block_n 128, 256, or 512 as two
            # MMA chunks sharing each A stage)
            if bn >= 128 and M > 128 and (bn <= 256 or N >= 512):
                pair_m = (M + 255) // 256
                plans += [(gm, 1, 2) for gm in sorted({min(g, pair_m) for g in group_choices})]
            for gm, sk, pair in plans:
                it = iter(range(1 << 30))

                def run(bn=bn, gm=gm, sk=sk, pair=pair):
                    i = next(it) % sets
                    pkg._native.check(lib.hxb_matmul_f16_tiled(
                        a[i].data_ptr(), K, b[i].data_ptr(), N, 0, c[i].data_ptr(), N, 0, M, N,
                        K, bn, gm, sk, pair, torch.cuda.current_stream().cuda_stream))
                ms = _time_graph(run, iters)
                cands.append({"block_n": bn, "group_m": gm, "split_k": sk, "cta_pair": pair,
                              "us": ms * 1e3, "tflops": flop / ms / 1e9})
        best = min(cands, key=lambda r: r["us"])
        pbn, pgm, psk, ppair = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
        pkg._native.check(lib.hxb_plan_matmul_f16(M, N, K, 0, sms, ctypes.byref(pbn),
                                                  ctypes.byref(pgm), ctypes.byref(psk),
                                                  ctypes.byref(ppair)))
        rows_m = (M + 128 * ppair.value - 1) // (128 * ppair.value)
        planned = next((r for r in cands if r["block_n"] == pbn.value and
                        r["split_k"] == psk.value and r["cta_pair"] == ppair.value and
                        (psk.value > 1 or r["group_m"] == min(max(pgm.value, 1), rows_m))),
                       None)
        results.append({"M": M, "N": N, "K": K, "best": best, "candidates": cands,
                        "table_plan": planned, "input_sets": sets})
        del a, b, c
        torch.cuda.empty_cache()
        print(f"{M:5d} {N:5d} {K:5d}  best bn={best['block_n']:3d} gm={best['group_m']:2d} "
              f"sk={best['split_k']} pair={best['cta_pair']} {best['tflops']:7.1f} TF/s",
              flush=True)
    return results


def write_table(results, path: Path) -> None:
    lines = ["// {M, N, K, bmode, block_n, group_m, split_k, cta_pair} -- written by "
             "tile_sweep.py (measured on a B200; row-major B, bmode 0)"]
    for r in results:
        b = r["best"]
        lines.append(f"{{{r['M']}, {r['N']}, {r['K']}, 0, {b['block_n']}, {b['group_m']}, "
                     f"{b['split_k']}, {b.get('cta_pair', 1)}}},")
    path.write_text("\n".join(lines) + "\n")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", type=Path, required=True, help="tile_table.inc to write")
    ap.add_argument("--json", type=Path, default=None)
    ap.add_argument("--sizes", type=int, nargs="+", default=[128, 512, 2048, 8192])
    ap.add_argument("--no-cfg1", dest="with_cfg1", action="store_false",
                    help="leave out configuration 1 (1024^3)")
    args = ap.parse_args()
    shapes = list(itertools.product(args.sizes, args.sizes, args.sizes))
    if args.with_cfg1:
        shapes.append((1024, 1024, 1024))
    results = sweep(shapes)
    write_table(results, args.out)
    if args.json:
        args.json.write_text(json.dumps(results, indent=1))


if __name__ == "__main__":
    main()
