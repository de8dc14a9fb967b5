"""Host-side checks of the int8-weight GEMM's work split
(hxb_plan_matmul_w8a16 enumerates the pieces with the kernel's own W8Work):
every (tile, K-block) is computed exactly once; a tile cut between CTAs is
finished by the CTA holding its first K-block, as the last piece of that CTA
(its activation stages then hold the partials), and that piece adds exactly
the CTAs holding the tile's other pieces, which follow it in CTA order; the
stream-K shares are equal to within one K-block. No GPU needed."""
from __future__ import annotations

import ctypes
from collections import defaultdict

import pytest

SMS = 148


def _plan(lib, M, N, K, sms=SMS):
    grid, dp = ctypes.c_int(), ctypes.c_int()
    count = ctypes.c_int64()
    assert lib.hxb_plan_matmul_w8a16(M, N, K, sms, ctypes.byref(grid), ctypes.byref(dp),
                                     None, 0, ctypes.byref(count)) == 0
    buf = (ctypes.c_int32 * (5 * count.value))()
    assert lib.hxb_plan_matmul_w8a16(M, N, K, sms, ctypes.byref(grid), ctypes.byref(dp), buf,
                                     count.value, ctypes.byref(count)) == 0
    rows = [tuple(buf[5 * i:5 * i + 5]) for i in range(count.value)]
    return grid.value, dp.value, rows


@pytest.mark.parametrize("M,K,N,kind", [
    (512, 4096, 4096, "sk"),        # decoder O projection: 64 tiles, stream-K over all
    (512, 11008, 4096, "sk"),       # decoder down projection
    (512, 4096, 12288, "sk"),       # decoder qkv
    (512, 4096, 22016, "hybrid"),   # decoder gate|up: two whole waves, stream-K tail
    (4096, 4096, 11008, "hybrid"),  # BASELINE cfg 2
    (300, 7992, 23008, "hybrid"),   # ragged M, K, N
    (100, 8192, 144, "sk"),         # 2 tiles cut into many pieces
    (200, 320, 528, "dp"),          # too little K to split
    (2048, 4096, 11008, "dp"),      # 4.65 waves: whole tiles win
])
def test_w8_schedule_covers_every_k_block_once(pkg, M, K, N, kind):
    lib = pkg._native.load()
    grid, dp, rows = _plan(lib, M, N, K)
    tiles_m, tiles_n, nkb = -(-M // 256), -(-N // 128), -(-K // 64)
    tiles = tiles_m * tiles_n
    assert grid == min(tiles, SMS) or kind != "dp"
    assert {"dp": dp == tiles, "sk": dp == 0, "hybrid": 0 < dp < tiles}[kind], (kind, dp, tiles)
    seen = defaultdict(int)
    by_cta = defaultdict(list)
    holders = defaultdict(set)
    for cta, tile, k0, k1, nadd in rows:
        assert 0 <= cta < grid and 0 <= tile < tiles and 0 <= k0 < k1 <= nkb
        for kb in range(k0, k1):
            seen[(tile, kb)] += 1
        by_cta[cta].append((tile, k0, k1, nadd))
        holders[tile].add(cta)
    assert len(seen) == tiles * nkb and set(seen.values()) == {1}
    # whole tiles first, round-robin; then at most one stream-K share per CTA
    sk_kb = []
    for cta, pcs in by_cta.items():
        whole = [p for p in pcs if p[0] < dp]
        assert [p[0] for p in whole] == list(range(cta, dp, grid))
        assert all(p[1] == 0 and p[2] == nkb and p[3] == 0 for p in whole)
        cut = pcs[len(whole):]
        assert all(p[0] >= dp for p in cut)
        sk_kb.append(sum(p[2] - p[1] for p in cut))
        for i, (tile, k0, k1, nadd) in enumerate(cut):
            if k0 == 0 and k1 < nkb:
                # finisher of a cut tile: the CTA's last piece, adding every
                # other holder of the tile, all later in CTA order
                assert i == len(cut) - 1
                others = holders[tile] - {cta}
                assert nadd == len(others) and others == set(range(cta + 1, cta + 1 + nadd))
            else:
                assert nadd == 0
                if k0 > 0:
                    assert i == 0  # a contributor piece opens the share
    if dp < tiles:
        assert max(sk_kb) - min(sk_kb) <= 1


@pytest.mark.parametrize("sms", [132, 160, 7])
@pytest.mark.parametrize("M,K,N", [(512, 4096, 22016), (4096, 4096, 11008), (300, 7992, 23008),
                                   (129, 4000, 272)])
def test_w8_schedule_other_sm_counts(pkg, sms, M, K, N):
    """The split invariants hold whatever the SM count the plan is made for."""
    lib = pkg._native.load()
    grid, dp, rows = _plan(lib, M, N, K, sms)
    tiles_m, tiles_n, nkb = -(-M // 256), -(-N // 128), -(-K // 64)
    tiles = tiles_m * tiles_n
    assert 1 <= grid <= sms and 0 <= dp <= tiles
    seen = defaultdict(int)
    last_piece = {}
    for cta, tile, k0, k1, nadd in rows:
        for kb in range(k0, k1):
            seen[(tile, kb)] += 1
        last_piece[cta] = (tile, k0, k1)
    assert len(seen) == tiles * nkb and set(seen.values()) == {1}
    for cta, tile, k0, k1, nadd in rows:
        if k0 == 0 and k1 < nkb:
            assert last_piece[cta] == (tile, k0, k1)


def test_w8_schedule_rejects_gemv_shapes(pkg):
    grid, dp = ctypes.c_int(), ctypes.c_int()
    assert pkg._native.load().hxb_plan_matmul_w8a16(16, 4096, 4096, SMS, ctypes.byref(grid),
                                            ctypes.byref(dp), None, 0, None) != 0
