"""Host logic of the N-sharded matmul: the column
split and the once-per-run exchange of peer-buffer handles, run as gloo ranks
on the CPU (world size 2, 3 and 8)."""
from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp


def _shard_columns():
    import __graft_entry__ as ge
    return ge.load_package().sharded.shard_columns


@pytest.mark.parametrize("N,world", [(28672, 1), (28672, 2), (28672, 8), (11008, 3), (64, 8), (8, 1)])
def test_shards_cover_n_exactly_aligned(N, world):
    shard_columns = _shard_columns()
    cols = [shard_columns(N, world, r) for r in range(world)]
    assert cols[0][0] == 0 and cols[-1][1] == N
    for (b0, e0), (b1, e1) in zip(cols, cols[1:]):
        assert e0 == b1
    sizes = [e - b for b, e in cols]
    assert all(b % 8 == 0 for b, _ in cols) and all(s % 8 == 0 for s in sizes)
    assert max(sizes) - min(sizes) <= 8


def test_cfg5_shards_are_equal_and_tile_aligned():
    shard_columns = _shard_columns()
    for world in (1, 2, 4, 8):
        sizes = {e - b for b, e in (shard_columns(28672, world, r) for r in range(world))}
        assert sizes == {28672 // world}
        assert (28672 // world) % 256 == 0  # whole 256-column GEMM tiles


def test_unaligned_n_rejected():
    with pytest.raises(ValueError):
        _shard_columns()(100, 2, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, results):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        import __graft_entry__ as ge
        sharded = ge.load_package().sharded
        got = sharded.exchange_peer_payloads({"rank": rank, "handle": bytes([rank]) * 64})
        results[rank] = [g["rank"] for g in got], [g["handle"][0] for g in got]
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 8])
def test_peer_handle_exchange_gloo(world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, results))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        for r in range(world):
            peers, first_bytes = results[r]
            assert peers == [x for x in range(world) if x != r]
            assert first_bytes == peers
