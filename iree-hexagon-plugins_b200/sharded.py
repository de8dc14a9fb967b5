"""Multi-GPU splits of the hot path (one process per GPU, torch.distributed
for the plumbing):

  * ShardedMatmul: one large f16 matmul split along N (BASELINE
    configuration 5: A [16384, 8192] x B [8192, 28672], 1/2/4/8 GPUs);
  * ShardedMatmulW8: the int8-weight matmul split along N (configuration 2:
    W [4096, 11008] in column shards of a multiple of 16 columns, 1376 per
    rank at 8 ranks), for the GEMM (M > 16) and the decode GEMV (M <= 16);
  * head_range: the fused attention split by heads (configuration 3: the
    B*H = 128 heads in contiguous groups; no collective).

One process per GPU, torch.distributed for the plumbing. Rank r of G holds A
(replicated) and the column shard B[:, cols_r] and computes C[:, cols_r] with
the tcgen05 GEMM. The gathered C is produced one of two ways:

  * "fused" (the product path): every rank keeps a full [M, N] output buffer;
    the ranks exchange CUDA IPC handles of these buffers once, and the GEMM's
    epilogue writes each output tile into all G buffers -- its own and, over
    NVLink, the peers' -- at the shard's columns
    (hxb_matmul_f16_allgather). A stream-ordered peer barrier
    (hxb_peer_barrier, flags in the same IPC-shared allocation) before the
    GEMM keeps a rank from overwriting a peer's C while that peer still reads
    the previous result, and one after it tells every rank that all peers'
    tiles have landed. No gather copy and no layout fix-up remain.
  * "nccl" (the baseline it is measured against): GEMM into a local shard,
    NCCL all-gather of the shards into [G, M, N/G], then the [G, M, n] ->
    [M, N] layout step (hxb_gather_column_blocks_f16).

The reference itself has no collectives (plugins/runtime/hexagon/channel.c:
55-56 returns IREE_STATUS_UNIMPLEMENTED). Peer memory here is plain CUDA IPC
(no NVLink multicast objects), and the TMA loads of the GEMM only ever read
this rank's own A and B.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native
from ._native import check


def shard_columns(N: int, world: int, rank: int, align: int = 8) -> tuple[int, int]:
    """[begin, end) of rank's column shard: N split into `world` contiguous
    blocks whose sizes are multiples of `align` (the last block takes the
    remainder), so every block starts on a 16-byte boundary."""
    if N % align:
        raise ValueError(f"N={N} must be a multiple of {align}")
    units = N // align
    base, extra = divmod(units, world)
    begin = (rank * base + min(rank, extra)) * align
    size = (base + (1 if rank < extra else 0)) * align
    return begin, begin + size


def exchange_peer_payloads(payload, *, group=None) -> list:
    """All-gathers one picklable payload per rank over `group` and returns the
    other ranks' payloads in rank order (this rank's own left out)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    infos = [None] * world
    dist.all_gather_object(infos, (rank, payload), group=group)
    assert [r for r, _ in infos] == list(range(world)), "ranks out of order"
    return [p for r, p in infos if r != rank]


def _stream_ptr(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def head_range(heads: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of the heads rank computes when `heads` independent
    attention heads (batch x heads flattened) are split over `world` ranks in
    contiguous groups that differ by at most one head."""
    base, extra = divmod(heads, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


class ShardedMatmul:
    """C = A @ B for B split along N across the ranks of `group` (one GPU
    per rank). Holds this rank's full output buffer and the peers' buffers
    opened through CUDA IPC."""

    ALIGN = 8  # columns per shard unit: 16-byte rows of f16 C

    def __init__(self, M: int, N: int, K: int, *, group=None, device=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("at most 8 ranks (one replica per peer in the epilogue)")
        self.M, self.N, self.K = M, N, K
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.cols = [shard_columns(N, self.world, r, self.ALIGN) for r in range(self.world)]
        self.begin, self.end = self.cols[self.rank]
        # the full output, then this rank's flag array of the peer barrier (one
        # uint32 per rank) in the same allocation, so one IPC handle maps both
        self._flag_off = (M * N * 2 + 255) // 256 * 256
        self._buf = torch.zeros(self._flag_off + 256, dtype=torch.uint8, device=self.device)
        self.out = self._buf[:M * N * 2].view(torch.float16).view(M, N)
        self.flags = self._buf[self._flag_off:].view(torch.int32)
        self._peer_storages: list = []  # (mapped pointer, offset) of opened peers
        self.peer_ptrs: list[int] = []
        self.flag_ptrs: list[int] = [self.flags.data_ptr()] * self.world
        self._epoch = 0
        if self.world > 1:
            self._open_peers()

    def _open_peers(self) -> None:
        # CUDA IPC: (handle, offset) of this rank's output, exchanged once over
        # the process group; each peer buffer is mapped into THIS rank's
        # device context (hxb_ipc_open), where the GEMM epilogue runs
        lib = _native.load()

        def handle_of(t):
            handle = ctypes.create_string_buffer(64)
            offset = ctypes.c_int64(0)
            check(lib.hxb_ipc_get_handle(t.data_ptr(), handle, ctypes.byref(offset)))
            return bytes(handle.raw), offset.value

        def open_handle(h, off):
            p = ctypes.c_void_p(0)
            check(lib.hxb_ipc_open(h, off, ctypes.byref(p)))
            self._peer_storages.append((p.value, off))
            return p.value
        payload = (self.rank, handle_of(self._buf))
        ptrs = []
        for peer, buf_h in exchange_peer_payloads(payload, group=self.group):
            base = open_handle(*buf_h)
            ptrs.append(base)
            self.flag_ptrs[peer] = base + self._flag_off
        self.peer_ptrs = ptrs

    def _sync(self) -> None:
        # stream-ordered barrier through peer memory (hxb_peer_barrier): every
        # rank's earlier work on its stream -- the GEMM and its remote stores
        # -- is done and visible before any rank continues on its stream
        if self.world > 1:
            self._epoch += 1
            arr = (ctypes.c_void_p * self.world)(*self.flag_ptrs)
            check(_native.load().hxb_peer_barrier(arr, self.world, self.rank, self._epoch,
                                                 _stream_ptr(self.out)))

    def fused(self, a: torch.Tensor, b_shard: torch.Tensor) -> torch.Tensor:
        """GEMM with the all-gather in its epilogue; returns the full C."""
        lib = _native.load()
        n = self.end - self.begin
        assert b_shard.shape == (self.K, n) and a.shape == (self.M, self.K)
        # peers may still be reading the previous result out of their buffers
        self._sync()
        reps = (ctypes.c_void_p * max(1, len(self.peer_ptrs)))(
            *[p + self.begin * 2 for p in self.peer_ptrs] or [0])
        check(lib.hxb_matmul_f16_allgather(
            a.data_ptr(), a.stride(0), b_shard.data_ptr(), b_shard.stride(0), 0,
            self.out.data_ptr() + self.begin * 2, reps if self.peer_ptrs else None,
            len(self.peer_ptrs), self.out.stride(0), self.M, n, self.K, _stream_ptr(a)))
        self._sync()
        return self.out

    def nccl(self, a: torch.Tensor, b_shard: torch.Tensor, *, shard_out: torch.Tensor,
             gathered: torch.Tensor) -> torch.Tensor:
        """Baseline: GEMM into the local shard, NCCL all-gather, layout step.
        Needs equal shards (N divisible by 8 * world). The shard's GEMM runs
        the tile plan the fused path runs (the persistent kernel: the
        all-gather epilogue has no split-K form), so both paths give the same
        bits."""
        lib = _native.load()
        n = self.end - self.begin
        sms = torch.cuda.get_device_properties(a.device).multi_processor_count
        bn, gm, sk, pair = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
        check(lib.hxb_plan_matmul_f16(self.M, n, self.K, 0, sms, ctypes.byref(bn),
                                      ctypes.byref(gm), ctypes.byref(sk), ctypes.byref(pair)))
        check(lib.hxb_matmul_f16_tiled(a.data_ptr(), a.stride(0), b_shard.data_ptr(),
                                       b_shard.stride(0), 0, shard_out.data_ptr(),
                                       shard_out.stride(0), 0, self.M, n, self.K, bn.value,
                                       gm.value, 1, pair.value, _stream_ptr(a)))
        if self.world > 1:
            self.dist.all_gather_into_tensor(gathered, shard_out, group=self.group)
            src = gathered
        else:
            src = shard_out
        check(lib.hxb_gather_column_blocks_f16(src.data_ptr(), self.out.data_ptr(), self.world,
                                               self.M, n, self.out.stride(0), _stream_ptr(a)))
        return self.out

    def close(self) -> None:
        lib = _native.load()
        for p, off in self._peer_storages:
            check(lib.hxb_ipc_close(p, off))
        self._peer_storages.clear()
        self.peer_ptrs = []


class ShardedMatmulW8(ShardedMatmul):
    """C[M, N] = (A[M, K] . W[K, N] int8) * scale[N] for W and scale split
    along N across the ranks of `group`. Rank r holds W[:, cols_r] (a
    contiguous [K, n_r] int8 tensor, n_r a multiple of 16 so its rows keep
    the 16-byte TMA pitch) and scale[cols_r], and computes C[:, cols_r]; the
    fused path writes each output tile to every rank's full C
    (hxb_matmul_w8a16_allgather)."""

    ALIGN = 16

    def __init__(self, M: int, N: int, K: int, *, group=None, device=None, workspace=None):
        super().__init__(M, N, K, group=group, device=device)
        self.workspace = workspace

    def fused(self, a: torch.Tensor, w_shard: torch.Tensor,
              s_shard: torch.Tensor) -> torch.Tensor:
        lib = _native.load()
        n = self.end - self.begin
        assert w_shard.shape == (self.K, n) and s_shard.numel() == n
        assert a.shape == (self.M, self.K)
        self._sync()
        reps = (ctypes.c_void_p * max(1, len(self.peer_ptrs)))(
            *[p + self.begin * 2 for p in self.peer_ptrs] or [0])
        ws = self.workspace
        check(lib.hxb_matmul_w8a16_allgather(
            a.data_ptr(), a.stride(0), w_shard.data_ptr(), w_shard.stride(0), s_shard.data_ptr(),
            self.out.data_ptr() + self.begin * 2, reps if self.peer_ptrs else None,
            len(self.peer_ptrs), self.out.stride(0), self.M, n, self.K,
            ws.data_ptr() if ws is not None else None,
            ws.numel() * ws.element_size() if ws is not None else 0, _stream_ptr(a)))
        self._sync()
        return self.out

    def nccl(self, a: torch.Tensor, w_shard: torch.Tensor, s_shard: torch.Tensor, *,
             shard_out: torch.Tensor, gathered: torch.Tensor) -> torch.Tensor:
        """Baseline: W8 matmul into the local shard, NCCL all-gather, layout
        step. Needs equal shards."""
        from .dispatch import matmul_w8a16
        lib = _native.load()
        n = self.end - self.begin
        matmul_w8a16(a, w_shard, s_shard, out=shard_out, workspace=self.workspace)
        if self.world > 1:
            self.dist.all_gather_into_tensor(gathered, shard_out, group=self.group)
            src = gathered
        else:
            src = shard_out
        check(lib.hxb_gather_column_blocks_f16(src.data_ptr(), self.out.data_ptr(), self.world,
                                               self.M, n, self.out.stride(0), _stream_ptr(a)))
        return self.out
