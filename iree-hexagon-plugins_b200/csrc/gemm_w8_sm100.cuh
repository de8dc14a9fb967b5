// Int8-weight GEMM for sm_100a: C[M,N] f16 = (A[M,K] f16 . W[K,N] int8) * scale[N] (+ R).
//
// The kernel computes the transposed product D[n, m] = sum_k W[k, n] A[m, k]
// on the tensor core so that the dequantised weights never pass through
// shared memory a second time:
//   * TMA lands the raw int8 weight tile [64 k][128 n] (8 KB, 128-byte
//     swizzle) and the activation tile [256 m][64 k] f16 (32 KB) in two
//     independent rings;
//   * eight converter warps transpose the int8 tile on its way out of shared
//     memory (ldmatrix.trans), convert it exactly to f16 (|w| <= 127) in
//     registers and write it into TMEM with tcgen05.st, where it is the A
//     operand (M = 128 weight columns) of tcgen05.mma. The converters form two
//     groups of four that take alternate K-blocks, so two blocks are in
//     conversion at once and the latency of one (shared-memory load, TMEM
//     store, wait) is hidden behind the other;
//   * one thread issues tcgen05.mma (A from TMEM, B = activations from shared
//     memory, N = 256 activation rows) into a 256-column f32 TMEM
//     accumulator. N = 256 amortises each converted weight block over the
//     most activation rows one MMA takes; measured on B200 it beats two
//     double-buffered 192-column accumulators (366 -> 317 us on the 4096 x
//     4096 x 11008 dispatch). TMEM then has no room for a second accumulator,
//     so the MMA waits while the epilogue drains the tile; the TMA and the
//     converters keep running meanwhile and fill up to kW8SA converted
//     K-blocks for the next tile;
//   * four epilogue warps read the accumulator back and apply the
//     per-column scale once (it factors out of the K sum). The tile is
//     packed to f16 into a 64 KB shared-memory staging tile, the accumulator
//     is released to the MMA as soon as it is read, and one thread writes C
//     with two TMA stores that overlap the next tile's main loop. A residual
//     is loaded by TMA into the same staging tile while the main loop runs
//     (same boxes and swizzle as the output, so each thread reads its
//     residual pair where it then writes its result: one f16 rounding of
//     acc * s + r).
//   * Measured decomposition of the 4096 x 4096 x 11008 dispatch on B200
//     (307 us before the staging was sized as below): tensor pipe alone
//     ~167 us; with TMA feeding but no conversion and no epilogue 234 us;
//     the int8 conversion adds ~62 us, the epilogue ~11 us.
// Shared-memory traffic per k-block is the int8 tile (written by TMA, read
// once by the converters) plus the activation tile (written by TMA, read by
// the tensor core); the f16 weights live only in registers and TMEM.
//
// Work split. Data-parallel: CTA b owns whole output tiles b, b + grid, ...
// Stream-K (args.streamk): the tiles x K-blocks iteration space of the tiles
// from args.sk_dp_tiles on (all of them, or the last partial wave after
// whole-tile waves) is cut into `grid` equal contiguous shares, so every SM
// gets the same number of MMAs whatever the tile count. A tile cut between CTAs is summed as follows: the
// CTA holding the tile's first K-block (it processes that piece LAST, at the
// end of its share) finalises it; every other CTA holding a piece of the
// tile holds it FIRST, writes its f32 partial accumulator to
// args.sk_partials[cta] and raises args.sk_flags[cta][quarter]. The finaliser
// brings the partials of each quarter into the (then idle) activation stages
// with 1-D bulk copies and adds them into its TMEM accumulator in CTA order
// (deterministic), then runs the normal epilogue and clears the flags, so the
// flag array is all zero again when the kernel ends. No CTA waits on a
// lower-numbered CTA, and every wait is bounded.
//
// Roles (512 threads, one CTA per SM, persistent):
//   warp 0        TMA producer (one lane)
//   warp 1        TMEM owner + MMA issuer (one lane)
//   warps 2-3     idle
//   warps 4-11    int8 -> f16 converters: warp 4 + 4 g + q converts TMEM lane
//                 quarter q (16-column chunks 2q, 2q + 1) of the CTA's
//                 K-blocks g, g + 2, g + 4, ...
//   warps 12-15   epilogue
// TMEM: the accumulator in columns [0, 256), kW8SA = 8 converted weight
// stages of 32 columns from column 256. Shared memory: 4 activation stages
// (32 KB), 4 int8 stages (8 KB), the 64 KB output staging tile.
#pragma once

#include "gemm_sm100.cuh"
#include "w8_tmem.cuh"

namespace hxb {

constexpr int kW8BN = 128;  // weight columns per tile (MMA M, TMEM lanes)
constexpr int kW8BM = 256;  // activation rows per tile (MMA N)
constexpr int kW8Acc = 1;   // TMEM accumulators (kW8Acc * kW8BM + 32 * kW8SA <= 512)
constexpr int kW8SX = 4;    // activation stages
constexpr int kW8SW = 4;    // int8 weight stages
constexpr int kW8SA = 8;    // TMEM weight stages
constexpr int kW8ACol = kW8Acc * kW8BM;  // first TMEM column of the weight stages
static_assert(kW8ACol + 32 * kW8SA <= 512, "TMEM budget");
constexpr int kW8Threads = 16 * 32;
constexpr int kW8ConvGroups = 2;    // converter groups (alternate K-blocks)
constexpr int kW8ConvWarps = 4 * kW8ConvGroups;
constexpr int kW8EpiWarps = 4;
// f32 partial accumulator of one tile: 128 x 256 floats
constexpr int kW8PartialFloats = kW8BN * kW8BM;
// Stream-K workspace: flags [CTA][quarter] (int, up to 256 CTAs) in the first
// kW8FlagBytes, then one partial accumulator per CTA.
constexpr size_t kW8FlagBytes = 4096;
constexpr int kW8MaxStreamKCtas = (int)(kW8FlagBytes / 16);
// Smallest stream-K share, in K-blocks: a shorter share costs more in partial
// traffic than it gains in balance.
constexpr int kW8MinShare = 8;

struct W8Smem {
  static constexpr int kXBytes = kW8BM * kBK * 2;  // 32 KB
  static constexpr int kWBytes = kW8BN * kBK;      // 8 KB
  // f16 output tile [256 m][128 n] as two TMA-store boxes [256 m][64 n]
  // (128-byte rows, 128-byte swizzle)
  static constexpr int kBoxBytes = kW8BM * 128;    // 32 KB
  static constexpr int kOffX = 0;
  static constexpr int kOffW = kOffX + kW8SX * kXBytes;
  static constexpr int kOffStage = kOffW + kW8SW * kWBytes;
  static constexpr int kOffBar = kOffStage + 2 * kBoxBytes;
  // x_full, x_empty [SX]; w_full, w_empty [SW]; a_full, a_empty [SA];
  // t_full[2], t_empty[2], drain; fix_full[4 epilogue warps][2] (partial
  // segments of a cut tile, landing in the activation stages once the last
  // main loop is done); r_full (residual tile in the staging tile)
  static constexpr int kNumBars = 2 * kW8SX + 2 * kW8SW + 2 * kW8SA + 5 + 2 * kW8EpiWarps + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

// Position in an S-deep ring of mbarrier-guarded slots: slot index and the
// parity of the phase the slot is in.
template <int S>
struct RingCursor {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void advance() {
    if (++slot == S) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// Bounded wait for the last min(issued, S) bulk copies of a ring (cursor `c`
// points one past the most recent issue).
template <int S>
__device__ __forceinline__ void drain_ring(uint64_t* full, RingCursor<S> c, int issued) {
  for (int i = 0; i < issued && i < S; ++i) {
    if (c.slot == 0) {
      c.slot = S - 1;
      c.phase ^= 1u;
    } else {
      --c.slot;
    }
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait(&full[c.slot], c.phase) && globaltimer_ns() - t0 < kWaitLimitNs) {
    }
  }
}

// One piece of work: K-blocks [k0, k1) of output tile `tile`.
struct W8Seg {
  int tile, k0, k1;
};

// The sequence of pieces one work unit (a CTA) processes; the same for all
// roles of the unit (and for the host-side schedule query). Units are numbered 0 .. nunits-1. Tiles [0, dp_tiles)
// are whole tiles dealt round-robin (unit u takes u, u + nunits, ...); the
// K-blocks of tiles [dp_tiles, num_tiles) are cut into nunits equal
// contiguous stream-K shares, which each unit processes after its whole
// tiles (dp_tiles = num_tiles without stream-K, 0 for stream-K over all
// tiles). Positions count iterations: tile * num_kb + K-block.
struct W8Work {
  int num_kb, num_tiles, dp_tiles, unit, nunits;
  long long sk_base, sk_total, it0, it1;

  // First iteration of unit c's stream-K share (sk_total >= nunits when
  // there is a stream-K part, so no share is empty).
  __host__ __device__ __forceinline__ long long share_begin(int c) const {
    return sk_base + sk_total * c / nunits;
  }
  __host__ __device__ __forceinline__ void init(const GemmArgs& a, int unit_, int nunits_) {
    unit = unit_;
    nunits = nunits_;
    num_kb = (a.K + kBK - 1) / kBK;
    num_tiles = a.tiles_m * a.tiles_n;
    dp_tiles = a.streamk ? a.sk_dp_tiles : num_tiles;
    sk_base = (long long)dp_tiles * num_kb;
    sk_total = (long long)(num_tiles - dp_tiles) * num_kb;
    it0 = share_begin(unit);
    it1 = share_begin(unit + 1);
  }
  __host__ __device__ __forceinline__ long long first() const {
    return unit < dp_tiles ? (long long)unit * num_kb : it0;
  }
  // K-blocks this unit processes in all.
  __host__ __device__ __forceinline__ long long kb_count() const {
    const long long nt = unit < dp_tiles ? (dp_tiles - 1 - unit) / nunits + 1 : 0;
    return nt * num_kb + (it1 - it0);
  }
  __host__ __device__ __forceinline__ bool next(long long& pos, W8Seg& s) const {
    if (pos < sk_base) {
      s.tile = (int)(pos / num_kb);
      s.k0 = 0;
      s.k1 = num_kb;
      pos += (long long)nunits * num_kb;
      if (pos >= sk_base) pos = it0;
      return true;
    }
    if (pos >= it1) return false;
    s.tile = (int)(pos / num_kb);
    s.k0 = (int)(pos - (long long)s.tile * num_kb);
    const long long k1 = s.k0 + (it1 - pos);
    s.k1 = k1 < num_kb ? (int)k1 : num_kb;
    pos += s.k1 - s.k0;
    return true;
  }
  // Units whose partial accumulators the finalising piece `sg` adds:
  // [*lo, *hi) (empty unless sg is cut and holds the tile's first K-block).
  __host__ __device__ __forceinline__ void contributors(const W8Seg& sg, int* lo, int* hi) const {
    *lo = *hi = unit + 1;
    if (sg.k0 == 0 && sg.k1 < num_kb) {
      const long long tile_end = (long long)(sg.tile + 1) * num_kb;
      while (*hi < nunits && share_begin(*hi) < tile_end) ++*hi;
    }
  }
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *flag == 1 (raised by another CTA of this grid).
__device__ __forceinline__ bool wait_flag(const int* flag, const FailState& fs) {
  if (ld_acquire_gpu(flag) == 1) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i) {
      if (ld_acquire_gpu(flag) == 1) return true;
      __nanosleep(64);
    }
    if (*fs.abort) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_failure(fs);
      return false;
    }
  }
}

// float4 index of (epilogue quarter q, half h, 32-column chunk c, rep r, lane)
// inside one CTA's partial accumulator image: the float4 a thread writes for
// one tcgen05.ld repetition, so each warp access is 512 contiguous bytes.
__device__ __forceinline__ int w8_partial_index(int q, int h, int c, int r, int lane) {
  return (((q * 2 + h) * (kW8BM / 32) + c) * 4 + r) * 32 + lane;
}

// Contributor epilogue (epilogue warp q, lane t): a piece that does not hold
// its tile's first K-block writes its raw f32 accumulator (TMEM at
// `acc_tmem`, waited for on t_full, phase `parity`) to partial slot
// `self_slot` and raises that slot's flag for quarter q. tcgen05.ld.16x256b
// gives lane t, for repetition r, the accumulator values of TMEM lanes t/4 and
// t/4 + 8 of a 16-lane group at columns 8r + 2(t%4), +1; each warp store is
// 512 contiguous bytes (w8_partial_index). Returns false after a timeout.
__device__ __forceinline__ bool w8_write_partial(const GemmArgs& args, const FailState& fs,
                                                 uint64_t* t_full, uint32_t parity,
                                                 uint32_t acc_tmem, int q, int t, int self_slot) {
  const bool ready = mbar_wait(t_full, parity, fs);
  if (!__all_sync(0xffffffffu, ready)) return false;
  tc_fence_after();
  float4* part =
      reinterpret_cast<float4*>(args.sk_partials) + (size_t)self_slot * (kW8PartialFloats / 4);
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    const uint32_t taddr = acc_tmem + ((uint32_t)(16 * (2 * q + h)) << 16);
#pragma unroll 1
    for (int c = 0; c < kW8BM / 32; c += 4) {
      // four 32-column chunks per TMEM round trip
      uint32_t r[4][16];
#pragma unroll
      for (int u = 0; u < 4; ++u) tmem_ld_16x256b_x4(taddr + 32 * (c + u), r[u]);
      tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int rep = 0; rep < 4; ++rep)
          __stcg(part + w8_partial_index(q, h, c + u, rep, t),
                 make_float4(__uint_as_float(r[u][4 * rep]), __uint_as_float(r[u][4 * rep + 1]),
                             __uint_as_float(r[u][4 * rep + 2]),
                             __uint_as_float(r[u][4 * rep + 3])));
    }
  }
  // publish: every lane's stores, then the flag of this quarter
  __threadfence();
  __syncwarp();
  if (t == 0) st_release_gpu(args.sk_flags + 4 * self_slot + q, 1);
  return true;
}

// Finaliser of a tile cut between CTAs (epilogue warp q, lane `lane`): adds
// the f32 partial accumulators that CTAs c_lo .. c_hi - 1 wrote for this tile
// into this CTA's TMEM accumulator at `acc_tmem`, lane quarter q, in CTA
// order, then clears their flags. Called after the accumulator is complete.
// The segments (CTA, half h) of the quarter, 16 KB each, come in by 1-D bulk
// copies into the warp's two 16 KB buffers `buf` (shared memory that the
// CTA's last main loop no longer uses) under bars[0..1], one segment ahead of
// the one being added; each 32 accumulator columns cost a TMEM load, 32 adds
// from shared memory and a TMEM store. Returns false (every lane agreeing)
// after a timeout, once the copies it issued have landed.
__device__ __forceinline__ bool w8_add_partials(const GemmArgs& args, const FailState& fs,
                                                uint8_t* buf, uint64_t* bars, uint32_t acc_tmem,
                                                int q, int lane, int c_lo, int c_hi) {
  constexpr uint32_t kSegBytes = kW8PartialFloats / 8 * sizeof(float);
  bool ready = true;
  for (int c2 = c_lo; c2 < c_hi && ready; ++c2) ready = wait_flag(args.sk_flags + 4 * c2 + q, fs);
  if (!__all_sync(0xffffffffu, ready)) return false;
  tc_fence_after();
  const int nc = c_hi - c_lo, S = 2 * nc;
  const uint8_t* part = reinterpret_cast<const uint8_t*>(args.sk_partials);
  // segment s: half s / nc of CTA c_lo + s % nc (partial layout of
  // w8_partial_index: 8 segments (q, h) of 16 KB per CTA)
  auto src = [&](int s) {
    return part + ((size_t)(c_lo + s % nc) * 8 + (size_t)(2 * q + s / nc)) * kSegBytes;
  };
  if (lane == 0) {
    fence_proxy_async_global();
    for (int s = 0; s < 2 && s < S; ++s) {
      mbar_arrive_expect_tx(&bars[s], kSegBytes);
      bulk_load_1d(buf + s * kSegBytes, src(s), kSegBytes, &bars[s]);
    }
  }
  int s = 0;
  bool ok = true;
  for (; s < S; ++s) {
    const int b = s & 1;
    ok = mbar_wait(&bars[b], (uint32_t)(s >> 1) & 1u, fs);
    if (!__all_sync(0xffffffffu, ok)) {
      ok = false;
      break;
    }
    const float4* p = reinterpret_cast<const float4*>(buf + b * kSegBytes);
    const uint32_t taddr = acc_tmem + ((uint32_t)(16 * (2 * q + s / nc)) << 16);
#pragma unroll 1
    for (int c = 0; c < kW8BM / 32; c += 4) {
      // four 32-column chunks per TMEM round trip
      uint32_t r[4][16];
#pragma unroll
      for (int u = 0; u < 4; ++u) tmem_ld_16x256b_x4(taddr + 32 * (c + u), r[u]);
      tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int rep = 0; rep < 4; ++rep) {
          const float4 v = p[((c + u) * 4 + rep) * 32 + lane];
          r[u][4 * rep] = __float_as_uint(__uint_as_float(r[u][4 * rep]) + v.x);
          r[u][4 * rep + 1] = __float_as_uint(__uint_as_float(r[u][4 * rep + 1]) + v.y);
          r[u][4 * rep + 2] = __float_as_uint(__uint_as_float(r[u][4 * rep + 2]) + v.z);
          r[u][4 * rep + 3] = __float_as_uint(__uint_as_float(r[u][4 * rep + 3]) + v.w);
        }
#pragma unroll
      for (int u = 0; u < 4; ++u) tmem_st_16x256b_x4(taddr + 32 * (c + u), r[u]);
    }
    tmem_wait_st();
    // every lane has read buffer b: refill it with segment s + 2
    __syncwarp();
    if (lane == 0 && s + 2 < S) {
      mbar_arrive_expect_tx(&bars[b], kSegBytes);
      bulk_load_1d(buf + b * kSegBytes, src(s + 2), kSegBytes, &bars[b]);
    }
  }
  if (!ok) {
    // segments s and s + 1 may still be landing in the buffers
    if (lane == 0) {
      const unsigned long long t0 = globaltimer_ns();
      for (int s2 = s; s2 < S && s2 < s + 2; ++s2)
        while (!mbar_try_wait(&bars[s2 & 1], (uint32_t)(s2 >> 1) & 1u) &&
               globaltimer_ns() - t0 < kWaitLimitNs) {
        }
    }
    __syncwarp();
    return false;
  }
  tc_fence_before();
  if (lane == 0)
    for (int c2 = c_lo; c2 < c_hi; ++c2) args.sk_flags[4 * c2 + q] = 0;
  return true;
}

// Staged epilogue of epilogue warp q (lane t): reads the warp's accumulator
// quarter (TMEM at `acc_tmem`, lanes 32q .. 32q + 31) four 32-column chunks per
// TMEM round trip (two with a residual, whose pairs take the registers of the
// other two), applies the column scales (plus the residual pair that
// sits at the same staging address when RESID: one f16 rounding of
// acc * s + r) and writes f16 pairs into the staging box `box` of its quarter
// pair. Lane t writes the pair (n, n + 1), n = 16 (2q + h) + 2 (t >> 2), of
// row m = 32 c + 8 rep + 2 (t & 3) + j at 16-byte chunk
// (4 (q & 1) + 2 h + (t >> 4)) ^ (m & 7), word (t >> 2) & 3 of the 128-byte
// row m: the 32 lanes of each access hit 32 different banks.
// All-gather epilogue: the staged f16 tile (two 128B-swizzled boxes of 64
// columns x 256 rows; 16-byte chunk c of row m at (c ^ (m & 7)) * 16) is also
// written to the other ranks' copies of the output, dests[1..ndests), at the
// same row and column, with 16-byte stores over NVLink. Consecutive threads
// take consecutive chunks of a row (256 contiguous bytes per row and peer).
// Rows past M and columns past N (the shard's width, a multiple of 8) are
// skipped, as the local TMA store clips them. Every epilogue thread reads
// its chunks before it reaches the next tile's barrier, so the staging tile
// is free by then.
template <class Args>
__device__ __forceinline__ void w8_store_replicas(const Args& args, const uint8_t* stage,
                                                  int tm, int tn) {
  const int tid = threadIdx.x - 32 * (4 + kW8ConvWarps);
  const int rows = min(kW8BM, args.M - tm * kW8BM);
  const int cols = min(kW8BN, args.N - tn * kW8BN);
#pragma unroll 1
  for (int idx = tid; idx < rows * 16; idx += 32 * kW8EpiWarps) {
    const int m = idx >> 4, c16 = idx & 15;
    if (c16 * 8 >= cols) continue;
    const uint4 v = *reinterpret_cast<const uint4*>(stage + (c16 >> 3) * (kW8BM * 128) +
                                                   m * 128 + (((c16 & 7) ^ (m & 7)) << 4));
    const long long off =
        (long long)(tm * kW8BM + m) * args.ldc + (long long)tn * kW8BN + c16 * 8;
    for (int d = 1; d < args.ndests; ++d)
      *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(args.dests[d]) + off) = v;
  }
}

template <bool RESID>
__device__ __forceinline__ void w8_stage_tile(uint32_t acc_tmem, uint8_t* box, int q, int lane,
                                              const float (&sc)[2][2]) {
  constexpr int CH = RESID ? 2 : 4;  // 32-column chunks per TMEM round trip
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    const uint32_t taddr = acc_tmem + ((uint32_t)(16 * (2 * q + h)) << 16);
    const float s0 = h ? sc[1][0] : sc[0][0], s1 = h ? sc[1][1] : sc[0][1];
    const int chunk0 = 4 * (q & 1) + 2 * h + (lane >> 4);
    const int word = 4 * ((lane >> 2) & 3);
#pragma unroll 1
    for (int c = 0; c < kW8BM / 32; c += CH) {
      uint32_t r[CH][16];
#pragma unroll
      for (int u = 0; u < CH; ++u) tmem_ld_16x256b_x4(taddr + 32 * (c + u), r[u]);
      uint32_t res[CH][8];
      if (RESID) {
#pragma unroll
        for (int u = 0; u < CH; ++u)
#pragma unroll
          for (int rep = 0; rep < 4; ++rep)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int m = 32 * (c + u) + 8 * rep + 2 * (lane & 3) + j;
              res[u][2 * rep + j] = *reinterpret_cast<const uint32_t*>(
                  box + m * 128 + ((chunk0 ^ (m & 7)) << 4) + word);
            }
      }
      tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < CH; ++u)
#pragma unroll
        for (int rep = 0; rep < 4; ++rep)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int m = 32 * (c + u) + 8 * rep + 2 * (lane & 3) + j;
            const float a0 = __uint_as_float(r[u][4 * rep + j]);
            const float a1 = __uint_as_float(r[u][4 * rep + 2 + j]);
            uint32_t v;
            if (RESID) {
              const float2 rv =
                  __half22float2(*reinterpret_cast<const __half2*>(&res[u][2 * rep + j]));
              v = pack_half2(__fmaf_rn(a0, s0, rv.x), __fmaf_rn(a1, s1, rv.y));
            } else {
              v = pack_half2(a0 * s0, a1 * s1);
            }
            *reinterpret_cast<uint32_t*>(box + m * 128 + ((chunk0 ^ (m & 7)) << 4) + word) = v;
          }
    }
  }
}

__global__ void __launch_bounds__(kW8Threads, 1)
    gemm_w8_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmW,
                         const __grid_constant__ CUtensorMap tmC,
                         const __grid_constant__ CUtensorMap tmR, const GemmArgs args) {
  using L = W8Smem;
  // D[128 n x 256 m] += W^T (TMEM, K-major) . A^T (shared, K-major)
  constexpr uint32_t kIdesc = make_idesc_f16(kW8BN, kW8BM, 0, 0);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* x_full = bars;
  uint64_t* x_empty = x_full + kW8SX;
  uint64_t* w_full = x_empty + kW8SX;
  uint64_t* w_empty = w_full + kW8SW;
  uint64_t* a_full = w_empty + kW8SW;
  uint64_t* a_empty = a_full + kW8SA;
  uint64_t* t_full = a_empty + kW8SA;
  uint64_t* t_empty = t_full + 2;
  uint64_t* drain = t_empty + 2;
  uint64_t* fix_full = drain + 1;
  uint64_t* r_full = fix_full + 2 * kW8EpiWarps;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  W8Work work;
  work.init(args, blockIdx.x, gridDim.x);
  const FailState fs{abort_flag, args.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < kW8SX; ++s) { mbar_init(&x_full[s], 1); mbar_init(&x_empty[s], 1); }
    for (int s = 0; s < kW8SW; ++s) { mbar_init(&w_full[s], 1); mbar_init(&w_empty[s], 4); }
    for (int s = 0; s < kW8SA; ++s) { mbar_init(&a_full[s], 4); mbar_init(&a_empty[s], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], kW8EpiWarps);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 2 * kW8EpiWarps; ++i) mbar_init(&fix_full[i], 1);
    mbar_init(r_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmC);
    if (args.C_init) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      RingCursor<kW8SX> cx;
      RingCursor<kW8SW> cw;
      int issued_x = 0, issued_w = 0;
      bool ok = true;
      long long pos = work.first();
      W8Seg sg;
      while (ok && work.next(pos, sg)) {
        int tm, tn;
        tile_coords(sg.tile, args, tm, tn);
        for (int kb = sg.k0; kb < sg.k1; ++kb) {
          if (!mbar_wait(&w_empty[cw.slot], cw.phase ^ 1, fs)) { ok = false; break; }
          mbar_arrive_expect_tx(&w_full[cw.slot], L::kWBytes);
          tma_load_2d(smem + L::kOffW + cw.slot * L::kWBytes, &tmW, &w_full[cw.slot],
                      tn * kW8BN, kb * kBK);
          cw.advance();
          ++issued_w;
          if (!mbar_wait(&x_empty[cx.slot], cx.phase ^ 1, fs)) { ok = false; break; }
          mbar_arrive_expect_tx(&x_full[cx.slot], L::kXBytes);
          tma_load_2d(smem + L::kOffX + cx.slot * L::kXBytes, &tmA, &x_full[cx.slot],
                      kb * kBK, tm * kW8BM);
          cx.advance();
          ++issued_x;
        }
      }
      drain_ring<kW8SW>(w_full, cw, issued_w);
      drain_ring<kW8SX>(x_full, cx, issued_x);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      RingCursor<kW8SX> cx;
      RingCursor<kW8SA> ca;
      int tl = 0;
      bool ok = true, issued_any = false;
      long long pos = work.first();
      W8Seg sg;
      // activation descriptors built once; a slot or a K step moves only the
      // start-address field (address >> 4 in 14 bits)
      const uint64_t x_desc0 =
          make_smem_desc(smem_u32(smem + L::kOffX), 16, 1024, kLayoutSwizzle128);
      while (ok && work.next(pos, sg)) {
        const int acc = tl % kW8Acc;
        if (!mbar_wait(&t_empty[acc], (uint32_t)((tl / kW8Acc) & 1) ^ 1, fs)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + kW8BM * acc;
        for (int kb = sg.k0; kb < sg.k1; ++kb) {
          const int sx = cx.slot, sa = ca.slot;
          if (!mbar_wait(&x_full[sx], cx.phase, fs) || !mbar_wait(&a_full[sa], ca.phase, fs)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t x_desc = x_desc0 + (uint64_t)(sx * (L::kXBytes >> 4));
          const uint32_t a_tmem = tmem_base + kW8ACol + 32 * sa;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t bdesc = x_desc + (uint64_t)(k * 32 >> 4);
            umma_f16_ts(d_tmem, a_tmem + 8 * k, bdesc, kIdesc, (kb != sg.k0) || (k != 0));
          }
          issued_any = true;
          umma_commit(&x_empty[sx]);
          umma_commit(&a_empty[sa]);
          cx.advance();
          ca.advance();
        }
        if (ok) umma_commit(&t_full[acc]);
        ++tl;
      }
      if (!ok && issued_any) {
        umma_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp >= 4 && warp < 4 + kW8ConvWarps) {
    // ------------------------------------------------------ int8 -> f16 -> TMEM
    // The g-th K-block of this CTA (over all its pieces, in order) sits in
    // weight stage g % SW and goes to TMEM stage g % SA; group `grp` converts
    // the blocks g = grp, grp + 2, ...
    const int q = warp & 3;
    const int grp = (warp - 4) >> 2;
    const long long nkb = work.kb_count();
    for (long long g = grp; g < nkb; g += kW8ConvGroups) {
      const int sw = (int)(g % kW8SW), sa = (int)(g % kW8SA);
      const uint32_t pw = (uint32_t)((g / kW8SW) & 1), pa = (uint32_t)((g / kW8SA) & 1);
      const bool ready = mbar_wait(&w_full[sw], pw, fs) && mbar_wait(&a_empty[sa], pa ^ 1, fs);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      w8_chunks_to_tmem<2>(smem_u32(smem + L::kOffW + sw * L::kWBytes), tmem_base, 32 * q,
                           kW8ACol + 32 * sa, 2 * q, lane);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[sa]);
        mbar_arrive(&w_empty[sw]);
      }
    }
  } else if (warp >= 4 + kW8ConvWarps) {
    // ------------------------------------------------------ epilogue
    // Every piece that ends a tile leaves through shared memory: a tile cut
    // between CTAs first has the other CTAs' partial accumulators added into
    // its TMEM accumulator (w8_add_partials); the residual, if any, is loaded
    // by TMA into the staging tile while the main loop still runs; the
    // accumulator is read, scaled (plus the residual: one f16 rounding of
    // acc * s + r) and packed to f16 into the staging tile, released to the
    // MMA at once, and one thread writes the tile to C with two TMA stores
    // that run while the next tile's main loop does. Contributor pieces
    // write their raw accumulator to the stream-K workspace instead
    // (w8_write_partial).
    const int q = warp & 3;
    const bool issuer = warp == 4 + kW8ConvWarps && lane == 0;
    uint8_t* stage = smem + L::kOffStage;
    // the warp's two 16 KB partial buffers: activation stage q (free once the
    // CTA's last main loop is done; a cut tile's finaliser is its last piece)
    uint8_t* fix_buf = smem + L::kOffX + q * L::kXBytes;
    const bool resid = args.C_init != nullptr;
    int tl = 0, rl = 0, r_landed = 0;
    bool stores_pending = false;
    long long pos = work.first();
    W8Seg sg;
    while (work.next(pos, sg)) {
      int tm, tn;
      tile_coords(sg.tile, args, tm, tn);
      const int acc = tl % kW8Acc;
      const uint32_t parity = (uint32_t)((tl / kW8Acc) & 1);
      const uint32_t acc_tmem = tmem_base + kW8BM * acc;
      int c_lo, c_hi;
      work.contributors(sg, &c_lo, &c_hi);
      if (sg.k0 > 0) {
        if (!w8_write_partial(args, fs, &t_full[acc], parity, acc_tmem, q, lane, blockIdx.x))
          break;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&t_empty[acc]);
        ++tl;
        continue;
      }
      float sc[2][2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = tn * kW8BN + 16 * (2 * q + h) + 2 * (lane >> 2);
        sc[h][0] = n < args.N ? __half2float(args.scale[n]) : 0.0f;
        sc[h][1] = n + 1 < args.N ? __half2float(args.scale[n + 1]) : 0.0f;
      }
      if (issuer) {
        // the previous tile's stores must have read the staging tile before
        // the residual lands in it (or the warps write it)
        if (stores_pending) bulk_wait_read_all();
        if (resid) {
          mbar_arrive_expect_tx(r_full, 2 * L::kBoxBytes);
          tma_load_2d(stage, &tmR, r_full, tn * kW8BN, tm * kW8BM);
          tma_load_2d(stage + L::kBoxBytes, &tmR, r_full, tn * kW8BN + 64, tm * kW8BM);
        }
      }
      // (a failed wait raises the CTA's abort flag before the barrier, so all
      // four warps leave together after it)
      bool ok = mbar_wait(&t_full[acc], parity, fs);
      if (ok && c_hi > c_lo)
        ok = w8_add_partials(args, fs, fix_buf, fix_full + 2 * q, acc_tmem, q, lane, c_lo, c_hi);
      if (ok && resid && mbar_wait(r_full, (uint32_t)(rl & 1), fs)) ++r_landed;
      if (resid) ++rl;
      named_barrier_sync(1, 32 * kW8EpiWarps);
      if (*abort_flag) break;
      tc_fence_after();
      uint8_t* box = stage + (q >> 1) * L::kBoxBytes;
      if (resid)
        w8_stage_tile<true>(acc_tmem, box, q, lane, sc);
      else
        w8_stage_tile<false>(acc_tmem, box, q, lane, sc);
      // the accumulator is read: the MMA may start the next tile
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&t_empty[acc]);
      fence_proxy_async_smem();
      named_barrier_sync(1, 32 * kW8EpiWarps);
      if (issuer) {
        tma_store_2d(&tmC, stage, tn * kW8BN, tm * kW8BM);
        tma_store_2d(&tmC, stage + L::kBoxBytes, tn * kW8BN + 64, tm * kW8BM);
        bulk_commit();
        stores_pending = true;
      }
      if (args.ndests > 1) w8_store_replicas(args, stage, tm, tn);
      ++tl;
    }
    if (issuer && stores_pending) bulk_wait_all();
    // the peer stores of w8_store_replicas are performed system-wide before
    // the kernel ends (see hxb_peer_barrier)
    if (args.ndests > 1) __threadfence_system();
    // after a failure: a residual load this thread issued may still be
    // landing in the staging tile
    if (issuer && r_landed < rl) {
      const unsigned long long t0 = globaltimer_ns();
      while (!mbar_try_wait(r_full, (uint32_t)((rl - 1) & 1)) &&
             globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace hxb
