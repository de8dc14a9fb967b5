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
//     per-column scale once (it factors out of the K sum). A whole tile
//     without a residual is packed to f16 into a 64 KB shared-memory staging
//     tile, the accumulator is released to the MMA as soon as it is read,
//     and one thread writes C with two TMA stores that overlap the next
//     tile's main loop. Stream-K pieces and residual tiles take a register
//     path (scales fetched before the accumulator is ready, residual and
//     partial-sum loads issued ahead of the TMEM reads, f16x2 column-pair
//     stores, one f16 rounding of acc * s + r).
//   * Measured decomposition of the 4096 x 4096 x 11008 dispatch on B200
//     (307 us before the staging was sized as below): tensor pipe alone
//     ~167 us; with TMA feeding but no conversion and no epilogue 234 us;
//     the int8 conversion adds ~62 us, the epilogue ~11 us.
// Shared-memory traffic per k-block is the int8 tile (written by TMA, read
// once by the converters) plus the activation tile (written by TMA, read by
// the tensor core); the f16 weights live only in registers and TMEM.
//
// Work split. Data-parallel: CTA b owns whole output tiles b, b + grid, ...
// Stream-K (args.streamk): the tiles x K-blocks iteration space is cut into
// `grid` equal contiguous shares, so every SM gets the same number of MMAs
// whatever the tile count. A tile cut between CTAs is summed as follows: the
// CTA holding the tile's first K-block (it processes that piece LAST, at the
// end of its share) finalises it; every other CTA holding a piece of the
// tile holds it FIRST, writes its f32 partial accumulator to
// args.sk_partials[cta] and raises args.sk_flags[cta][quarter]. The finaliser
// adds the partials in CTA order (deterministic), stores C and clears the
// flags, so the flag array is all zero again when the kernel ends. No CTA
// waits on a lower-numbered CTA, and every wait is bounded.
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
  // t_full[2], t_empty[2], drain
  static constexpr int kNumBars = 2 * kW8SX + 2 * kW8SW + 2 * kW8SA + 5;
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
// roles of the unit. Units are numbered 0 .. nunits-1.
struct W8Work {
  int num_kb, num_tiles, streamk, unit, nunits;
  long long total, it0, it1;

  // First iteration of unit c's stream-K share (total >= nunits, so no share
  // is empty).
  __device__ __forceinline__ long long share_begin(int c) const { return total * c / nunits; }
  __device__ __forceinline__ void init(const GemmArgs& a, int unit_, int nunits_) {
    unit = unit_;
    nunits = nunits_;
    num_kb = (a.K + kBK - 1) / kBK;
    num_tiles = a.tiles_m * a.tiles_n;
    streamk = a.streamk;
    total = (long long)num_tiles * num_kb;
    it0 = share_begin(unit);
    it1 = share_begin(unit + 1);
  }
  __device__ __forceinline__ long long first() const { return streamk ? it0 : unit; }
  // K-blocks this unit processes in all.
  __device__ __forceinline__ long long kb_count() const {
    if (streamk) return it1 - it0;
    const long long nt = unit < num_tiles ? (num_tiles - 1 - unit) / nunits + 1 : 0;
    return nt * num_kb;
  }
  __device__ __forceinline__ bool next(long long& pos, W8Seg& s) const {
    if (!streamk) {
      if (pos >= num_tiles) return false;
      s.tile = (int)pos;
      s.k0 = 0;
      s.k1 = num_kb;
      pos += nunits;
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
  __device__ __forceinline__ void contributors(const W8Seg& sg, int* lo, int* hi) const {
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

// Epilogue of one piece for epilogue warp q (lane t) of a CTA whose TMEM
// accumulator at column `acc_tmem` holds weight columns n0 .. n0 + 127 (lane
// order of w8_tmem.cuh) by activation rows m0 .. m0 + kW8BM - 1. Waits for the
// accumulator (t_full, phase `parity`). A contributor piece writes the raw
// accumulator to partial slot `self_slot` and raises that slot's flag; any
// other piece adds the partials of slots c * slot_mul + slot_add for c in
// [c_lo, c_hi) (waiting for their flags and clearing them afterwards), then
// applies the scale and the optional residual and stores C.
//
// tcgen05.ld.16x256b gives lane t the TMEM lanes t/4 and t/4 + 8 of a 16-lane
// group -- weight columns n and n + 1 -- at accumulator columns (activation
// rows) m, m + 1: each pair (n, n + 1) of one row m is stored as one 4-byte
// f16x2. Scales are fetched before the accumulator is ready; residual and
// partial-sum loads are issued ahead of the TMEM reads they pair with, two
// 32-column chunks at a time. Returns false after a timeout.
__device__ __forceinline__ bool w8_epilogue_piece(const GemmArgs& args, const FailState& fs,
                                                  uint64_t* t_full, uint32_t parity,
                                                  uint32_t acc_tmem, int n0, int m0, int q,
                                                  int t, bool contributor, int self_slot,
                                                  int c_lo, int c_hi, int slot_mul,
                                                  int slot_add) {
  const int lane = t;
  float sc[2][2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int n = n0 + 16 * (2 * q + h) + 2 * (t >> 2);
    sc[h][0] = (!contributor && n < args.N) ? __half2float(args.scale[n]) : 0.0f;
    sc[h][1] = (!contributor && n + 1 < args.N) ? __half2float(args.scale[n + 1]) : 0.0f;
  }
  bool ready = mbar_wait(t_full, parity, fs);
  for (int c2 = c_lo; c2 < c_hi && ready; ++c2)
    ready = wait_flag(args.sk_flags + 4 * (c2 * slot_mul + slot_add) + q, fs);
  if (!__all_sync(0xffffffffu, ready)) return false;
  tc_fence_after();

  if (contributor) {
    float4* part = reinterpret_cast<float4*>(args.sk_partials) +
                   (size_t)self_slot * (kW8PartialFloats / 4);
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      const uint32_t taddr = acc_tmem + ((uint32_t)(16 * (2 * q + h)) << 16);
#pragma unroll 1
      for (int c = 0; c < kW8BM / 32; c += 2) {
        uint32_t r[2][16];
        tmem_ld_16x256b_x4(taddr + 32 * c, r[0]);
        tmem_ld_16x256b_x4(taddr + 32 * (c + 1), r[1]);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 2; ++u)
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
    if (lane == 0) st_release_gpu(args.sk_flags + 4 * self_slot + q, 1);
    return true;
  }
  const bool rows_full = m0 + kW8BM <= args.M;
  const __half* R = reinterpret_cast<const __half*>(args.C_init);
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    const int chunk = 2 * q + h;
    const int n = n0 + 16 * chunk + 2 * (t >> 2);
    const bool n0_ok = n < args.N, n1_ok = n + 1 < args.N;
    const bool fast = rows_full && n1_ok;
    const float s0 = h ? sc[1][0] : sc[0][0], s1 = h ? sc[1][1] : sc[0][1];
    const uint32_t taddr = acc_tmem + ((uint32_t)(16 * chunk) << 16);
    // row of (chunk c, rep, j) = row0 + 32 c + 8 rep + j
    const int row0 = m0 + 2 * (t & 3);
    __half* cbase = reinterpret_cast<__half*>(args.C) + (long long)row0 * args.ldc + n;
    const __half* rbase = R ? R + (long long)row0 * args.ldc + n : nullptr;
#pragma unroll 1
    for (int c = 0; c < kW8BM / 32; c += 2) {
      // residual pairs and partial sums of the two chunks, loaded ahead
      // of the TMEM reads
      uint32_t res[2][8];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int e = 0; e < 8; ++e) res[u][e] = 0u;
      if (rbase && fast) {
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int rep = 0; rep < 4; ++rep)
#pragma unroll
            for (int j = 0; j < 2; ++j)
              res[u][2 * rep + j] = __ldg(reinterpret_cast<const unsigned int*>(
                  rbase + (long long)(32 * (c + u) + 8 * rep + j) * args.ldc));
      }
      float v[2][16];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int e = 0; e < 16; ++e) v[u][e] = 0.0f;
      for (int c2 = c_lo; c2 < c_hi; ++c2) {
        const float4* part = reinterpret_cast<const float4*>(args.sk_partials) +
                             (size_t)(c2 * slot_mul + slot_add) * (kW8PartialFloats / 4);
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int rep = 0; rep < 4; ++rep) {
            const float4 p = __ldcg(part + w8_partial_index(q, h, c + u, rep, t));
            v[u][4 * rep] += p.x;
            v[u][4 * rep + 1] += p.y;
            v[u][4 * rep + 2] += p.z;
            v[u][4 * rep + 3] += p.w;
          }
      }
      uint32_t r[2][16];
      tmem_ld_16x256b_x4(taddr + 32 * c, r[0]);
      tmem_ld_16x256b_x4(taddr + 32 * (c + 1), r[1]);
      tmem_wait_ld();
      // this CTA's accumulator plus the partials (summed in CTA order)
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int e = 0; e < 16; ++e) v[u][e] = __uint_as_float(r[u][e]) + v[u][e];
      if (fast) {
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int rep = 0; rep < 4; ++rep)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              float v0 = v[u][4 * rep + j] * s0;
              float v1 = v[u][4 * rep + 2 + j] * s1;
              if (rbase) {
                const float2 rv = __half22float2(
                    *reinterpret_cast<const __half2*>(&res[u][2 * rep + j]));
                v0 += rv.x;
                v1 += rv.y;
              }
              *reinterpret_cast<__half2*>(
                  cbase + (long long)(32 * (c + u) + 8 * rep + j) * args.ldc) =
                  __floats2half2_rn(v0, v1);
            }
      } else if (n0_ok) {
        // ragged edge: rows past M, or the last column of an odd N
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int rep = 0; rep < 4; ++rep)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int dm = 32 * (c + u) + 8 * rep + j;
              if (row0 + dm >= args.M) continue;
              const long long off = (long long)dm * args.ldc;
              float v0 = v[u][4 * rep + j] * s0;
              float v1 = v[u][4 * rep + 2 + j] * s1;
              if (n1_ok) {
                if (rbase) {
                  const float2 rv =
                      __half22float2(*reinterpret_cast<const __half2*>(rbase + off));
                  v0 += rv.x;
                  v1 += rv.y;
                }
                *reinterpret_cast<__half2*>(cbase + off) = __floats2half2_rn(v0, v1);
              } else {
                if (rbase) v0 += __half2float(rbase[off]);
                cbase[off] = __float2half_rn(v0);
              }
            }
      }
    }
  }
  // the partials of this tile are consumed: clear their flags for the next
  // launch
  if (lane == 0)
    for (int c2 = c_lo; c2 < c_hi; ++c2) args.sk_flags[4 * (c2 * slot_mul + slot_add) + q] = 0;
  return true;
}

__global__ void __launch_bounds__(kW8Threads, 1)
    gemm_w8_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmW,
                         const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
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
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmC);
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
          const uint32_t x_addr = smem_u32(smem + L::kOffX + sx * L::kXBytes);
          const uint32_t a_tmem = tmem_base + kW8ACol + 32 * sa;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t bdesc = make_smem_desc(x_addr + k * 32, 16, 1024, kLayoutSwizzle128);
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
    // Whole tiles without a residual leave through shared memory: the
    // accumulator is read, scaled and packed to f16 into the staging tile,
    // the accumulator is released to the MMA at once, and one thread writes
    // the tile to C with two TMA stores that run while the next tile's main
    // loop does. Cut (stream-K) pieces and tiles with a residual use
    // w8_epilogue_piece (register path, one f16 rounding of acc * s + r).
    const int q = warp & 3;
    const bool issuer = warp == 4 + kW8ConvWarps && lane == 0;
    uint8_t* stage = smem + L::kOffStage;
    const uint32_t stage_s = smem_u32(stage);
    int tl = 0;
    bool stores_pending = false;
    long long pos = work.first();
    W8Seg sg;
    while (work.next(pos, sg)) {
      int tm, tn;
      tile_coords(sg.tile, args, tm, tn);
      const int acc = tl % kW8Acc;
      const uint32_t parity = (uint32_t)((tl / kW8Acc) & 1);
      int c_lo, c_hi;
      work.contributors(sg, &c_lo, &c_hi);
      const bool staged = sg.k0 == 0 && c_lo == c_hi && args.C_init == nullptr;
      if (!staged) {
        if (!w8_epilogue_piece(args, fs, &t_full[acc], parity, tmem_base + kW8BM * acc,
                               tn * kW8BN, tm * kW8BM, q, lane, sg.k0 > 0, blockIdx.x, c_lo,
                               c_hi, 1, 0))
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
      // (a failed wait raises the CTA's abort flag before the barrier, so all
      // four warps leave together after it)
      mbar_wait(&t_full[acc], parity, fs);
      // the previous tile's stores must have read the staging tile
      if (issuer && stores_pending) bulk_wait_read_all();
      named_barrier_sync(1, 32 * kW8EpiWarps);
      if (*abort_flag) break;
      tc_fence_after();
      // lane t writes f16 pairs (n, n + 1), n = 16 (2q + h) + 2 (t >> 2), of
      // rows m = 32 c + 8 rep + 2 (t & 3) + j into box q >> 1 at 16-byte
      // chunk (4 (q & 1) + 2 h + (t >> 4)) ^ (m & 7), word (t >> 2) & 3: the 32
      // lanes of each store hit 32 different banks.
      const uint32_t box_s = stage_s + (uint32_t)((q >> 1) * L::kBoxBytes);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const uint32_t taddr = tmem_base + ((uint32_t)(16 * (2 * q + h)) << 16) + kW8BM * acc;
        const float s0 = h ? sc[1][0] : sc[0][0], s1 = h ? sc[1][1] : sc[0][1];
        const int chunk0 = 4 * (q & 1) + 2 * h + (lane >> 4);
        const uint32_t word = 4u * (uint32_t)((lane >> 2) & 3);
#pragma unroll 1
        for (int c = 0; c < kW8BM / 32; c += 2) {
          uint32_t r[2][16];
          tmem_ld_16x256b_x4(taddr + 32 * c, r[0]);
          tmem_ld_16x256b_x4(taddr + 32 * (c + 1), r[1]);
          tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int rep = 0; rep < 4; ++rep)
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int m = 32 * (c + u) + 8 * rep + 2 * (lane & 3) + j;
                const uint32_t v = pack_half2(__uint_as_float(r[u][4 * rep + j]) * s0,
                                              __uint_as_float(r[u][4 * rep + 2 + j]) * s1);
                const uint32_t a =
                    box_s + (uint32_t)(m * 128 + ((chunk0 ^ (m & 7)) << 4)) + word;
                asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
              }
        }
      }
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
      ++tl;
    }
    if (issuer && stores_pending) bulk_wait_all();
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
