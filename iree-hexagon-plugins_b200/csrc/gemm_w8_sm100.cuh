// Int8-weight GEMM for sm_100a: C[M,N] f16 = (A[M,K] f16 . W[K,N] int8) * scale[N].
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
//     operand (M = 128 weight columns) of tcgen05.mma;
//   * one thread issues tcgen05.mma (A from TMEM, B = activations from shared
//     memory, N = 192 activation rows) into one of two 192-column f32 TMEM
//     accumulators, so the epilogue of tile t overlaps the main loop of t+1;
//   * four epilogue warps read the accumulator back, apply the per-column
//     scale once (it factors out of the K sum), add the optional residual and
//     store C transposed.
// Shared-memory traffic per k-block is the int8 tile (written by TMA, read
// once by the converters) plus the activation tile (written by TMA, read by
// the tensor core); the f16 weights live only in registers and TMEM.
//
// Roles (512 threads, one CTA per SM, persistent over output tiles):
//   warp 0        TMA producer (one lane)
//   warp 1        TMEM owner + MMA issuer (one lane)
//   warps 2-3     idle
//   warps 4-11    int8 -> f16 converters (two per TMEM lane quarter, each one
//                 16-column chunk of the block)
//   warps 12-15   epilogue
// TMEM: accumulators in columns [0, 192) and [192, 384), kW8SA converted
// weight stages of 32 columns from column 384.
#pragma once

#include "gemm_sm100.cuh"
#include "w8_tmem.cuh"

namespace hxb {

constexpr int kW8BN = 128;  // weight columns per tile (MMA M, TMEM lanes)
constexpr int kW8BM = 192;  // activation rows per tile (MMA N)
constexpr int kW8SX = 6;    // activation stages
constexpr int kW8SW = 8;    // int8 weight stages
constexpr int kW8SA = 4;    // TMEM weight stages
constexpr int kW8ACol = 2 * kW8BM;  // first TMEM column of the weight stages
constexpr int kW8Threads = 16 * 32;
constexpr int kW8ConvWarps = 8;
constexpr int kW8EpiWarps = 4;

struct W8Smem {
  static constexpr int kXBytes = kW8BM * kBK * 2;  // 24 KB
  static constexpr int kWBytes = kW8BN * kBK;      // 8 KB
  static constexpr int kOffX = 0;
  static constexpr int kOffW = kOffX + kW8SX * kXBytes;
  static constexpr int kOffBar = kOffW + kW8SW * kWBytes;
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

__global__ void __launch_bounds__(kW8Threads, 1)
    gemm_w8_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmW, const GemmArgs args) {
  using L = W8Smem;
  // D[128 n x 192 m] += W^T (TMEM, K-major) . A^T (shared, K-major)
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
  const int num_tiles = args.tiles_m * args.tiles_n;
  const int num_kb = (args.K + kBK - 1) / kBK;
  const FailState fs{abort_flag, args.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < kW8SX; ++s) { mbar_init(&x_full[s], 1); mbar_init(&x_empty[s], 1); }
    for (int s = 0; s < kW8SW; ++s) { mbar_init(&w_full[s], 1); mbar_init(&w_empty[s], kW8ConvWarps); }
    for (int s = 0; s < kW8SA; ++s) { mbar_init(&a_full[s], kW8ConvWarps); mbar_init(&a_empty[s], 1); }
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
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, args, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
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
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++tl) {
        const int acc = tl & 1;
        if (!mbar_wait(&t_empty[acc], (uint32_t)((tl >> 1) & 1) ^ 1, fs)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + kW8BM * acc;
        for (int kb = 0; kb < num_kb; ++kb) {
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
            umma_f16_ts(d_tmem, a_tmem + 8 * k, bdesc, kIdesc, (kb | k) != 0);
          }
          issued_any = true;
          umma_commit(&x_empty[sx]);
          umma_commit(&a_empty[sa]);
          cx.advance();
          ca.advance();
        }
        if (ok) umma_commit(&t_full[acc]);
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
    const int q = warp & 3;
    const int h = (warp - 4) >> 2;  // the warp's 16-column chunk of the quarter
    const int chunk = 2 * q + h;
    RingCursor<kW8SW> cw;
    RingCursor<kW8SA> ca;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < num_kb; ++kb) {
        const int sw = cw.slot, sa = ca.slot;
        const bool ready = mbar_wait(&w_full[sw], cw.phase, fs) &&
                           mbar_wait(&a_empty[sa], ca.phase ^ 1, fs);
        if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
        tc_fence_after();
        w8_chunk_to_tmem(smem_u32(smem + L::kOffW + sw * L::kWBytes), tmem_base, 16 * chunk,
                         kW8ACol + 32 * sa, chunk, lane);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&a_full[sa]);
          mbar_arrive(&w_empty[sw]);
        }
        cw.advance();
        ca.advance();
      }
    }
  } else if (warp >= 4 + kW8ConvWarps) {
    // ------------------------------------------------------ epilogue
    // tcgen05.ld.16x256b gives lane t the TMEM lanes t/4 and t/4 + 8 of a
    // 16-lane group -- weight columns n and n + 1 (see w8_tmem.cuh) -- at
    // accumulator columns (activation rows) m, m + 1: each pair (n, n + 1) of
    // one row m is stored as one 4-byte f16x2.
    const int q = warp & 3;
    const int t = lane;
    int tl = 0;
    for (int tt = blockIdx.x; tt < num_tiles; tt += gridDim.x, ++tl) {
      int tm, tn;
      tile_coords(tt, args, tm, tn);
      const int acc = tl & 1;
      const bool ready = mbar_wait(&t_full[acc], (uint32_t)((tl >> 1) & 1), fs);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const int m0 = tm * kW8BM;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int chunk = 2 * q + h;
        const int n = tn * kW8BN + 16 * chunk + 2 * (t >> 2);
        const bool n0_ok = n < args.N, n1_ok = n + 1 < args.N;
        const float s0 = n0_ok ? __half2float(args.scale[n]) : 0.0f;
        const float s1 = n1_ok ? __half2float(args.scale[n + 1]) : 0.0f;
        __half* cbase = reinterpret_cast<__half*>(args.C) + n;
        const __half* rbase =
            args.C_init ? reinterpret_cast<const __half*>(args.C_init) + n : nullptr;
        const uint32_t taddr = tmem_base + ((uint32_t)(16 * chunk) << 16) + kW8BM * acc;
#pragma unroll 1
        for (int c = 0; c < kW8BM / 32; ++c) {
          uint32_t r[16];
          tmem_ld_16x256b_x4(taddr + 32 * c, r);
          tmem_wait_ld();
          if (!n0_ok) continue;
#pragma unroll
          for (int rep = 0; rep < 4; ++rep) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int m = m0 + 32 * c + 8 * rep + 2 * (t & 3) + j;
              if (m >= args.M) continue;
              float v0 = __uint_as_float(r[4 * rep + j]) * s0;
              float v1 = __uint_as_float(r[4 * rep + 2 + j]) * s1;
              const long long off = (long long)m * args.ldc;
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
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&t_empty[acc]);
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
