// Int8-weight GEMM for sm_100a: C[M,N] f16 = (A[M,K] f16 . W[K,N] int8) * scale[N].
//
// The weights are dequantised inside the main loop: TMA lands the raw int8
// tile, converter warps turn it into f16 (exactly: |w| <= 127) directly in the
// 128B-swizzled MN-major layout tcgen05.mma reads, and the per-column scale is
// applied once in the epilogue (it factors out of the K sum).
//
// Three decoupled shared-memory rings keep every stage busy:
//   A ring   (SA deep)  f16 activations, filled by TMA, freed by the MMA
//   W8 ring  (SW deep)  raw int8 weights, filled by TMA, freed by converters
//   B16 ring (SB deep)  converted f16 weights, filled by converters, freed by
//                       the MMA
// so the int8 bytes leave shared memory as soon as they are converted and the
// TMA latency is covered by the deep A / W8 rings rather than by the large f16
// buffers.
#pragma once

#include "gemm_sm100.cuh"

namespace hxb {

// Position in an S-deep ring of mbarrier-guarded slots: slot index and the
// parity of the phase the slot is in. Advancing is two adds and a compare, so
// the single-thread producer / MMA loops carry no division on their critical
// path.
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
    // step the cursor back by one
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

template <int BN, int SA, int SW, int SB>
struct W8Smem {
  static constexpr int kABytes = kBM * kBK * 2;   // 16 KB
  static constexpr int kWBytes = BN * kBK;        // int8 tile
  static constexpr int kBBytes = BN * kBK * 2;    // converted f16 tile
  static constexpr int kOffA = 0;
  static constexpr int kOffW = kOffA + SA * kABytes;
  static constexpr int kOffB = kOffW + SW * kWBytes;
  static constexpr int kOffBar = kOffB + SB * kBBytes;
  // full_a, empty_a [SA]; full_w, empty_w [SW]; conv_full, conv_empty [SB];
  // tfull[2], tempty[2], drain
  static constexpr int kNumBars = 2 * SA + 2 * SW + 2 * SB + 5;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;  // tmem addr, abort, go
  static constexpr int kAlloc = kBytes + 1024;
  static constexpr int kThreads = 14 * 32;  // 6 + 8 converter warps
  static constexpr int kConvWarps = 8;
  static constexpr int kTmemCols = 2 * BN;
};

template <int BN, int SA, int SW, int SB>
__global__ void __launch_bounds__(448, 1)
    gemm_w8_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmW,
                         const GemmArgs args) {
  using L = W8Smem<BN, SA, SW, SB>;
  constexpr uint32_t kIdesc = make_idesc_f16(kBM, BN, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* full_a = bars;
  uint64_t* empty_a = full_a + SA;
  uint64_t* full_w = empty_a + SA;
  uint64_t* empty_w = full_w + SW;
  uint64_t* conv_full = empty_w + SW;
  uint64_t* conv_empty = conv_full + SB;
  uint64_t* tfull = conv_empty + SB;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = args.tiles_m * args.tiles_n;
  const int num_kb = (args.K + kBK - 1) / kBK;
  const FailState fs{abort_flag, args.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < SA; ++s) { mbar_init(&full_a[s], 1); mbar_init(&empty_a[s], 1); }
    for (int s = 0; s < SW; ++s) { mbar_init(&full_w[s], 1); mbar_init(&empty_w[s], 1); }
    for (int s = 0; s < SB; ++s) { mbar_init(&conv_full[s], 1); mbar_init(&conv_empty[s], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], 4); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      RingCursor<SW> cw;
      RingCursor<SA> ca;
      int issued_w = 0, issued_a = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, args, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_w[cw.slot], cw.phase ^ 1, fs)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_w[cw.slot], L::kWBytes);
          tma_load_2d(smem + L::kOffW + cw.slot * L::kWBytes, &tmW, &full_w[cw.slot],
                      tn * BN, kb * kBK);
          cw.advance();
          ++issued_w;
          if (!mbar_wait(&empty_a[ca.slot], ca.phase ^ 1, fs)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_a[ca.slot], L::kABytes);
          tma_load_2d(smem + L::kOffA + ca.slot * L::kABytes, &tmA, &full_a[ca.slot],
                      kb * kBK, tm * kBM);
          ca.advance();
          ++issued_a;
        }
      }
      // Wait (bounded) for the last copies of each ring to land before the
      // CTA may exit; on the normal path they have long completed. Walking
      // the cursors backwards visits the most recent issue of every slot.
      drain_ring<SW>(full_w, cw, issued_w);
      drain_ring<SA>(full_a, ca, issued_a);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      RingCursor<SA> ca;
      RingCursor<SB> cb;
      int tl = 0;
      bool ok = true, issued_any = false;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++tl) {
        const int acc = tl & 1;
        if (!mbar_wait(&tempty[acc], ((tl >> 1) & 1) ^ 1, fs)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          const int sa = ca.slot, sb = cb.slot;
          if (!mbar_wait(&full_a[sa], ca.phase, fs) || !mbar_wait(&conv_full[sb], cb.phase, fs)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + L::kOffA + sa * L::kABytes);
          const uint32_t b_addr = smem_u32(smem + L::kOffB + sb * L::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = make_smem_desc(a_addr + k * 32, 16, 1024, kLayoutSwizzle128);
            const uint64_t bdesc = make_smem_desc(b_addr + k * 16 * 128, kBK * 128, 1024,
                                                  kLayoutSwizzle128);
            umma_f16_ss(d_tmem, adesc, bdesc, kIdesc, (kb | k) != 0);
          }
          issued_any = true;
          umma_commit(&empty_a[sa]);
          umma_commit(&conv_empty[sb]);
          ca.advance();
          cb.advance();
        }
        if (ok) umma_commit(&tfull[acc]);
      }
      if (!ok && issued_any) {
        umma_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------------ epilogue
    const int q = warp & 3;
    int tl = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tl) {
      int tm, tn;
      tile_coords(t, args, tm, tn);
      const int acc = tl & 1;
      const bool ready = mbar_wait(&tfull[acc], (tl >> 1) & 1, fs);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const int row = tm * kBM + q * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c, r);
        tmem_wait_ld();
        const int col0 = tn * BN + c;
        if (row >= args.M || col0 >= args.N) continue;
        store_chunk<true, kOutF16>(args, row, col0, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  } else {
    // ------------------------------------------------------ int8 -> f16
    // One elected converter thread does the mbarrier handshakes; the group
    // of kConvWarps warps meets on a named barrier, so each k-block costs one
    // wake-up from the MMA's commit instead of one per warp.
    const int ct = threadIdx.x - 6 * 32;  // 0..32*kConvWarps-1
    constexpr int kConvThreads = 32 * L::kConvWarps;
    volatile int* go = abort_flag + 1;  // per-k-block decision of the leader
    RingCursor<SW> cw;
    RingCursor<SB> cb;
    constexpr int kUnitsPerRow = BN / 16;  // 16-byte int8 units per k row
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int sw = cw.slot, sb = cb.slot;
        if (ct == 0)
          *go = mbar_wait(&full_w[sw], cw.phase, fs) &&
                mbar_wait(&conv_empty[sb], cb.phase ^ 1, fs);
        named_barrier_sync(1, kConvThreads);
        if (!*go) { ok = false; break; }
        const uint8_t* src = smem + L::kOffW + sw * L::kWBytes;
        uint8_t* dst = smem + L::kOffB + sb * L::kBBytes;
#pragma unroll
        for (int it = 0; it < kBK * kUnitsPerRow / kConvThreads; ++it) {
          const int w = ct + it * kConvThreads;
          const int k = w / kUnitsPerRow;
          const int c16 = w - k * kUnitsPerRow;
          const uint4 raw = *reinterpret_cast<const uint4*>(src + k * BN + c16 * 16);
          uint4 o0, o1;
          i8x4_to_f16x4(raw.x, o0.x, o0.y);
          i8x4_to_f16x4(raw.y, o0.z, o0.w);
          i8x4_to_f16x4(raw.z, o1.x, o1.y);
          i8x4_to_f16x4(raw.w, o1.z, o1.w);
          store_swizzled_pair(dst, c16, k, o0, o1);
        }
        fence_proxy_async_smem();
        named_barrier_sync(1, kConvThreads);
        if (ct == 0) {
          mbar_arrive(&conv_full[sb]);
          mbar_arrive(&empty_w[sw]);
        }
        cw.advance();
        cb.advance();
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

}  // namespace hxb
