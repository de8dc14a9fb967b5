// Split-K tcgen05 GEMM for sm_100a: the f16 matmul dispatch for shapes whose
// output tiles are too few to occupy the SMs (
// 1024^3, and the small-M / small-N shapes of the configuration-5b sweep).
//
//   C[M,N] = A[M,K] . B  (+ C_init)            f16 x f16 -> f32 accumulate
//
// One thread-block cluster of SPLIT CTAs computes one 128 x BN output tile;
// CTA r of the cluster runs the K-blocks [r * kb / SPLIT, (r + 1) * kb /
// SPLIT) through the same TMA -> shared-memory ring -> tcgen05.mma -> TMEM
// pipeline as the persistent kernel (gemm_sm100.cuh), so each CTA streams
// 1 / SPLIT of the tile's operands and the grid holds tiles * SPLIT CTAs.
// The partial accumulators are summed through distributed shared memory:
//   1. each CTA's epilogue warps copy its f32 accumulator from TMEM into its
//      own shared memory (the operand ring, idle once the last MMA retired);
//   2. a cluster barrier (release / acquire) publishes the partials;
//   3. CTA r sums rows [r * 128 / SPLIT, (r + 1) * 128 / SPLIT) of all
//      SPLIT partials, reading its peers' shared memory with
//      ld.shared::cluster, in cluster-rank order (deterministic), adds
//      C_init if any, rounds once and stores;
//   4. a second cluster barrier keeps every CTA's shared memory alive until
//      its peers have read it.
// No global workspace, no flags and no atomics are involved. Every thread of
// every CTA reaches both cluster barriers, on the failure path too (its
// mbarrier waits are bounded and a failed role falls through to them), and
// the CTAs of a cluster are co-scheduled by the hardware, so the barriers
// always complete.
#pragma once

#include "gemm_sm100.cuh"

namespace hxb {

template <int BN, int STAGES>
struct SplitSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + STAGES * kABytes;
  static constexpr int kRingBytes = kOffB + STAGES * kBBytes;
  // f32 partial [128 rows][BN + 4] (4 floats of padding per row keep the
  // row-per-thread float4 writes free of bank conflicts)
  static constexpr int kRedPitch = BN + 4;
  static constexpr int kRedBytes = kBM * kRedPitch * 4;
  static_assert(kRedBytes <= kRingBytes, "the partial reuses the operand ring");
  static constexpr int kOffBar = kRingBytes;
  // full[S], empty[S], tfull
  static constexpr int kNumBars = 2 * STAGES + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <int BN, int STAGES, int BMODE, int OUT, int SPLIT>
__global__ void __launch_bounds__(GemmShape<BN, BMODE>::kThreads, 1)
    gemm_splitk_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                             const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  using L = SplitSmem<BN, STAGES>;
  constexpr int kTmemCols = BN < 32 ? 32 : BN;
  constexpr uint32_t kIdesc = make_idesc_f16(kBM, BN, 0, BMODE == kBF16RowMajorNK ? 0 : 1);
  constexpr uint32_t kTxBytes = L::kABytes + L::kBBytes;
  constexpr int kRows = kBM / SPLIT;  // output rows each CTA of the cluster finishes

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  float* red = reinterpret_cast<float*>(smem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int tile = blockIdx.y;
  int tm, tn;
  tile_coords(tile, args, tm, tn);
  const int num_kb = (args.K + kBK - 1) / kBK;
  const int kb0 = (int)((long long)num_kb * rank / SPLIT);
  const int kb1 = (int)((long long)num_kb * (rank + 1) / SPLIT);
  const FailState fs{abort_flag, args.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      // (no L2 prefetch before the wait here: measured 2 % slower on
      // 512 x 512 x 8192, while the persistent kernel gains 1 % from it)
      pdl_wait();
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, fs)) break;
        mbar_arrive_expect_tx(&full[stage], kTxBytes);
        tma_load_2d(smem + L::kOffA + stage * L::kABytes, &tmA, &full[stage], kb * kBK, tm * kBM);
        if constexpr (BMODE == kBF16RowMajorKN) {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(smem + L::kOffB + stage * L::kBBytes + j * (kBK * 128), &tmB,
                        &full[stage], tn * BN + 64 * j, kb * kBK);
        } else {
          tma_load_2d(smem + L::kOffB + stage * L::kBBytes, &tmB, &full[stage], kb * kBK,
                      tn * BN);
        }
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      // never leave copies landing in shared memory (bounded on failure)
      const long long nd = issued < STAGES ? issued : STAGES;
      for (long long i = 0; i < nd; ++i) {
        const long long u = issued - 1 - i;
        const int s = (int)(u % STAGES);
        const uint32_t ph = (uint32_t)((u / STAGES) & 1);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[s], ph) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, fs)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + L::kOffA + stage * L::kABytes);
        const uint32_t b_addr = smem_u32(smem + L::kOffB + stage * L::kBBytes);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t adesc = make_smem_desc(a_addr + k * 32, 16, 1024, kLayoutSwizzle128);
          uint64_t bdesc;
          if (BMODE == kBF16RowMajorNK)
            bdesc = make_smem_desc(b_addr + k * 32, 16, 1024, kLayoutSwizzle128);
          else
            bdesc = make_smem_desc(b_addr + k * 16 * 128, kBK * 128, 1024, kLayoutSwizzle128);
          umma_f16_ss(tmem_base, adesc, bdesc, kIdesc, (kb > kb0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      // tfull completes when every MMA issued so far has retired (also on
      // the failure path, so TMEM is never freed under a running MMA)
      umma_commit(tfull);
      (void)ok;
    }
  } else {
    // ------------------------------------------------------ partial -> smem
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool ready = kb1 > kb0 ? mbar_wait(tfull, 0, fs) : true;
    if (__all_sync(0xffffffffu, ready)) {
      tc_fence_after();
      // the operand ring is idle: the last MMA (and so every copy it read)
      // has completed
      fence_proxy_async_smem();
      const int row = q * 32 + lane;
      float* dst = red + row * L::kRedPitch;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        if (kb1 > kb0) {
          tmem_ld_32x32b_x32(t_row + c, r);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0u;
        }
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(dst + c + j) =
              make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                          __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
      }
    }
  }

  // -------------------------------------------------- cluster reduction
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // every partial of the cluster is in shared memory
  {
    const int rows = kRows;
    const int chunks = BN / 4;  // float4 columns per row
    const uint32_t red_addr = smem_u32(red);
    const int row0 = (int)rank * rows;
    for (int i = threadIdx.x; i < rows * chunks; i += blockDim.x) {
      const int lr = row0 + i / chunks;
      const int c4 = (i % chunks) * 4;
      const int grow = tm * kBM + lr, gcol = tn * BN + c4;
      if (grow >= args.M || gcol >= args.N) continue;
      const uint32_t off = (uint32_t)((lr * L::kRedPitch + c4) * 4);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < SPLIT; ++r) {
        const float4 p = ld_cluster_f4(map_to_rank(red_addr + off, (uint32_t)r));
        acc.x += p.x;
        acc.y += p.y;
        acc.z += p.z;
        acc.w += p.w;
      }
      float v[4] = {acc.x, acc.y, acc.z, acc.w};
      const int nv = min(4, args.N - gcol);
      if constexpr (OUT == kOutF16) {
        __half* crow = reinterpret_cast<__half*>(args.C) + (long long)grow * args.ldc + gcol;
        const __half* irow = args.C_init ? reinterpret_cast<const __half*>(args.C_init) +
                                               (long long)grow * args.ldc + gcol
                                         : nullptr;
        if (nv == 4 && args.vec_ok) {
          if (irow) {
            const uint2 i2 = *reinterpret_cast<const uint2*>(irow);
            const __half2* h = reinterpret_cast<const __half2*>(&i2);
            const float2 a = __half22float2(h[0]), b = __half22float2(h[1]);
            v[0] += a.x;
            v[1] += a.y;
            v[2] += b.x;
            v[3] += b.y;
          }
          uint2 o;
          o.x = pack_half2(v[0], v[1]);
          o.y = pack_half2(v[2], v[3]);
          *reinterpret_cast<uint2*>(crow) = o;
        } else {
          for (int j = 0; j < nv; ++j) {
            float x = v[j];
            if (irow) x += __half2float(irow[j]);
            crow[j] = __float2half_rn(x);
          }
        }
      } else {
        float* crow = reinterpret_cast<float*>(args.C) + (long long)grow * args.ldc + gcol;
        const float* irow = args.C_init ? reinterpret_cast<const float*>(args.C_init) +
                                              (long long)grow * args.ldc + gcol
                                        : nullptr;
        if (nv == 4 && args.vec_ok) {
          float4 o = make_float4(v[0], v[1], v[2], v[3]);
          if (irow) {
            const float4 i4 = *reinterpret_cast<const float4*>(irow);
            o.x += i4.x;
            o.y += i4.y;
            o.z += i4.z;
            o.w += i4.w;
          }
          *reinterpret_cast<float4*>(crow) = o;
        } else {
          for (int j = 0; j < nv; ++j) crow[j] = v[j] + (irow ? irow[j] : 0.f);
        }
      }
    }
  }
  cluster_sync_all();  // peers are done reading this CTA's partial
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace hxb
