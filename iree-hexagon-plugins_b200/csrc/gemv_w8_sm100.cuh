// Decode-shaped int8-weight matmul for sm_100a (M <= 16 activation rows):
//   C[M,N] f16 = (A[M,K] f16 . W[K,N] int8) * scale[N]
//
// With M <= 16 the dispatch is bound by streaming W from HBM (45 MB for the
// BASELINE 4096 x 11008 weight), so the design goal is to keep enough bytes in
// flight on every SM and to touch W exactly once:
//   * swap-AB: the dequantised weight tile is the 128-row MMA operand
//     (D[128 n, 16 m] = W^T . A^T), so tcgen05 runs at M=128, N=16 and the
//     activations (padded to 16 rows by TMA zero fill) are the small operand;
//   * split-K over a thread-block cluster of KSPLIT CTAs, each streaming its
//     own K range of one 128-column weight tile; all of a CTA's int8 tiles are
//     in flight at once (SW-deep ring);
//   * the KSPLIT partial sums are reduced through distributed shared memory
//     (no global scratch, deterministic order), then scaled and stored.
#pragma once

#include "gemm_sm100.cuh"

namespace hxb {

constexpr int kGemvKSplit = 8;   // cluster size along K
constexpr int kGemvBN = 128;     // weight columns per CTA (MMA M)
constexpr int kGemvRows = 16;    // activation rows (MMA N)

template <int SW>
struct GemvSmem {
  static constexpr int kWBytes = kGemvBN * kBK;          // 8 KB int8 tile
  static constexpr int kXBytes = kGemvRows * kBK * 2;    // 2 KB activations
  static constexpr int kBBytes = kGemvBN * kBK * 2;      // 16 KB converted W
  static constexpr int kSB = 2;
  static constexpr int kOffW = 0;
  static constexpr int kOffX = kOffW + SW * kWBytes;
  static constexpr int kOffB = kOffX + SW * kXBytes;
  static constexpr int kOffRed = kOffB + kSB * kBBytes;  // [16][128] f32
  static constexpr int kOffBar = kOffRed + kGemvRows * kGemvBN * 4;
  // full[SW], empty[SW], conv_full[2], conv_empty[2], tfull, drain
  static constexpr int kNumBars = 2 * SW + 2 * kSB + 2;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static constexpr int kThreads = 6 * 32;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t local_addr, uint32_t cta) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(cta));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

template <int SW>
__global__ void __launch_bounds__(192, 2)
    gemv_w8_sm100_kernel(const __grid_constant__ CUtensorMap tmX,
                         const __grid_constant__ CUtensorMap tmW,
                         const GemmArgs args) {
  using L = GemvSmem<SW>;
  constexpr int kSB = L::kSB;
  // D[128 x 16]: A = converted W (MN-major), B = activations (K-major)
  constexpr uint32_t kIdesc = make_idesc_f16(kGemvBN, kGemvRows, 1, 0);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = full + SW;
  uint64_t* conv_full = empty + SW;
  uint64_t* conv_empty = conv_full + kSB;
  uint64_t* tfull = conv_empty + kSB;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  float* red = reinterpret_cast<float*>(smem + L::kOffRed);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = (int)cluster_ctarank();
  const int n0 = blockIdx.x * kGemvBN;
  const int nkb = (args.K + kBK - 1) / kBK;
  const int kb0 = (int)((long long)split * nkb / kGemvKSplit);
  const int kb1 = (int)((long long)(split + 1) * nkb / kGemvKSplit);
  const int my_kb = kb1 - kb0;
  const FailState fs{abort_flag, args.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < SW; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int s = 0; s < kSB; ++s) { mbar_init(&conv_full[s], 4); mbar_init(&conv_empty[s], 1); }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < my_kb; ++i) {
        const int s = i % SW;
        if (!mbar_wait(&empty[s], (uint32_t)((i / SW) & 1) ^ 1, fs)) break;
        mbar_arrive_expect_tx(&full[s], L::kWBytes + L::kXBytes);
        tma_load_2d(smem + L::kOffW + s * L::kWBytes, &tmW, &full[s], n0, (kb0 + i) * kBK);
        tma_load_2d(smem + L::kOffX + s * L::kXBytes, &tmX, &full[s], (kb0 + i) * kBK, 0);
        ++issued;
      }
      for (int i = issued - 1; i >= 0 && i >= issued - SW; --i) {
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[i % SW], (uint32_t)((i / SW) & 1)) &&
               globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && my_kb > 0) {
      bool ok = true;
      for (int i = 0; i < my_kb; ++i) {
        const int s = i % SW, sb = i % kSB;
        if (!mbar_wait(&full[s], (uint32_t)((i / SW) & 1), fs) ||
            !mbar_wait(&conv_full[sb], (uint32_t)((i / kSB) & 1), fs)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t w_addr = smem_u32(smem + L::kOffB + sb * L::kBBytes);
        const uint32_t x_addr = smem_u32(smem + L::kOffX + s * L::kXBytes);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t adesc = make_smem_desc(w_addr + k * 16 * 128, kBK * 128, 1024,
                                                kLayoutSwizzle128);
          const uint64_t bdesc = make_smem_desc(x_addr + k * 32, 16, 1024, kLayoutSwizzle128);
          umma_f16_ss(tmem_base, adesc, bdesc, kIdesc, (i | k) != 0);
        }
        umma_commit(&empty[s]);
        umma_commit(&conv_empty[sb]);
      }
      if (ok) {
        umma_commit(tfull);
      } else {
        umma_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    // warps 2-5: int8 -> f16 converters, then the TMEM read-out
    const int ct = threadIdx.x - 2 * 32;  // 0..127
    bool ok = true;
    constexpr int kUnitsPerRow = kGemvBN / 16;  // 8
    for (int i = 0; i < my_kb && ok; ++i) {
      const int s = i % SW, sb = i % kSB;
      if (!mbar_wait(&full[s], (uint32_t)((i / SW) & 1), fs) ||
          !mbar_wait(&conv_empty[sb], (uint32_t)((i / kSB) & 1) ^ 1, fs)) {
        ok = false;
        break;
      }
      const uint8_t* src = smem + L::kOffW + s * L::kWBytes;
      uint8_t* dst = smem + L::kOffB + sb * L::kBBytes;
#pragma unroll
      for (int it = 0; it < kBK * kUnitsPerRow / 128; ++it) {
        const int w = ct + it * 128;
        const int k = w / kUnitsPerRow;
        const int c16 = w - k * kUnitsPerRow;
        const uint4 raw = *reinterpret_cast<const uint4*>(src + k * kGemvBN + c16 * 16);
        uint4 o0, o1;
        i8x4_to_f16x4(raw.x, o0.x, o0.y);
        i8x4_to_f16x4(raw.y, o0.z, o0.w);
        i8x4_to_f16x4(raw.z, o1.x, o1.y);
        i8x4_to_f16x4(raw.w, o1.z, o1.w);
        store_swizzled_pair(dst, c16, k, o0, o1);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv_full[sb]);
    }
    // partial D (128 weight columns x 16 rows) -> red[m][n] in shared memory
    const int q = warp & 3;
    const int n_local = q * 32 + lane;
    bool have = my_kb > 0 && ok;
    if (have) have = mbar_wait(tfull, 0, fs);
    if (__all_sync(0xffffffffu, have)) {
      tc_fence_after();
      uint32_t r[16];
      tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(q * 32) << 16), r);
      tmem_wait_ld();
#pragma unroll
      for (int m = 0; m < kGemvRows; ++m) red[m * kGemvBN + n_local] = __uint_as_float(r[m]);
    } else {
#pragma unroll
      for (int m = 0; m < kGemvRows; ++m) red[m * kGemvBN + n_local] = 0.0f;
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 32);
  }
  // every CTA of the cluster has its partial in shared memory
  cluster_sync_all();
  if (warp >= 2) {
    // CTA `split` finishes rows m = split*2 .. split*2+1 for the 128 columns,
    // summing the KSPLIT partials in a fixed order.
    const int n_local = threadIdx.x - 2 * 32;
    const int n = n0 + n_local;
    constexpr int kRowsPerCta = kGemvRows / kGemvKSplit;
#pragma unroll
    for (int j = 0; j < kRowsPerCta; ++j) {
      const int m = split * kRowsPerCta + j;
      if (m >= args.M) continue;
      const uint32_t laddr = smem_u32(red + m * kGemvBN + n_local);
      float acc = 0.0f;
#pragma unroll
      for (int r = 0; r < kGemvKSplit; ++r) acc += ld_dsmem_f32(laddr, (uint32_t)r);
      if (n < args.N) {
        const float sc = __half2float(args.scale[n]);
        reinterpret_cast<__half*>(args.C)[(long long)m * args.ldc + n] =
            __float2half_rn(acc * sc);
      }
    }
  }
  // keep shared memory alive until every CTA has read its peers
  cluster_sync_all();
}

}  // namespace hxb
