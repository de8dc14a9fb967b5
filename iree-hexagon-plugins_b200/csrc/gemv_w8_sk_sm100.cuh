// Decode-shaped int8-weight matmul over every SM (M <= 16 activation rows):
//   C[M,N] f16 = (A[M,K] f16 . W[K,N] int8) * scale[N] (+ R)
//
// The dispatch streams W (45 MB at BASELINE configuration 2) once from HBM;
// it is bound by how evenly and how cheaply that stream is spread over the
// SMs. This kernel:
//   * cuts W into tiles of 64 k rows x 256 columns (two 128-byte TMA boxes:
//     256-byte row segments) and hands every SM an equal run of tiles in
//     (column strip, k) order, so all SMs stream the same number of bytes
//     whatever N is;
//   * a run that starts inside a strip contributes a partial sum for it: the
//     SM holding the strip's first tile adds the other SMs' partials (in SM
//     order, deterministic). Every SM works its run from its first strip
//     start to the end, then the leading tiles it contributes, so partials
//     are published when an SM is done streaming and every SM completes its
//     shared strip after its own last tile;
//   * one producer thread keeps a 4-stage TMA ring of weight tiles (and the
//     matching 64-k slice of the activations) in flight, 72 KB per CTA
//     (4, 5 and 6 stages measured within 1 % of each other, 8 stages 5 %
//     slower). One CTA per SM: its registers fill an SM sub-partition's
//     share, so the next launch's CTAs start as this launch's CTAs exit;
//   * eight consumer warps each own 32 columns of a strip and contract with
//     warp-level MMAs in the swapped orientation D[n, m] = W^T[n, k] X^T[k, m]:
//     one m16n8k16 consumes 256 weights, and ldmatrix.trans hands every lane
//     the (k, k+1) byte pairs of two neighbouring columns, so the exact
//     int8 -> f16 conversion is a mask, an exponent splice and one f16x2
//     subtract per pair of weights.
// Cross-SM publication uses one bit per consumer warp in a per-SM flag word:
// warp w of the finishing SM reads only what warp w of the contributing SM
// wrote, so no CTA-wide barrier is needed, and it clears the bit after
// reading (the flags are zero again when the dispatch ends).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "gemm_w8_sm100.cuh"
#include "sm100.cuh"

namespace hxb {

constexpr int kGsBK = 64;                         // k rows per tile
constexpr int kGsBN = 256;                        // weight columns per strip
constexpr int kGsStages = 4;                      // TMA ring stages
constexpr int kGsConsumers = 8;                   // consumer warps, 32 columns each
constexpr int kGsThreads = 32 * (1 + kGsConsumers);
constexpr int kGsWBox = kGsBK * 128;              // one [64 k][128 B] weight box
constexpr int kGsXBox = 16 * kGsBK * 2;           // [16 m][64 k] f16 activations
constexpr int kGsStageBytes = 2 * kGsWBox + kGsXBox;
constexpr int kGsPartialFloats = kGsConsumers * 2 * 2 * 32 * 4;  // per SM: 16 KB
static_assert(kGsStageBytes % 1024 == 0, "stages stay 1024-byte aligned (128-byte swizzle)");
static_assert(kGsPartialFloats <= kW8PartialFloats, "partials fit the stream-K workspace");

struct GsSmem {
  static constexpr int kOffBar = kGsStages * kGsStageBytes;
  static constexpr int kOffMisc = kOffBar + 2 * kGsStages * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

struct GsArgs {
  const __half* scale;
  __half* C;
  const __half* R;  // optional residual, same layout as C
  long long ldc;
  int M, N, K;
  int kc;           // k tiles per strip
  int tiles;        // strips * kc
  int ctas;
  int* flags;       // [ctas] words, zero at rest
  float* partials;  // [ctas][kGsPartialFloats]
  int* status;
};

// Processing order of SM b's run [u0, u1): the tiles from the first strip
// start inside the run (rot) to its end, then the run's leading tiles, which
// finish a strip begun by an earlier SM. The partial sum those leading tiles
// contribute is therefore published when the SM has no tiles left (its
// stores never hold up the ring), and the one strip this SM must complete
// with other SMs' partials is the last one it finishes.
struct GsOrder {
  int u0, u1, rot;
  __device__ __forceinline__ int tile(int i) const {
    return i < u1 - rot ? rot + i : u0 + (i - (u1 - rot));
  }
};

// First tile of SM b's run, and the SM whose run holds tile u.
__device__ __forceinline__ int gs_begin(int b, const GsArgs& a) {
  return (int)((long long)b * a.tiles / a.ctas);
}
__device__ __forceinline__ int gs_owner(int u, const GsArgs& a) {
  return (int)(((long long)(u + 1) * a.ctas - 1) / a.tiles);
}

__device__ __forceinline__ void ldsm_x4_trans_b16(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// f16x2 of bytes 0 and 2 (lo) or 1 and 3 (hi) of `raw`, exact int8 values:
// {b ^ 0x80, 0x64} is the f16 1024 + (b + 128), minus 1152.
__device__ __forceinline__ uint32_t i8_lo_pair(uint32_t raw) {
  const uint32_t v = (raw & 0x00FF00FFu) ^ 0x64806480u;
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(0x64806480u));
  return r;
}
__device__ __forceinline__ uint32_t i8_hi_pair(uint32_t raw) {
  const uint32_t v = ((raw >> 8) & 0x00FF00FFu) ^ 0x64806480u;
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(0x64806480u));
  return r;
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// *p |= v with release semantics at GPU scope: every write this thread has
// observed (the whole warp's partial stores, ordered by the preceding
// __syncwarp) is visible before the bit.
__device__ __forceinline__ void red_or_release_gpu(int* p, int v) {
  asm volatile("red.release.gpu.global.or.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until `bit` of *flag is set (by the same warp of another SM).
__device__ __forceinline__ bool gs_wait_bit(const int* flag, int bit, const FailState& fs) {
  if (ld_acquire_gpu(flag) & bit) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i) {
      if (ld_acquire_gpu(flag) & bit) return true;
      __nanosleep(128);
    }
    if (*fs.abort) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_failure(fs);
      return false;
    }
  }
}

// MT = 1 serves M <= 8 (one 8-row activation group), MT = 2 serves M <= 16.
template <int MT>
__global__ void __launch_bounds__(kGsThreads, 1)
    gemv_w8_sk_kernel(const __grid_constant__ CUtensorMap tmW,
                      const __grid_constant__ CUtensorMap tmX, const GsArgs a) {
  using L = GsSmem;
  extern __shared__ uint8_t gs_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(gs_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* empty = full + kGsStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  const int u0 = gs_begin(b, a), u1 = gs_begin(b + 1, a);
  const GsOrder order{u0, u1, min(u1, (u0 + a.kc - 1) / a.kc * a.kc)};
  const int n = u1 - u0;
  const FailState fs{abort_flag, a.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGsStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGsConsumers);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      // The weights of the first stages are requested before waiting for the
      // previous kernel of the stream (no dispatch of this library writes
      // int8 weights); the activations, which that kernel may produce, after.
      const int pre = min(n, kGsStages);
      for (int i = 0; i < pre; ++i) {
        const int u = order.tile(i);
        const int s = u / a.kc, j = u - s * a.kc;
        uint8_t* st = smem + i * kGsStageBytes;
        mbar_arrive_expect_tx(&full[i], kGsStageBytes);
        tma_load_2d(st, &tmW, &full[i], s * kGsBN, j * kGsBK);
        tma_load_2d(st + kGsWBox, &tmW, &full[i], s * kGsBN + 128, j * kGsBK);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(smem + i * kGsStageBytes + 2 * kGsWBox, &tmX, &full[i],
                    order.tile(i) % a.kc * kGsBK, 0);
      int stage = pre % kGsStages, issued = pre;
      uint32_t phase = pre == kGsStages ? 1u : 0u;
      for (int i = pre; i < n; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1, fs)) break;
        const int u = order.tile(i);
        const int s = u / a.kc, j = u - s * a.kc;
        uint8_t* st = smem + stage * kGsStageBytes;
        mbar_arrive_expect_tx(&full[stage], kGsStageBytes);
        tma_load_2d(st, &tmW, &full[stage], s * kGsBN, j * kGsBK);
        tma_load_2d(st + kGsWBox, &tmW, &full[stage], s * kGsBN + 128, j * kGsBK);
        tma_load_2d(st + 2 * kGsWBox, &tmX, &full[stage], j * kGsBK, 0);
        ++issued;
        if (++stage == kGsStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // bounded wait for the copies still landing (complete on the normal path)
      for (int i = 0; i < issued && i < kGsStages; ++i) {
        if (stage == 0) {
          stage = kGsStages - 1;
          phase ^= 1u;
        } else {
          --stage;
        }
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[stage], phase) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - 1;                 // columns [32 cw, 32 cw + 32) of a strip
  const int g = lane >> 2, tq = lane & 3;  // MMA fragment coordinates
  const int bit = 1 << cw;
  // ldmatrix row address of this lane inside a 32-k half of chunk ch:
  // matrix lane / 8 is k rows 8 (lane / 8) .., row lane % 8
  const int lrow = 8 * (lane >> 3) + (lane & 7);
  uint32_t woff[2][2];  // [k half][chunk]
#pragma unroll
  for (int kh = 0; kh < 2; ++kh)
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      const int cg = 2 * cw + ch;  // 16-column chunk 0..15 of the strip
      const int k = 32 * kh + lrow;
      woff[kh][ch] = (cg >> 3) * kGsWBox + k * 128 + (((cg & 7) ^ (k & 7)) << 4);
    }
  // activation fragment offsets: row g (+8), k pair 2 tq (+8) of k-step ks
  uint32_t xoff[4][MT][2];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int row = g + 8 * mt;
#pragma unroll
      for (int h = 0; h < 2; ++h)
        xoff[ks][mt][h] = 2 * kGsWBox + row * 128 + (((2 * ks + h) ^ (row & 7)) << 4) + 4 * tq;
    }

  float acc[2][MT][4];
  auto clear = [&] {
#pragma unroll
    for (int ch = 0; ch < 2; ++ch)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[ch][mt][e] = 0.0f;
  };
  clear();
  const size_t frag0 = (size_t)cw * 2 * MT * 32;  // this warp's float4 fragments in a partial
  float4* my_part = reinterpret_cast<float4*>(a.partials + (size_t)b * kGsPartialFloats);

  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;

  // C = acc * scale (+ R) for strip s; D rows g / g + 8 are columns n0 /
  // n0 + 1, columns 2 tq / 2 tq + 1 are activation rows. The scale and
  // residual operands are loaded first (epi_load), so the finisher of a
  // shared strip has them in registers before it waits for the partials.
  struct EpiIn {
    float sc[2][2];         // [chunk][column n0, n0 + 1]
    float r[2][MT][2][2];   // [chunk][mt][e][column]
  };
  auto epi_load = [&](int s, EpiIn& in) {
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      const int n0 = s * kGsBN + 32 * cw + 16 * ch + 2 * g;
      const bool one = n0 < a.N, two = n0 + 1 < a.N;
      in.sc[ch][0] = one ? __half2float(a.scale[n0]) : 0.0f;
      in.sc[ch][1] = two ? __half2float(a.scale[n0 + 1]) : 0.0f;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int m = 8 * mt + 2 * tq + e;
          const long long off = (long long)m * a.ldc + n0;
          const bool row = m < a.M && a.R;
          in.r[ch][mt][e][0] = row && one ? __half2float(a.R[off]) : 0.0f;
          in.r[ch][mt][e][1] = row && two ? __half2float(a.R[off + 1]) : 0.0f;
        }
    }
  };
  auto epi_store = [&](const float (&v)[2][MT][4], int s, const EpiIn& in) {
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      const int n0 = s * kGsBN + 32 * cw + 16 * ch + 2 * g;
      if (n0 >= a.N) continue;
      const bool two = n0 + 1 < a.N;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int m = 8 * mt + 2 * tq + e;
          if (m >= a.M) continue;
          const long long off = (long long)m * a.ldc + n0;
          const float v0 = fmaf(v[ch][mt][e], in.sc[ch][0], in.r[ch][mt][e][0]);
          const float v1 = fmaf(v[ch][mt][2 + e], in.sc[ch][1], in.r[ch][mt][e][1]);
          if (two && (off & 1) == 0) {
            *reinterpret_cast<__half2*>(a.C + off) = __floats2half2_rn(v0, v1);
          } else {
            a.C[off] = __float2half_rn(v0);
            if (two) a.C[off + 1] = __float2half_rn(v1);
          }
        }
    }
  };

  float held[2][MT][4];  // the strip finished last, completed with others' partials
  int held_s = -1;
  int seg_j0 = 0;        // k tile at which the current segment started
  bool new_seg = true;
  for (int i = 0; i < n && ok; ++i) {
    const int u = order.tile(i);
    const int s = u / a.kc, j = u - s * a.kc;
    if (new_seg) {
      seg_j0 = j;
      new_seg = false;
    }
    if (!mbar_wait(&full[stage], phase, fs)) {
      ok = false;
      break;
    }
    const uint32_t st = smem_u32(smem + stage * kGsStageBytes);
    uint32_t xb[4][MT][2];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) xb[ks][mt][h] = lds32(st + xoff[ks][mt][h]);
#pragma unroll
    for (int kh = 0; kh < 2; ++kh)
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        uint32_t raw[4];
        ldsm_x4_trans_b16(st + woff[kh][ch], raw);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          // A rows: g <-> column 2g of the chunk (bytes 0, 2), g + 8 <-> 2g + 1
          const uint32_t a0 = i8_lo_pair(raw[2 * h]), a1 = i8_hi_pair(raw[2 * h]);
          const uint32_t a2 = i8_lo_pair(raw[2 * h + 1]), a3 = i8_hi_pair(raw[2 * h + 1]);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            mma_16816(acc[ch][mt], a0, a1, a2, a3, xb[2 * kh + h][mt][0], xb[2 * kh + h][mt][1]);
        }
      }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == kGsStages) {
      stage = 0;
      phase ^= 1u;
    }

    if (j != a.kc - 1 && i != (u1 - order.rot) - 1 && i != n - 1) continue;
    // ----------------------------------------------- end of a strip segment
    new_seg = true;
    if (seg_j0 != 0) {
      // contributor (the run's leading tiles, processed last): publish this
      // warp's fragments, then its bit
#pragma unroll
      for (int ch = 0; ch < 2; ++ch)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          __stcg(my_part + frag0 + (ch * MT + mt) * 32 + lane,
                 make_float4(acc[ch][mt][0], acc[ch][mt][1], acc[ch][mt][2], acc[ch][mt][3]));
      __syncwarp();
      if (lane == 0) red_or_release_gpu(a.flags + b, bit);
    } else if (j == a.kc - 1) {
      EpiIn in;  // a whole strip inside this run
      epi_load(s, in);
      epi_store(acc, s, in);
    } else {
#pragma unroll
      for (int ch = 0; ch < 2; ++ch)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int e = 0; e < 4; ++e) held[ch][mt][e] = acc[ch][mt][e];
      held_s = s;
    }
    clear();
  }
  if (!ok || held_s < 0) return;
  EpiIn held_in;
  epi_load(held_s, held_in);

  // finisher of strip held_s: add the partials of the SMs holding the rest of
  // it. The flags of up to 32 contributors are polled at once (lane i polls
  // contributor i of the group), their partials are loaded together and then
  // added in SM order: two memory round trips per group.
  const int last = gs_owner(min((held_s + 1) * a.kc, a.tiles) - 1, a);
  for (int c0 = b + 1; c0 <= last; c0 += 32) {
    const int nc = min(32, last - c0 + 1);
    bool ready = true;
    if (lane < nc) ready = gs_wait_bit(a.flags + c0 + lane, bit, fs);
    // the warp barrier of __all_sync orders every lane's reads after the
    // polling lanes' acquires
    if (!__all_sync(0xffffffffu, ready)) return;
    for (int i = 0; i < nc; i += 4) {
      float4 v[4][2][MT];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (i + q < nc) {
          const float4* part = reinterpret_cast<const float4*>(
              a.partials + (size_t)(c0 + i + q) * kGsPartialFloats);
#pragma unroll
          for (int ch = 0; ch < 2; ++ch)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
              v[q][ch][mt] = __ldcg(part + frag0 + (ch * MT + mt) * 32 + lane);
        }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (i + q < nc) {
#pragma unroll
          for (int ch = 0; ch < 2; ++ch)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              held[ch][mt][0] += v[q][ch][mt].x;
              held[ch][mt][1] += v[q][ch][mt].y;
              held[ch][mt][2] += v[q][ch][mt].z;
              held[ch][mt][3] += v[q][ch][mt].w;
            }
        }
    }
    __syncwarp();
    if (lane < nc) atomicAnd(a.flags + c0 + lane, ~bit);
  }
  epi_store(held, held_s, held_in);
}

}  // namespace hxb
