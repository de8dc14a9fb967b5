// Decode-shaped int8-weight matmul for sm_100a (M <= 16 activation rows):
//   C[M,N] f16 = (A[M,K] f16 . W[K,N] int8) * scale[N]
//
// With M <= 16 the dispatch is bound by streaming W from HBM (45 MB for the
// BASELINE 4096 x 11008 weight): 2 FLOP per weight byte at M = 1, 32 at
// M = 16, far below the B200 ridge point. What sets the speed is how many
// bytes are in flight (about 20 MB across the GPU to approach the HBM
// ceiling) and how few instructions each byte costs on its SM:
//   * one CTA per SM owns a 96-column strip of W over the whole of K, so no
//     cross-CTA reduction and no global scratch are needed and no CTA waits
//     for a second wave (N = 11008 gives 115 CTAs);
//   * each of its warps owns a slice of K and streams it through its own
//     kGemvStages-deep shared-memory ring with cp.async: 192 KB of copies in
//     flight per CTA, no registers held by data in flight, and no warp ever
//     waits for another;
//   * each warp contracts every 16-row group with warp-level m16n8k16 MMAs
//     (f32 accumulation): A = activations (16 m x 16 k), B = weights
//     (16 k x 8 n), 12 column tiles per group;
//   * the int8 -> f16 dequantisation is exact and done in registers: a byte
//     permute pairs the same column of two weight rows, one LOP3 splices the
//     pair under the f16 exponent of 1024 with the sign bias folded in, one
//     f16x2 subtract yields the weights;
//   * every shared-memory load of a warp hits 32 distinct banks (the ring
//     images are XOR-swizzled, see gemv_w_offset / gemv_x_offset);
//   * the per-column scale is applied once after the K sum (it factors out);
//     the warps' partial sums are reduced in shared memory in a fixed order
//     (deterministic) and stored as f16.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "sm100.cuh"

namespace hxb {

constexpr int kGemvRows = 16;           // largest M served by this kernel
constexpr int kGemvSub = 3;             // 32-column sub-tiles per CTA
constexpr int kGemvBN = 32 * kGemvSub;  // weight columns per CTA
constexpr int kGemvWarps = 12;          // warps per CTA, each a slice of K
constexpr int kGemvSlotRows = 32;       // K rows per ring slot (two 16-row MMA groups)
constexpr int kGemvStages = 4;          // ring slots per warp
constexpr int kGemvThreads = kGemvWarps * 32;

struct GemvSmem {
  static constexpr int kSubBytes = kGemvSlotRows * 32;           // [32 rows][32 B] int8
  static constexpr int kWBytes = kGemvSub * kSubBytes;           // 3 KB
  static constexpr int kXBytes = kGemvRows * kGemvSlotRows * 2;  // [16 m][32 k] f16
  static constexpr int kSlotBytes = kWBytes + kXBytes;           // 4 KB
  static constexpr int kWarpBytes = kGemvStages * kSlotBytes;
  static constexpr int kBytes = kGemvWarps * kWarpBytes;         // 192 KB
  // partial sums reuse the rings: [warp][m][n] f32
  static_assert(kGemvWarps * kGemvRows * kGemvBN * 4 <= kBytes, "reduction space");
};

struct GemvArgs {
  const __half* X;  // [M, K], leading dimension ldx (elements)
  const int8_t* W;  // [K, N], leading dimension ldw (bytes)
  const __half* scale;
  __half* C;        // [M, N], leading dimension ldc
  const __half* R;  // optional residual, same layout as C: C = X.W * scale + R
  long long ldx, ldw, ldc;
  int M, N, K;
};

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mma_m16n8k16_f16_f32(float (&d)[4], const uint32_t (&a)[4],
                                                     uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// f16x2 of byte J of x (low half) and byte J of y (high half), both exact
// int8 values (|w| <= 127).
template <int J>
__device__ __forceinline__ uint32_t i8pair_to_f16x2(uint32_t x, uint32_t y) {
  uint32_t t;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(t) : "r"(x), "r"(y), "n"(((4 + J) << 8) | J));
  // {b0 ^ 0x80, 0x64, b1 ^ 0x80, 0x64} is the f16 pair 1024 + (b + 128)
  const uint32_t v = (t & 0x00FF00FFu) ^ 0x64806480u;
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(0x64806480u));
  return r;
}

// Byte offset of 16-byte chunk c (0, 1) of row r (0..31) inside a [32 rows]
// [32 B] weight sub-tile: rows are grouped four to a 128-byte line and the
// 32-byte row slots of a line are XOR-rotated by the line index, so the four
// rows 4t + r' (t = 0..3) that one load instruction reads sit in four
// different 8-bank groups.
__device__ __forceinline__ int gemv_w_offset(int row, int chunk) {
  return (row >> 2) * 128 + (((row & 3) ^ ((row >> 2) & 3)) << 5) + 16 * chunk;
}

// Byte offset of 16-byte chunk c (0..3) of activation row m inside the
// [16 m][32 k] f16 image of a slot: chunk position c ^ (2 * ((m >> 1) & 1))
// keeps the 8-byte fragment loads of each half-warp on distinct banks.
__device__ __forceinline__ int gemv_x_offset(int m, int chunk) {
  return m * 64 + ((chunk ^ (((m >> 1) & 1) << 1)) << 4);
}

// Per-lane copy plan of a ring slot (K rows [k0, k0 + 32) of the CTA's 96
// weight columns plus the matching activations), as source pointers for
// k0 = 0 and shared-memory offsets inside a slot. Copy (sub-tile s, half i)
// of a lane moves 16 bytes of weight row 16i + lane / 2, columns
// 32s + 16 (lane & 1) .. +15; activation copy i moves row m = lane / 4 + 8i,
// k 8 (lane & 3) .. +7. Rows past K, columns past N and activation rows past
// M are zero-filled by the copy itself.
template <int MROWS>
struct GemvCopyPlan {
  const int8_t* w_src;  // half 0; half 1 is 16 rows further
  uint32_t w_dst;       // half 0 of sub-tile 0; half 1 is 512 bytes further
  const __half* x_src[MROWS / 8];
  uint32_t x_dst;       // row lane / 4; row + 8 is 512 bytes further
  uint32_t x_bytes[MROWS / 8];
  int w_row, w_n, x_k;

  __device__ __forceinline__ void init(const GemvArgs& p, int n0, int lane) {
    w_row = lane >> 1;
    w_n = n0 + 16 * (lane & 1);
    w_src = p.W + (long long)w_row * p.ldw + w_n;
    w_dst = gemv_w_offset(w_row, lane & 1);
    x_k = 8 * (lane & 3);
    x_dst = GemvSmem::kWBytes + gemv_x_offset(lane >> 2, lane & 3);
#pragma unroll
    for (int i = 0; i < MROWS / 8; ++i) {
      const int m = (lane >> 2) + 8 * i;
      x_bytes[i] = m < p.M ? 16u : 0u;
      x_src[i] = m < p.M ? p.X + (long long)m * p.ldx + x_k : p.X;
    }
  }

  // Issues the copies of the slot starting at K row k0 into shared address
  // `slot`. `full` = all 32 rows inside K and all 96 columns inside N.
  __device__ __forceinline__ void issue(const GemvArgs& p, uint32_t slot, int k0, bool full) const {
    if (full) {
      const int8_t* s0 = w_src + (long long)k0 * p.ldw;
      const int8_t* s1 = s0 + 16 * p.ldw;
#pragma unroll
      for (int s = 0; s < kGemvSub; ++s) {
        cp_async_16(slot + w_dst + s * GemvSmem::kSubBytes, s0 + 32 * s, 16u);
        cp_async_16(slot + w_dst + s * GemvSmem::kSubBytes + 512, s1 + 32 * s, 16u);
      }
#pragma unroll
      for (int i = 0; i < MROWS / 8; ++i)
        cp_async_16(slot + x_dst + 512 * i, x_bytes[i] ? x_src[i] + k0 : p.X, x_bytes[i]);
    } else {
#pragma unroll
      for (int s = 0; s < kGemvSub; ++s)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int k = k0 + w_row + 16 * i, n = w_n + 32 * s;
          const bool ok = k < p.K && n < p.N;
          cp_async_16(slot + w_dst + s * GemvSmem::kSubBytes + 512 * i,
                      ok ? p.W + (long long)k * p.ldw + n : p.W, ok ? 16u : 0u);
        }
#pragma unroll
      for (int i = 0; i < MROWS / 8; ++i) {
        const int k = k0 + x_k;
        const uint32_t bytes = (x_bytes[i] && k < p.K) ? (uint32_t)(min(8, p.K - k) * 2) : 0u;
        cp_async_16(slot + x_dst + 512 * i, bytes ? x_src[i] + k0 : p.X, bytes);
      }
    }
  }
};

// MROWS = 8 serves M <= 8 (activation rows 8..15 of the MMA are zero and are
// neither copied nor read), MROWS = 16 serves M <= 16.
template <int MROWS>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_w8_kernel(const GemvArgs p) {
  using L = GemvSmem;
  extern __shared__ __align__(16) uint8_t gemv_smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * kGemvBN;
  const int slots = (p.K + kGemvSlotRows - 1) / kGemvSlotRows;
  const int sb = (int)((long long)warp * slots / kGemvWarps);
  const int se = (int)((long long)(warp + 1) * slots / kGemvWarps);
  const int ns = se - sb;
  const bool n_full = n0 + kGemvBN <= p.N;
  uint8_t* ring = gemv_smem + warp * L::kWarpBytes;
  const uint32_t ring_s = smem_u32(ring);

  GemvCopyPlan<MROWS> plan;
  plan.init(p, n0, lane);
  auto slot_full = [&](int si) { return n_full && (sb + si + 1) * kGemvSlotRows <= p.K; };

  float acc[kGemvSub][4][4];
#pragma unroll
  for (int s = 0; s < kGemvSub; ++s)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[s][j][e] = 0.0f;

  // Lane offsets of the weight words (word g of row 4t + r of a 16-row group,
  // see gemv_w_offset) and of the activation fragments (rows g and g + 8,
  // physical k 4t .. 4t+3 of each group) inside a slot.
  uint32_t woff[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) woff[r] = gemv_w_offset(4 * t + r, g >> 2) + 4 * (g & 3);
  uint32_t xoff[2];
#pragma unroll
  for (int grp = 0; grp < 2; ++grp)
    xoff[grp] = L::kWBytes + gemv_x_offset(g, (t >> 1) + 2 * grp) + 8 * (t & 1);

  // prologue: kGemvStages - 1 slots in flight (one commit group each; empty
  // groups past the end keep the wait counts uniform)
#pragma unroll
  for (int s = 0; s < kGemvStages - 1; ++s) {
    if (s < ns) plan.issue(p, ring_s + s * L::kSlotBytes, (sb + s) * kGemvSlotRows, slot_full(s));
    cp_async_commit();
  }
  for (int i0 = 0; i0 < ns; i0 += kGemvStages) {
#pragma unroll
    for (int s = 0; s < kGemvStages; ++s) {
      const int i = i0 + s;
      if (i >= ns) break;
      {
        // refill the slot the previous iteration finished with
        const int f = i + kGemvStages - 1;
        if (f < ns)
          plan.issue(p, ring_s + ((s + kGemvStages - 1) % kGemvStages) * L::kSlotBytes,
                     (sb + f) * kGemvSlotRows, slot_full(f));
        cp_async_commit();
      }
      cp_async_wait<kGemvStages - 1>();
      __syncwarp();
      const uint8_t* st = ring + s * L::kSlotBytes;
#pragma unroll
      for (int grp = 0; grp < kGemvSlotRows / 16; ++grp) {
        // A fragment {a0a1, a2a3, a4a5, a6a7} = {(m g, k 2t..2t+1), (m g+8, ..),
        // (m g, k 2t+8..2t+9), (m g+8, ..)}; logical k 2t, 2t+1 <-> physical
        // 4t, 4t+1 and 2t+8, 2t+9 <-> 4t+2, 4t+3
        const uint2 xa = *reinterpret_cast<const uint2*>(st + xoff[grp]);
        uint2 xb = make_uint2(0u, 0u);
        if (MROWS == 16) xb = *reinterpret_cast<const uint2*>(st + xoff[grp] + 8 * 64);
        const uint32_t a[4] = {xa.x, xb.x, xa.y, xb.y};
#pragma unroll
        for (int sub = 0; sub < kGemvSub; ++sub) {
          uint32_t w[4];
#pragma unroll
          for (int r = 0; r < 4; ++r)
            w[r] = *reinterpret_cast<const uint32_t*>(st + sub * L::kSubBytes + 512 * grp + woff[r]);
          mma_m16n8k16_f16_f32(acc[sub][0], a, i8pair_to_f16x2<0>(w[0], w[1]),
                               i8pair_to_f16x2<0>(w[2], w[3]));
          mma_m16n8k16_f16_f32(acc[sub][1], a, i8pair_to_f16x2<1>(w[0], w[1]),
                               i8pair_to_f16x2<1>(w[2], w[3]));
          mma_m16n8k16_f16_f32(acc[sub][2], a, i8pair_to_f16x2<2>(w[0], w[1]),
                               i8pair_to_f16x2<2>(w[2], w[3]));
          mma_m16n8k16_f16_f32(acc[sub][3], a, i8pair_to_f16x2<3>(w[0], w[1]),
                               i8pair_to_f16x2<3>(w[2], w[3]));
        }
      }
      __syncwarp();  // every lane has read the slot before it is refilled
    }
  }
  cp_async_wait<0>();

  // partial sums -> shared memory -> fixed-order reduction over the warps ->
  // scale, store
  __syncthreads();
  float* red = reinterpret_cast<float*>(gemv_smem);  // [warp][m][n]
  {
    // D: d0, d1 = (m g, tile column 2t, 2t+1), d2, d3 = (m g+8, ...); in tile
    // (sub, j), column c is weight column 32 sub + 4c + j
    float* base = red + warp * (kGemvRows * kGemvBN);
#pragma unroll
    for (int sub = 0; sub < kGemvSub; ++sub)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float* d = acc[sub][j];
        const int nA = 32 * sub + 8 * t + j, nB = nA + 4;
        base[g * kGemvBN + nA] = d[0];
        base[g * kGemvBN + nB] = d[1];
        base[(g + 8) * kGemvBN + nA] = d[2];
        base[(g + 8) * kGemvBN + nB] = d[3];
      }
  }
  __syncthreads();
  for (int o = threadIdx.x; o < kGemvRows * kGemvBN; o += kGemvThreads) {
    const int m = o / kGemvBN, nl = o % kGemvBN;
    const int n = n0 + nl;
    if (m >= p.M || n >= p.N) continue;
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < kGemvWarps; ++w) sum += red[w * (kGemvRows * kGemvBN) + o];
    const long long off = (long long)m * p.ldc + n;
    const float rv = p.R ? __half2float(p.R[off]) : 0.0f;
    p.C[off] = __float2half_rn(fmaf(sum, __half2float(p.scale[n]), rv));
  }
}

}  // namespace hxb
