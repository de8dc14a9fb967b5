// Int8 weight tiles -> f16 tcgen05 A operand in TMEM (used by the W8 GEMM).
//
// The weights are W[K,N] int8, row-major (N contiguous). The kernel computes
// the transposed product D[n, m] = sum_k W[k, n] * X[m, k] so that the weight
// tile is the 128-row MMA operand A, read from TMEM: TMEM lane l holds one
// weight column n(l), each 32-bit TMEM column two consecutive k (lower k in
// the low half). The f16 tile therefore never touches shared memory; only the
// raw int8 tile does (written once by TMA, read once here).
//
// A weight tile in shared memory is [64 k rows][128 n bytes], loaded by TMA
// with the 128-byte swizzle: 16-byte chunk c of row k sits at chunk position
// c ^ (k & 7).
//
// Converter mapping (warps of TMEM lane quarter q, lane t = 4a + b):
//   * the four lanes a*4 + {0..3} cover one 4-byte word of n values and four
//     consecutive k rows; lane b loads row 4i+b of that word, then a 4x4 byte
//     transpose (two xor-shuffles and two byte permutes) leaves lane b with
//     rows 4i..4i+3 of the single column n = word + b;
//   * warp q covers 16-byte chunks q and q+4, so the 8 words one load
//     instruction reads from 4 rows land in 8 distinct bank groups;
//   * hence TMEM lane 32q + 4a + b holds weight column
//       n(l) = (a < 4 ? 16q + 4a : 64 + 16q + 4(a-4)) + b,
//     a fixed permutation the epilogue undoes.
#pragma once

#include "sm100.cuh"

namespace hxb {

// Weight column (0..127 within the tile) held by TMEM lane `l` (0..127).
__host__ __device__ __forceinline__ int w8_lane_to_col(int l) {
  const int q = l >> 5, t = l & 31, a = t >> 2, b = t & 3;
  return (a < 4 ? 16 * q + 4 * a : 64 + 16 * q + 4 * (a - 4)) + b;
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// Converts k rows [4 * I0, 4 * (I0 + NI)) of one [64 k][128 n] int8 tile
// (swizzled, see above) into the 2 * NI TMEM columns starting at
// `tmem_col + 2 * I0` of this warp's lane quarter: column j holds the f16
// pair (W[2j][n], W[2j+1][n]) for the lane's weight column n. Called by a
// whole warp; `quarter` = warp index % 4. Ends with the TMEM stores issued
// (the caller waits with tmem_wait_st()). All loads are issued before the
// first shuffle so their latencies overlap.
template <int I0, int NI>
__device__ __forceinline__ void w8_rows_to_tmem(const uint8_t* tile, uint32_t tmem_lane_base,
                                                uint32_t tmem_col, int quarter, int lane) {
  static_assert(NI == 8 || NI == 16, "8 or 16 row quads");
  const int a = lane >> 2, b = lane & 3;
  const int chunk = a < 4 ? quarter : quarter + 4;
  const int word = (a & 3) * 4;
  // prmt selectors of the two transpose stages
  const uint32_t sel1 = (b & 1) ? 0x3715u : 0x6240u;
  const uint32_t sel2 = (b & 2) ? 0x3276u : 0x5410u;
  uint32_t x[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int k = 4 * (I0 + i) + b;
    x[i] = *reinterpret_cast<const uint32_t*>(tile + k * 128 + ((chunk ^ (k & 7)) << 4) + word);
  }
  uint32_t out[2 * NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    // stage 1: 2x2 byte blocks with the neighbouring row
    const uint32_t y = __shfl_xor_sync(0xffffffffu, x[i], 1);
    uint32_t s1;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(s1) : "r"(x[i]), "r"(y), "r"(sel1));
    // stage 2: 16-bit halves with the row pair two lanes away
    const uint32_t z = __shfl_xor_sync(0xffffffffu, s1, 2);
    uint32_t col;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(col) : "r"(s1), "r"(z), "r"(sel2));
    // col = {W[4i][n], W[4i+1][n], W[4i+2][n], W[4i+3][n]}
    i8x4_to_f16x4(col, out[2 * i], out[2 * i + 1]);
  }
  if constexpr (NI == 16) {
    tmem_st_32x32b_x32(tmem_lane_base + tmem_col + 2 * I0, out);
  } else {
    tmem_st_32x32b_x16(tmem_lane_base + tmem_col + 2 * I0, out);
  }
}

}  // namespace hxb
