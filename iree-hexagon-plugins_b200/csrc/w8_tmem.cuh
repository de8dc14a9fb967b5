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
// The transpose is done by the shared-memory load itself: ldmatrix.trans on
// 8 x 8 matrices of 16-bit elements, where one element is a pair of
// neighbouring int8 columns (n, n+1) of one k row. Matrix g of a 16-column
// chunk is rows k = 8g .. 8g+7 (consecutive rows, so its eight 16-byte rows
// sit in eight different bank groups under the swizzle); lane t receives
// {W[k][n0], W[k][n0+1], W[k+1][n0], W[k+1][n0+1]} with k = 8g + 2(t % 4) and
// n0 = 16c + 2(t / 4). Bytes 0 and 2 are the f16 pair of column n0 for
// k-pair column 4g + t % 4, bytes 1 and 3 that of column n0 + 1, which is
// exactly the register layout of tcgen05.st.16x128b: lane t writes TMEM lanes
// t/4 (column n0) and t/4 + 8 (column n0 + 1) at column t % 4 + 4g.
//
// Hence, within the 16 TMEM lanes L0 .. L0+15 that hold chunk c, lane L0 + i
// holds weight column 16c + 2i for i < 8 and 16c + 2(i - 8) + 1 for i >= 8;
// warp quarter q holds chunks 2q (lanes 32q .. 32q+15) and 2q + 1.
#pragma once

#include "sm100.cuh"

namespace hxb {

// Weight column (0..127 within the tile) held by TMEM lane `l` (0..127).
__host__ __device__ __forceinline__ int w8_lane_to_col(int l) {
  const int i = l & 15;
  return 16 * (l >> 4) + (i < 8 ? 2 * i : 2 * (i - 8) + 1);
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void tmem_st_16x128b_x8(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x128b.x8.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// 16 TMEM lanes x 32 columns: lane t receives, for repetition r = 0..3,
// {lane t/4: columns 8r + 2(t%4), +1; lane t/4 + 8: the same columns} in
// registers 4r .. 4r+3.
__device__ __forceinline__ void tmem_ld_16x256b_x4(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Inverse of tmem_ld_16x256b_x4: writes the same register layout back.
__device__ __forceinline__ void tmem_st_16x256b_x4(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// Converts the 16-column chunk `chunk` (columns 16c .. 16c+15, all 64 k rows)
// of one int8 tile into the 32 TMEM columns starting at `tmem_col` of the 16
// TMEM lanes starting at lane `lane0` (a multiple of 16 inside this warp's
// lane quarter). Called by a whole warp. Ends with the TMEM store issued (the
// caller waits with tmem_wait_st()).
__device__ __forceinline__ void w8_chunk_to_tmem(uint32_t tile_s, uint32_t tmem_base, int lane0,
                                                 uint32_t tmem_col, int chunk, int lane) {
  // lane t addresses row (t % 8) of matrix t / 8 of each 4-matrix load
  const int mrow = lane & 7, mat = lane >> 3;
  uint32_t raw[8];
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int k = 8 * (4 * s + mat) + mrow;
    uint32_t r4[4];
    ldsm_x4_trans(tile_s + k * 128 + ((chunk ^ (k & 7)) << 4), r4);
#pragma unroll
    for (int i = 0; i < 4; ++i) raw[4 * s + i] = r4[i];
  }
  uint32_t out[16];
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    // bytes {0, 2}: column n0, bytes {1, 3}: column n0 + 1; each as
    // {b ^ 0x80, 0x64} = f16 1024 + (b + 128), minus 1152 -> exact b
    const uint32_t lo = (raw[g] & 0x00FF00FFu) ^ 0x64806480u;
    const uint32_t hi = ((raw[g] >> 8) & 0x00FF00FFu) ^ 0x64806480u;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(out[2 * g]) : "r"(lo), "r"(0x64806480u));
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(out[2 * g + 1]) : "r"(hi), "r"(0x64806480u));
  }
  tmem_st_16x128b_x8(tmem_base + ((uint32_t)lane0 << 16) + tmem_col, out);
}

// Converts NC consecutive 16-column chunks (chunk0, chunk0 + 1, ...) of one
// int8 tile into TMEM lanes lane0 + 16 c (c = 0 .. NC-1), columns [tmem_col,
// tmem_col + 32). All shared-memory loads are issued before the arithmetic so
// that their latencies overlap. Ends with the TMEM stores issued (the caller
// waits with tmem_wait_st()).
template <int NC>
__device__ __forceinline__ void w8_chunks_to_tmem(uint32_t tile_s, uint32_t tmem_base, int lane0,
                                                  uint32_t tmem_col, int chunk0, int lane) {
  const int mrow = lane & 7, mat = lane >> 3;
  uint32_t raw[NC][8];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int k = 8 * (4 * s + mat) + mrow;
      uint32_t r4[4];
      ldsm_x4_trans(tile_s + k * 128 + (((chunk0 + c) ^ (k & 7)) << 4), r4);
#pragma unroll
      for (int i = 0; i < 4; ++i) raw[c][4 * s + i] = r4[i];
    }
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    uint32_t out[16];
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const uint32_t lo = (raw[c][g] & 0x00FF00FFu) ^ 0x64806480u;
      const uint32_t hi = ((raw[c][g] >> 8) & 0x00FF00FFu) ^ 0x64806480u;
      asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(out[2 * g]) : "r"(lo), "r"(0x64806480u));
      asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(out[2 * g + 1]) : "r"(hi), "r"(0x64806480u));
    }
    tmem_st_16x128b_x8(tmem_base + ((uint32_t)(lane0 + 16 * c) << 16) + tmem_col, out);
  }
}

}  // namespace hxb
