// Tile planner for the tcgen05 GEMM dispatches: the B200 counterpart of the
// reference's HMX VTCM tile search (plugins/compiler/hexagon/CodeGen/Strategy/
// Planning/VTCMPlanning.cpp:186-260). Where the reference enumerates
// HMX-aligned divisors of M and N under a 2 MiB VTCM budget and ranks them by
// (over budget, DDR<->VTCM traffic, #tiles, -N), this one enumerates the
// tcgen05 tile widths whose shared-memory ring fits the 227 KB per-CTA budget
// and ranks them by (estimated time on the persistent grid, traffic, -N).
// Shapes measured by the offline sweep are answered from the baked table
// first.
#pragma once

#include <stdint.h>

namespace hxb {

struct GemmPlan {
  int block_n;    // N extent of one output tile
  int group_m;    // tile-rows per raster group (L2 reuse)
  int split = 1;  // 1: persistent kernel; 2, 4, 8: K split over a cluster
  int pair = 1;   // 1: 128-row tiles on one SM; 2: 256-row tiles on a CTA pair
};

struct TunedGemm {
  int M, N, K, bmode;
  int block_n, group_m;
  int split;  // 0 or 1: no split
  int pair;   // 0 or 1: one CTA per tile; 2: CTA pair
};

// Filled by the offline tile sweep (tile_table.inc); may be empty.
extern const TunedGemm kTunedGemms[];
extern const int kNumTunedGemms;

// Cycles one SM spends on a 128 x bn x 16 tcgen05.mma: the tensor pipe does
// 128x256x16 in 128 cycles; narrow tiles are bounded by shared-memory operand
// reads (A 4 KB + B bn*32 B at 128 B/cycle).
inline int64_t mma_cycles(int bn) {
  const int64_t tensor = bn / 2;
  const int64_t smem = (4096 + (int64_t)bn * 32) / 128;
  return tensor > smem ? tensor : smem;
}

// Cycles one SM spends bringing one K-block of operands (A 16 KB + B bn *
// 128 B) from L2 into shared memory: ~48 B/cycle per SM when every SM
// streams at once.
inline int64_t load_cycles(int bn) { return (16384 + (int64_t)bn * 128) / 48; }

// The same for one CTA of a pair (256 x bn tiles on two SMs): A 16 KB plus
// half of B.
inline int64_t load_cycles_pair(int bn) { return (16384 + (int64_t)bn * 64) / 48; }

// Largest split-K a shape takes: every CTA keeps at least two K-blocks, and
// the tiles x split CTAs fit one wave (clusters are co-scheduled; a GPC's
// SMs are not always all usable by clusters, hence the 7/8).
inline bool split_fits(int64_t tiles, int64_t kb, int split, int num_sms) {
  return kb >= 2 * split && tiles * split <= (int64_t)num_sms * 7 / 8;
}

inline GemmPlan plan_gemm(int M, int N, int K, int bmode, int num_sms) {
  for (int i = 0; i < kNumTunedGemms; ++i) {
    const TunedGemm& t = kTunedGemms[i];
    if (t.M == M && t.N == N && t.K == K && t.bmode == bmode)
      return GemmPlan{t.block_n, t.group_m, t.split > 1 ? t.split : 1, t.pair > 1 ? 2 : 1};
  }
  const int cands[3] = {256, 128, 64};
  const int splits[4] = {1, 2, 4, 8};
  const int64_t tiles_m = (M + 127) / 128;
  const int64_t kb = (K + 63) / 64;
  GemmPlan best{cands[0], 8, 1};
  int64_t best_cost = -1, best_traffic = -1;
  for (int i = 0; i < 3; ++i) {
    const int bn = cands[i];
    const int64_t tiles = tiles_m * ((N + bn - 1) / bn);
    const int64_t per_kb =
        4 * mma_cycles(bn) > load_cycles(bn) ? 4 * mma_cycles(bn) : load_cycles(bn);
    for (int j = 0; j < 4; ++j) {
      const int split = splits[j];
      if (split > 1 && !split_fits(tiles, kb, split, num_sms)) continue;
      int64_t cost;
      if (split == 1) {
        const int64_t waves = (tiles + num_sms - 1) / num_sms;
        // Per tile: the K loop plus a fixed pipeline fill / drain.
        cost = waves * (kb * per_kb + 1500);
      } else {
        // one wave of clusters; each CTA runs its share of the K loop, then
        // the partials are summed through distributed shared memory
        cost = (kb + split - 1) / split * per_kb + 1500 + 300 + 4 * (int64_t)bn;
      }
      // Operand bytes streamed from L2 per tile, summed over tiles.
      const int64_t traffic = tiles * kb * (128 * 64 + (int64_t)bn * 64);
      if (best_cost < 0 || cost < best_cost || (cost == best_cost && traffic < best_traffic)) {
        best = GemmPlan{bn, 8, split};
        best_cost = cost;
        best_traffic = traffic;
      }
    }
    // CTA pair: 256-row tiles, each SM loading A and half of B per K-block.
    // Taken only with at least one full wave of pairs (measured: fewer pairs
    // than SM pairs lose to 128-row tiles, e.g. 2048^3 and 1024^3).
    if (bn >= 128) {
      const int64_t pair_tiles = (M + 255) / 256 * ((N + bn - 1) / bn);
      const int64_t pairs = num_sms / 2;
      if (pair_tiles >= pairs) {
        const int64_t per_kb_pair = 4 * mma_cycles(bn) > load_cycles_pair(bn)
                                        ? 4 * mma_cycles(bn)
                                        : load_cycles_pair(bn);
        const int64_t waves = (pair_tiles + pairs - 1) / pairs;
        const int64_t cost = waves * (kb * per_kb_pair + 1800);
        const int64_t traffic = pair_tiles * kb * (256 * 64 + (int64_t)bn * 64);
        if (cost < best_cost || (cost == best_cost && traffic < best_traffic)) {
          best = GemmPlan{bn, 8, 1, 2};
          best_cost = cost;
          best_traffic = traffic;
        }
      }
    }
  }
  const int64_t rows = (M + 128 * best.pair - 1) / (128 * best.pair);
  if (best.group_m > rows) best.group_m = (int)rows;
  return best;
}

}  // namespace hxb
