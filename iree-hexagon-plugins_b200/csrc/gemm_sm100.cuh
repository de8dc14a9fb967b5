// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M,N] = A[M,K] . B  (+ C_init)            f16 x f16 -> f32 accumulate
//
// This is the B200 form of the reference's HMX matmul lowering
// (plugins/compiler/hexagon/CodeGen/Transforms/HexagonConvertMatmulToHmx.cpp:
// 558-610 and HexagonExpandHmxMatmul.cpp:286-331): the VTCM double-buffered
// DMA pipeline (HexagonPipelineVTCMTransfers.cpp) becomes a STAGES-deep ring of
// shared-memory tiles fed by TMA and guarded by mbarriers, the 32x32 HMX
// K-loop becomes 128xBNx16 tcgen05.mma instructions into a TMEM accumulator,
// and hmx unpack (which adds into the destination, hmx.c:334-336) becomes the
// TMEM -> register epilogue with an optional C_init add.
//
// Roles (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer (one lane)
//   warp 1      TMEM owner + MMA issuer (one lane)
//   warps 2-5   epilogue: TMEM -> registers -> global (128 threads = 128 rows)
// The accumulator is double-buffered in TMEM so the epilogue of tile t
// overlaps the main loop of tile t+1.
#pragma once

#include "sm100.cuh"

namespace hxb {

// B operand forms.
enum BMode : int {
  kBF16RowMajorKN = 0,  // B[K,N] row-major f16 (MN-major operand)
  kBF16RowMajorNK = 1,  // B[N,K] row-major f16, i.e. transposed RHS (K-major)
};

enum OutMode : int { kOutF16 = 0, kOutF32 = 1 };

constexpr int kMaxDests = 8;  // all-gather epilogue: output replicas (one per rank)

struct GemmArgs {
  int M, N, K;
  void* C;             // output, row-major with leading dimension ldc
  long long ldc;
  const void* C_init;  // optional, same type/ld as C; added to the product
  const __half* scale; // per-output-column scale (int8-weight dispatch only)
  int* status;         // device status word (timeouts), may be null
  int tiles_m, tiles_n;
  int group_m;         // L2 raster: tiles walk GROUP_M rows of tiles at a time
  int vec_ok;          // 1 if C/C_init rows allow 16-byte vector access
  // All-gather epilogue (f16 output only): when ndests > 0 every output tile
  // is also written to dests[1..ndests) -- other ranks' copies of the output,
  // reached over NVLink through peer pointers -- at the same row and column.
  int ndests;
  void* dests[kMaxDests];
  // Stream-K (int8-weight GEMM only): when streamk != 0 every CTA owns a
  // contiguous share of the tiles x K-blocks iteration space; tiles split
  // between CTAs are summed through sk_partials (f32) under sk_flags.
  int streamk;
  int* sk_flags;
  float* sk_partials;
  int sk_dp_tiles;  // tiles before the stream-K part, dealt whole round-robin
};

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 f16 = one 128-byte swizzle row

template <int BN, int STAGES, int BMODE>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;        // 16 KB
  static constexpr int kBBytes = BN * kBK * 2;         // f16 tile for the MMA
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + STAGES * kABytes;
  static constexpr int kOffBar = kOffB + STAGES * kBBytes;
  // full[S], empty[S], tfull[2], tempty[2], drain[1]
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  // all-gather epilogue: per epilogue warp, one 32-row x 32-column f16 chunk
  static constexpr int kOffStage = (kOffMisc + 16 + 127) / 128 * 128;
  static constexpr int kBytes = kOffStage + 4 * 32 * 64;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-B alignment
  static_assert(kAlloc <= 232448, "shared memory per CTA");
  static_assert(kOffStage % 16 == 0, "16-byte staging pieces");
};

template <int BN, int BMODE>
struct GemmShape {
  static constexpr int kWarps = 6;
  static constexpr int kThreads = kWarps * 32;
  // accumulator buffers in TMEM: two (the epilogue of one tile overlaps the
  // next tile's main loop) unless a 512-column tile fills TMEM with one
  static constexpr int kAccBufs = 2 * BN <= 512 ? 2 : 1;
  static constexpr int kTmemCols = kAccBufs * BN < 32 ? 32 : kAccBufs * BN;
};

__device__ __forceinline__ void tile_coords(int t, const GemmArgs& a,
                                            int& tm, int& tn) {
  // Grouped raster: consecutive tiles sweep group_m tile-rows before moving
  // to the next tile-column, so concurrently resident CTAs share A and B
  // tiles in L2.
  const int per_group = a.group_m * a.tiles_n;
  const int g = t / per_group;
  const int first_m = g * a.group_m;
  const int gm = min(a.tiles_m - first_m, a.group_m);
  const int r = t - g * per_group;
  tm = first_m + r % gm;
  tn = r / gm;
}

// Epilogue for one 32-column chunk of one output row: optional C_init add,
// conversion and store. `r` holds the f32 accumulator bits read from TMEM.
template <int OUT>
__device__ __forceinline__ void store_chunk(const GemmArgs& args, int row,
                                            int col0, const uint32_t (&r)[32],
                                            uint4 (&packed)[4], bool replicas = true) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  const bool full_chunk = args.vec_ok && (col0 + 32 <= args.N);
  if constexpr (OUT == kOutF16) {
    __half* crow = reinterpret_cast<__half*>(args.C) + (long long)row * args.ldc;
    const __half* irow =
        args.C_init ? reinterpret_cast<const __half*>(args.C_init) +
                          (long long)row * args.ldc
                    : nullptr;
    if (full_chunk) {
      if (irow) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 i4 = *reinterpret_cast<const uint4*>(irow + col0 + u * 8);
          const __half2* h = reinterpret_cast<const __half2*>(&i4);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float2 f = __half22float2(h[e]);
            v[u * 8 + 2 * e] += f.x;
            v[u * 8 + 2 * e + 1] += f.y;
          }
        }
      }
      uint4 o[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        o[u].x = pack_half2(v[u * 8 + 0], v[u * 8 + 1]);
        o[u].y = pack_half2(v[u * 8 + 2], v[u * 8 + 3]);
        o[u].z = pack_half2(v[u * 8 + 4], v[u * 8 + 5]);
        o[u].w = pack_half2(v[u * 8 + 6], v[u * 8 + 7]);
        *reinterpret_cast<uint4*>(crow + col0 + u * 8) = o[u];
        packed[u] = o[u];
      }
      // replicas on the other ranks: the same 64 bytes at the same offset
      if (replicas)
      for (int d = 1; d < args.ndests; ++d) {
        __half* prow = reinterpret_cast<__half*>(args.dests[d]) + (long long)row * args.ldc;
#pragma unroll
        for (int u = 0; u < 4; ++u) *reinterpret_cast<uint4*>(prow + col0 + u * 8) = o[u];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (col0 + j < args.N) {
          float x = v[j];
          if (irow) x += __half2float(irow[col0 + j]);
          const __half hx = __float2half_rn(x);
          crow[col0 + j] = hx;
          for (int d = 1; d < args.ndests; ++d)
            reinterpret_cast<__half*>(args.dests[d])[(long long)row * args.ldc + col0 + j] = hx;
        }
      }
    }
  } else {
    float* crow = reinterpret_cast<float*>(args.C) + (long long)row * args.ldc;
    const float* irow =
        args.C_init ? reinterpret_cast<const float*>(args.C_init) +
                          (long long)row * args.ldc
                    : nullptr;
    if (full_chunk) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float4 o = make_float4(v[u * 4], v[u * 4 + 1], v[u * 4 + 2], v[u * 4 + 3]);
        if (irow) {
          float4 i4 = *reinterpret_cast<const float4*>(irow + col0 + u * 4);
          o.x += i4.x; o.y += i4.y; o.z += i4.z; o.w += i4.w;
        }
        *reinterpret_cast<float4*>(crow + col0 + u * 4) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (col0 + j < args.N) {
          float x = v[j];
          if (irow) x += irow[col0 + j];
          crow[col0 + j] = x;
        }
      }
    }
  }
}

// PAIR = 2 is the CTA-pair form (cta_group::2, a cluster of two CTAs on two
// SMs): the pair computes a 256 x BN tile with M = 256 MMAs issued by the
// leader (cluster rank 0). Each CTA loads its own 128 rows of A and its own
// BN / 2 columns of B into its own shared memory -- per SM that is 2/3 of the
// operand bytes of a 128 x BN tile for the same tensor work -- and holds
// rows [rank * 128, rank * 128 + 128) of the accumulator in its own TMEM.
// Both CTAs' loads complete on the leader's `full` barriers; the leader's
// commits arrive on both CTAs' `empty` and `tfull` barriers; both CTAs'
// epilogue warps arrive on the leader's `tempty`. No multicast anywhere.
template <int BN, int STAGES, int BMODE, int OUT, int PAIR = 1>
__global__ void __launch_bounds__(GemmShape<BN, BMODE>::kThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const GemmArgs args) {
  static_assert(PAIR == 1 || PAIR == 2, "one CTA or a CTA pair per tile");
  static_assert(BN <= 256 || PAIR == 2, "512-column tiles only on CTA pairs");
  constexpr int kBNC = BN / PAIR;     // B columns this CTA loads
  constexpr int kTileM = kBM * PAIR;  // output rows of a tile
  // N of one MMA (at most 256): a 512-column pair tile is two MMA chunks
  // sharing each A stage; chunk j covers tile columns [256 j, 256 j + 256),
  // of which this CTA loads kChunkCols at rank * kChunkCols.
  constexpr int kMmaN = BN > 256 ? 256 : BN;
  constexpr int kChunks = BN / kMmaN;
  constexpr int kChunkCols = kMmaN / PAIR;
  constexpr int kChunkBytes = kChunkCols * kBK * 2;
  constexpr int kAccBufs = GemmShape<BN, BMODE>::kAccBufs;
  using L = GemmSmem<kBNC, STAGES, BMODE>;
  constexpr int kTmemCols = GemmShape<BN, BMODE>::kTmemCols;
  constexpr uint32_t kIdesc =
      make_idesc_f16(kTileM, kMmaN, 0, BMODE == kBF16RowMajorNK ? 0 : 1);
  // the (leader's) full barrier counts the bytes of every CTA of the tile
  constexpr uint32_t kTxBytes = (L::kABytes + L::kBBytes) * PAIR;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR > 1 ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit = (int)blockIdx.x / PAIR;  // this CTA's tile walker
  const int units = (int)gridDim.x / PAIR;
  const int num_tiles = args.tiles_m * args.tiles_n;
  const int num_kb = (args.K + kBK - 1) / kBK;
  const FailState fs{abort_flag, args.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4 * PAIR);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR == 1) {
      tmem_alloc(tmem_holder, kTmemCols);
      tmem_relinquish();
    } else {
      tmem_alloc_pair(tmem_holder, kTmemCols);
      tmem_relinquish_pair();
    }
  }
  tc_fence_before();
  // the peer's barriers must be initialised before any load, commit or
  // arrival of the pair reaches them
  __syncwarp();
  if constexpr (PAIR == 1) __syncthreads(); else cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // The set-up above overlaps the previous kernel of the stream (programmatic
  // dependent launch). Every global access below follows the producer's
  // pdl_wait(): operand loads directly, the epilogue through the mbarrier
  // chain of the tiles it drains.
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      // The operands of this CTA's first tile's first K-blocks are requested
      // into L2 while the previous kernel of the stream may still run; the
      // loads below, issued after the wait, then hit L2.
      if (unit < num_tiles) {
        int tm0, tn0;
        tile_coords(unit, args, tm0, tn0);
        const int a_row0 = tm0 * kTileM + (int)rank * kBM;
        const int pre = num_kb < STAGES ? num_kb : STAGES;
        for (int kb = 0; kb < pre; ++kb) {
          tma_prefetch_l2_2d(&tmA, kb * kBK, a_row0);
#pragma unroll
          for (int c = 0; c < kChunks; ++c) {
            const int b_col0 = tn0 * BN + c * kMmaN + (int)rank * kChunkCols;
            if constexpr (BMODE == kBF16RowMajorKN) {
#pragma unroll
              for (int j = 0; j < kChunkCols / 64; ++j)
                tma_prefetch_l2_2d(&tmB, b_col0 + 64 * j, kb * kBK);
            } else {
              tma_prefetch_l2_2d(&tmB, kb * kBK, b_col0);
            }
          }
        }
      }
      pdl_wait();
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = unit; t < num_tiles && ok; t += units) {
        int tm, tn;
        tile_coords(t, args, tm, tn);
        const int a_row = tm * kTileM + (int)rank * kBM;
        const int b_col = tn * BN + (int)rank * kChunkCols;  // chunk c adds c * kMmaN
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, fs)) { ok = false; break; }
          uint8_t* a_dst = smem + L::kOffA + stage * L::kABytes;
          uint8_t* b_dst = smem + L::kOffB + stage * L::kBBytes;
          if constexpr (PAIR == 1) {
            mbar_arrive_expect_tx(&full[stage], kTxBytes);
            tma_load_2d(a_dst, &tmA, &full[stage], kb * kBK, a_row);
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
              if constexpr (BMODE == kBF16RowMajorKN) {
#pragma unroll
                for (int j = 0; j < kChunkCols / 64; ++j)
                  tma_load_2d(b_dst + c * kChunkBytes + j * (kBK * 128), &tmB, &full[stage],
                              b_col + c * kMmaN + 64 * j, kb * kBK);
              } else {
                tma_load_2d(b_dst + c * kChunkBytes, &tmB, &full[stage], kb * kBK,
                            b_col + c * kMmaN);
              }
            }
          } else {
            // both CTAs' bytes complete on the leader's barrier; only the
            // leader arms it (a peer's bytes may land first: the phase cannot
            // complete before the leader's arrival)
            if (leader) mbar_arrive_expect_tx(&full[stage], kTxBytes);
            const uint32_t bar = map_to_rank(smem_u32(&full[stage]), 0);
            tma_load_2d_pair(a_dst, &tmA, bar, kb * kBK, a_row);
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
              if constexpr (BMODE == kBF16RowMajorKN) {
#pragma unroll
                for (int j = 0; j < kChunkCols / 64; ++j)
                  tma_load_2d_pair(b_dst + c * kChunkBytes + j * (kBK * 128), &tmB, bar,
                                   b_col + c * kMmaN + 64 * j, kb * kBK);
              } else {
                tma_load_2d_pair(b_dst + c * kChunkBytes, &tmB, bar, kb * kBK,
                                 b_col + c * kMmaN);
              }
            }
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Never leave the CTA with bulk copies still landing in its shared
      // memory: wait for the last STAGES issues (already complete on the
      // normal path). A pair's second CTA sees its copies complete through
      // its `empty` barriers (the MMAs that read them have retired).
      const long long nd = issued < STAGES ? issued : STAGES;
      for (long long i = 0; i < nd; ++i) {
        const long long u = issued - 1 - i;
        const int s = (int)(u % STAGES);
        const uint32_t ph = (uint32_t)((u / STAGES) & 1);
        uint64_t* bar = leader ? &full[s] : &empty[s];
        // bounded even on the failure path
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(bar, ph) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int tl = 0;
      bool ok = true;
      bool issued_any = false;
      // The tensor core takes an MMA about as fast as it runs one, so the
      // issue loop is kept to adds: the operand descriptors are built once and
      // a stage, a K step or an N chunk moves only their start-address field
      // (address >> 4 in 14 bits; shared memory stays below 256 KB).
      const uint64_t a_desc0 =
          make_smem_desc(smem_u32(smem + L::kOffA), 16, 1024, kLayoutSwizzle128);
      const uint64_t b_desc0 =
          BMODE == kBF16RowMajorNK
              ? make_smem_desc(smem_u32(smem + L::kOffB), 16, 1024, kLayoutSwizzle128)
              : make_smem_desc(smem_u32(smem + L::kOffB), kBK * 128, 1024, kLayoutSwizzle128);
      for (int t = unit; t < num_tiles && ok; t += units, ++tl) {
        const int acc = tl % kAccBufs;
        const uint32_t acc_phase = (tl / kAccBufs) & 1;
        // (a pair's tempty collects the peer's epilogue arrivals too)
        const bool free_acc = PAIR == 1 ? mbar_wait(&tempty[acc], acc_phase ^ 1, fs)
                                        : mbar_wait_cluster(&tempty[acc], acc_phase ^ 1, fs);
        if (!free_acc) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, fs)) { ok = false; break; }
          tc_fence_after();
          const uint64_t a_desc = a_desc0 + (uint64_t)(stage * (L::kABytes >> 4));
          const uint64_t b_desc = b_desc0 + (uint64_t)(stage * (L::kBBytes >> 4));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = a_desc + (uint64_t)(k * 32 >> 4);
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
              const int boff = c * kChunkBytes + (BMODE == kBF16RowMajorNK ? k * 32 : k * 16 * 128);
              const uint64_t bdesc = b_desc + (uint64_t)(boff >> 4);
              if constexpr (PAIR == 1)
                umma_f16_ss(d_tmem + c * kMmaN, adesc, bdesc, kIdesc, (kb | k) != 0);
              else
                umma_f16_ss_pair(d_tmem + c * kMmaN, adesc, bdesc, kIdesc, (kb | k) != 0);
            }
          }
          issued_any = true;
          if constexpr (PAIR == 1) {
            umma_commit(&empty[stage]);
          } else {
            umma_commit_pair(smem_u32(&empty[stage]));
            umma_commit_pair(map_to_rank(smem_u32(&empty[stage]), 1));
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) {
          if constexpr (PAIR == 1) {
            umma_commit(&tfull[acc]);
          } else {
            umma_commit_pair(smem_u32(&tfull[acc]));
            umma_commit_pair(map_to_rank(smem_u32(&tfull[acc]), 1));
          }
        }
      }
      if (!ok && issued_any) {
        // Failure path: let every MMA already issued retire before TMEM is
        // released.
        if constexpr (PAIR == 1) umma_commit(drain); else umma_commit_pair(smem_u32(drain));
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    // ------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int tl = 0;
    for (int t = unit; t < num_tiles; t += units, ++tl) {
      int tm, tn;
      tile_coords(t, args, tm, tn);
      const int acc = tl % kAccBufs;
      const uint32_t acc_phase = (tl / kAccBufs) & 1;
      const bool ready = mbar_wait(&tfull[acc], acc_phase, fs);
      // tcgen05.ld is .sync.aligned: reconverge and agree before touching TMEM
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const int row = tm * kTileM + (int)rank * kBM + q * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      // all-gather replicas of full f16 chunks go through this warp's staging
      // chunk: lanes write their rows' 64 bytes, then four lanes per row store
      // each row to every replica as one contiguous 64-byte run (row-per-lane
      // stores would scatter every warp store over 32 rows of a peer's matrix)
      uint4* stage = reinterpret_cast<uint4*>(smem + L::kOffStage) + q * 32 * 4;
      const int row0 = row - lane;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c, r);
        tmem_wait_ld();
        const int col0 = tn * BN + c;
        // the same for every lane of the warp
        const bool staged = OUT == kOutF16 && args.ndests > 1 && args.vec_ok &&
                            col0 + 32 <= args.N;
        uint4 packed[4];
        if (row < args.M && col0 < args.N) store_chunk<OUT>(args, row, col0, r, packed, !staged);
        if (staged) {
          // piece u of row `lane` sits at slot u ^ ((lane >> 1) & 3): both the
          // row-wise writes and the piece-wise reads hit distinct bank groups
#pragma unroll
          for (int u = 0; u < 4; ++u) stage[lane * 4 + (u ^ ((lane >> 1) & 3))] = packed[u];
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int p = lane + 32 * k, rr = p >> 2, u = p & 3;
            const int grow = row0 + rr;
            if (grow < args.M) {
              const uint4 v = stage[rr * 4 + (u ^ ((rr >> 1) & 3))];
              const long long off = (long long)grow * args.ldc + col0 + u * 8;
              for (int d = 1; d < args.ndests; ++d)
                *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(args.dests[d]) + off) = v;
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&tempty[acc]);
        else mbar_arrive_cluster(map_to_rank(smem_u32(&tempty[acc]), 0));
      }
    }
    // all-gather epilogue: this thread's stores into the other ranks' outputs
    // are performed system-wide before the kernel ends, so a barrier that
    // follows the kernel on the stream (hxb_peer_barrier) publishes them
    if (args.ndests > 1) __threadfence_system();
  }

  tc_fence_before();
  // a pair's CTAs stay resident until neither can still reach the other's
  // shared memory (remote arrivals, commits) or TMEM
  __syncwarp();
  if constexpr (PAIR == 1) __syncthreads(); else cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR == 1) tmem_dealloc(tmem_base, kTmemCols);
    else tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace hxb
