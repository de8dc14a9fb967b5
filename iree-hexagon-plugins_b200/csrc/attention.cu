// Fused attention dispatch for sm_100a:
//   O[bh, i, :] = softmax_j(scale * Q[bh, i, :] . K[bh, j, :] [causal mask]) . V[bh, j, :]
// f16 Q/K/V/O, f32 scores, f32 softmax statistics, f32 accumulation.
//
// This replaces the reference's decomposed attention layer
// (examples/attention_layer/attention_layer.mlir:17-111: an f32 batch_matmul
// for the scores, max / sub / exp / sum / div reductions and a second
// batch_matmul, each a separate dispatch with the full S x S score matrix in
// memory) by one kernel in which the scores never leave the SM:
//
//   * one CTA owns 2 query tiles of 128 rows (256 query rows of one head) and
//     walks the keys in blocks of 128; K and V tiles stream through a 4-slot
//     TMA ring (one K or one V tile of 32 KB per slot);
//   * S_t = Q_t K^T (tcgen05.mma, Q and K from shared memory) lands in TMEM;
//   * softmax warpgroup t (128 threads, thread r = query row r of tile t)
//     reads its S row from TMEM, applies the online-softmax update in the
//     log2 domain and writes P = exp2(S*c - m) as f16 back into the upper half
//     of the S columns;
//   * O_t += P_t V (tcgen05.mma with A = P read from TMEM, B = V from shared
//     memory) accumulates in TMEM; the two tiles ping-pong so that the tensor
//     core works on one tile while the other tile's softmax runs;
//   * the running maximum is only moved (and O rescaled in TMEM) when it grows
//     by more than 2^8; in between, P is formed against the stale maximum,
//     which stays exact because the final division by the row sum uses the
//     same maximum (P <= 2^8 fits f16 easily);
//   * rows whose keys are all masked produce 0, as attention_layer.mlir:86-103
//     selects.
//
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512);
// P_t aliases columns [64,128) of S_t. The next S_t is issued after PV_t by the
// same thread, so the tensor core has consumed P_t before S_t is rewritten.
//
// Roles (384 threads, one CTA per SM):
//   warp 0        TMA producer (one lane): Q once, then K0 V0 K1 V1 ...
//   warp 1        TMEM owner + MMA issuer (one lane)
//   warps 2-3     idle
//   warps 4-7     softmax + epilogue of query tile 0
//   warps 8-11    softmax + epilogue of query tile 1
#include <math.h>

#include <algorithm>

#include "runtime_common.h"
#include "sm100.cuh"

namespace hxb {
namespace {

constexpr int kAttBM = 128;      // query rows per tile
constexpr int kAttTiles = 2;     // query tiles per CTA
constexpr int kAttBN = 128;      // keys per block
constexpr int kAttBoxBytes = 128 * 64 * 2;      // one TMA box: 128 rows x 64 f16
constexpr float kRescaleLog2 = 8.0f;
constexpr int kAttThreads = 384;
// Registers per thread: the launch gives every warp kAttRegsLaunch (the
// __launch_bounds__ limit for 384 threads on one SM); then the TMA / MMA
// warpgroup drops to kAttRegsControl and the two softmax warpgroups, which
// hold a 128-score row per thread, rise to kAttRegsSoftmax.
constexpr int kAttRegsLaunch = 168;
constexpr int kAttRegsControl = 104;
constexpr int kAttRegsSoftmax = 200;
static_assert(kAttRegsControl * 128 + kAttRegsSoftmax * (kAttThreads - 128) <=
                  kAttRegsLaunch * kAttThreads,
              "register split exceeds the launch allocation");

// Shared-memory plan for head dimension D (64 or 128): a Q, K or V tile is
// D/64 boxes of [128 rows x 64] f16; the K/V ring keeps 128 KB of tiles
// (4 slots at D = 128, 8 at D = 64).
template <int D>
struct AttSmem {
  static_assert(D == 64 || D == 128, "head dimension 64 or 128");
  static constexpr int kBoxes = D / 64;
  static constexpr int kTileBytes = 128 * D * 2;
  static constexpr int kSlots = D == 64 ? 8 : 4;
  static constexpr int kOffQ = 0;
  static constexpr int kOffKV = kOffQ + kAttTiles * kTileBytes;
  static constexpr int kOffBar = kOffKV + kSlots * kTileBytes;
  // q_full, kv_full[slots], kv_empty[slots], s_full[2], p_full[2], o_full, drain
  static constexpr int kNumBars = 1 + 2 * kSlots + 2 * kAttTiles + 2;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

// Q, K, V are row-major matrices; a CTA head bh (one KV head) reads
//   Q rows [(bh / q_hpr) * Sq, +Sq)              columns [(bh % q_hpr) * D, +D)
//   K, V rows [(bh / kv_hpr) * kv_stride, +Skv)  columns [(bh % kv_hpr) * D, +D)
// with q_hpr / kv_hpr heads per matrix row: 1 is the contiguous [B*H, S, D]
// layout, H the [B, S, H*D] layout (e.g. the Q/K/V column blocks of a fused
// QKV projection output). kv_stride >= Skv lets K/V be the first Skv rows of
// a longer cache. Grouped-query attention packs the `group` query heads that
// share KV head bh into one CTA head of Sq = group * q_len rows
// (q_hpr = 1): packed row r is position r % q_len of query head
// bh * group + r / q_len. Output query head g (global index over batch x query
// heads) position s goes to O row (g / o_hpr) * q_len + s, columns
// [(g % o_hpr) * D, +D). Rows of a tile past Sq (or keys past Skv) belong to
// the next head or batch, or lie outside the matrix and read as zeros: their
// keys are masked and their query rows are not stored.
struct AttArgs {
  int Sq, Skv;
  int q_hpr, kv_hpr;  // Q and K/V heads per row
  int q_len;          // query positions per query head (Sq / group)
  int group;          // query heads per CTA head
  int o_hpr;          // O heads per row
  long long kv_stride;  // K/V rows per head
  long long ldo;      // O row pitch (elements)
  int q_rows;         // rows per query block: 256 (two tiles) or 128 (one)
  int q_blocks;       // query blocks per head: ceil(Sq / q_rows)
  int q_box;          // Q rows one TMA box brings (min(128, Sq rounded up to 8))
  int kv_splits;      // CTAs sharing one query block's keys (1: no split)
  int split_blocks;   // key blocks per split
  float* part_o;      // kv_splits > 1: normalised partial O, f32 [CTA][part_rows][D]
  float* part_lse;    // and its log2-sum-exp2, [CTA][part_rows]
  int part_rows;      // rows kept per CTA: min(256, Sq)
  int causal;
  int causal_offset;  // key j is visible to query position i iff j <= i + offset
  float c;            // scale * log2(e)
  const __half* Q;    // for the decode kernel, which copies Q without TMA
  long long ldq;
  __half* O;
  int* status;
};

// Number of key blocks CTA rows [q0, q0 + q_rows) may see.
__device__ __forceinline__ int kv_blocks_for(const AttArgs& a, int q0) {
  int last_key = a.Skv - 1;
  if (a.causal) {
    const int last_row = min(q0 + a.q_rows, a.Sq) - 1;
    // the largest query position among the rows: a CTA spanning two query
    // heads holds the last position of the first one
    const int last_pos = last_row / a.q_len != q0 / a.q_len ? a.q_len - 1 : last_row % a.q_len;
    last_key = min(last_key, last_pos + a.causal_offset);
  }
  return last_key < 0 ? 0 : last_key / kAttBN + 1;
}

// K-major 128B-swizzled operand made of two [128 rows x 64] boxes: the
// descriptor of its 16-element K step kk.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return make_smem_desc(base + (kk >> 2) * kAttBoxBytes + (kk & 3) * 32, 16, 1024,
                        kLayoutSwizzle128);
}

// MN-major (V: keys along K, head dim along N) operand made of two
// [128 keys x 64 d] boxes: the descriptor of its 16-key K step kk.
__device__ __forceinline__ uint64_t vmajor_desc(uint32_t base, int kk) {
  return make_smem_desc(base + kk * 16 * 128, kAttBoxBytes, 1024, kLayoutSwizzle128);
}

template <int S>
struct Cursor {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void advance() {
    if (++slot == S) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

template <int D>
__global__ void __launch_bounds__(kAttThreads, 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const AttArgs args) {
  using L = AttSmem<D>;
  constexpr int kAttSlots = L::kSlots;
  constexpr int kAttTileBytes = L::kTileBytes;
  constexpr uint32_t kIdescQK = make_idesc_f16(kAttBM, kAttBN, 0, 0);
  constexpr uint32_t kIdescPV = make_idesc_f16(kAttBM, D, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + kAttSlots;
  uint64_t* s_full = kv_empty + kAttSlots;
  uint64_t* p_full = s_full + kAttTiles;
  uint64_t* o_full = p_full + kAttTiles;
  uint64_t* drain = o_full + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x % args.kv_splits;
  const int qb = blockIdx.x / args.kv_splits % args.q_blocks;
  const int bh = blockIdx.x / args.kv_splits / args.q_blocks;
  const int qx = (bh % args.q_hpr) * D;   // Q column of this head
  const int qy = bh / args.q_hpr;         // Q row block of this head
  const int kx = (bh % args.kv_hpr) * D;  // K/V column
  const int ky = bh / args.kv_hpr;        // K/V row block
  const int q0 = qb * args.q_rows;
  // this CTA's key blocks: [j0, j0 + n_kv) of the query block's visible ones
  const int visible = kv_blocks_for(args, q0);
  const int j0 = split * args.split_blocks;
  const int n_kv = args.kv_splits == 1 ? visible : max(0, min(visible - j0, args.split_blocks));
  // a second query tile only when the rows reach into it
  const int n_tiles = args.q_rows > kAttBM && args.Sq - q0 > kAttBM ? kAttTiles : 1;
  const FailState fs{abort_flag, args.status};

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kAttSlots; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < kAttTiles; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], kAttBM);
    }
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // the set-up above overlaps the previous kernel of the stream; Q/K/V and O
  // are touched only after it has finished
  pdl_trigger();
  pdl_wait();

  // (each warpgroup changes its register count inside its own branch, so that
  // the compiler allocates each branch for the count it runs with)
  if (warp < 4) {
    reg_dealloc<kAttRegsControl>();  // warps 2-3 stay idle
    if (warp == 0) {
      // -------------------------------------------------------- TMA producer
      if (lane == 0 && n_kv > 0) {
        // a short Q (decode: a group's few rows) loads only q_box rows; the
        // rest of the tile keeps stale bytes, which reach only rows not stored
        mbar_arrive_expect_tx(q_full, n_tiles * L::kBoxes * args.q_box * 128);
        for (int t = 0; t < n_tiles; ++t)
          for (int b = 0; b < L::kBoxes; ++b)
            tma_load_2d(smem + L::kOffQ + t * kAttTileBytes + b * kAttBoxBytes, &tmQ, q_full,
                        qx + 64 * b, qy * args.Sq + q0 + t * kAttBM);
        Cursor<kAttSlots> c;
        int issued = 0;
        bool ok = true;
        for (int j = 0; j < n_kv && ok; ++j) {
          for (int which = 0; which < 2; ++which) {  // K_j then V_j
            if (!mbar_wait(&kv_empty[c.slot], c.phase ^ 1, fs)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&kv_full[c.slot], kAttTileBytes);
            const CUtensorMap* map = which ? &tmV : &tmK;
            for (int b = 0; b < L::kBoxes; ++b)
              tma_load_2d(smem + L::kOffKV + c.slot * kAttTileBytes + b * kAttBoxBytes, map,
                          &kv_full[c.slot], kx + 64 * b,
                          (int)(ky * args.kv_stride) + (j0 + j) * kAttBN);
            c.advance();
            ++issued;
          }
        }
        // bounded wait for the copies still landing (complete on the normal path)
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
        for (int i = 0; i < issued && i < kAttSlots; ++i) {
          if (c.slot == 0) {
            c.slot = kAttSlots - 1;
            c.phase ^= 1u;
          } else {
            --c.slot;
          }
          const unsigned long long t1 = globaltimer_ns();
          while (!mbar_try_wait(&kv_full[c.slot], c.phase) &&
                 globaltimer_ns() - t1 < kWaitLimitNs) {
          }
        }
      }
    } else if (warp == 1) {
      // -------------------------------------------------------- MMA issuer
      if (lane == 0 && n_kv > 0) {
        bool ok = mbar_wait(q_full, 0, fs);
        bool issued_any = false;
        Cursor<kAttSlots> c;
        // The tensor core accepts an MMA only about as fast as it executes one
        // (64 cycles at N = 128), so the issue loop is kept to adds: the
        // operand descriptors are built once, and a query tile, a ring slot or
        // a K step only moves their start-address field (address >> 4 in 14
        // bits; shared-memory addresses stay below 256 KB, so it never carries).
        const uint64_t q_desc = kmajor_desc(smem_u32(smem + L::kOffQ), 0);
        const uint64_t k_desc = kmajor_desc(smem_u32(smem + L::kOffKV), 0);
        const uint64_t v_desc = vmajor_desc(smem_u32(smem + L::kOffKV), 0);
        constexpr uint64_t kTileStep = kAttTileBytes >> 4;
        // S_t(0) = Q_t K_0^T
        int kslot = c.slot;
        if (ok) ok = mbar_wait(&kv_full[kslot], c.phase, fs);
        c.advance();
        if (ok) {
          tc_fence_after();
          const uint64_t kd = k_desc + kslot * kTileStep;
#pragma unroll
          for (int t = 0; t < kAttTiles; ++t) {
            if (t >= n_tiles) break;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint64_t off = (uint64_t)(((kk >> 2) * kAttBoxBytes + (kk & 3) * 32) >> 4);
              umma_f16_ss(tmem_base + t * 128, q_desc + t * kTileStep + off, kd + off, kIdescQK,
                          kk != 0);
            }
            umma_commit(&s_full[t]);
          }
          umma_commit(&kv_empty[kslot]);
          issued_any = true;
        }
        for (int j = 0; j < n_kv && ok; ++j) {
          const int vslot = c.slot;
          if (!mbar_wait(&kv_full[vslot], c.phase, fs)) { ok = false; break; }
          c.advance();
          const bool has_next = j + 1 < n_kv;
          if (has_next) {
            kslot = c.slot;
            if (!mbar_wait(&kv_full[kslot], c.phase, fs)) { ok = false; break; }
            c.advance();
          }
          const uint64_t vd = v_desc + vslot * kTileStep, kd = k_desc + kslot * kTileStep;
#pragma unroll
          for (int t = 0; t < kAttTiles; ++t) {
            if (t >= n_tiles) break;
            if (!mbar_wait(&p_full[t], (uint32_t)(j & 1), fs)) { ok = false; break; }
            tc_fence_after();
            const uint32_t o_tmem = tmem_base + 256 + t * D;
            const uint32_t p_tmem = tmem_base + t * 128 + 64;
#pragma unroll
            for (int kk = 0; kk < kAttBN / 16; ++kk)
              umma_f16_ts(o_tmem, p_tmem + kk * 8, vd + (uint64_t)(kk * 16 * 128 >> 4), kIdescPV,
                          (j | kk) != 0);
            if (has_next) {
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk) {
                const uint64_t off = (uint64_t)(((kk >> 2) * kAttBoxBytes + (kk & 3) * 32) >> 4);
                umma_f16_ss(tmem_base + t * 128, q_desc + t * kTileStep + off, kd + off, kIdescQK,
                            kk != 0);
              }
              umma_commit(&s_full[t]);
            }
          }
          if (!ok) break;
          umma_commit(&kv_empty[vslot]);
          if (has_next) umma_commit(&kv_empty[kslot]);
        }
        if (ok) {
          umma_commit(o_full);
        } else if (issued_any) {
          umma_commit(drain);
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else {
    // -------------------------------------------------------- softmax
    reg_alloc<kAttRegsSoftmax>();
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qrow = q0 + t * kAttBM + r;  // packed row of the CTA head
    const int qpos = qrow % args.q_len;     // its query position
    const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const uint32_t s_col = t * 128, p_col = t * 128 + 64, o_col = 256 + t * D;
    const float c = args.c;
    float m_run = -INFINITY;  // running max of S*c (log2 domain)
    float l_run = 0.0f;       // running sum of P against m_run
    bool ok = true;
    const int my_kv = t < n_tiles ? n_kv : 0;
    for (int j = 0; j < my_kv; ++j) {
      const bool ready = mbar_wait(&s_full[t], (uint32_t)(j & 1), fs);
      if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
      tc_fence_after();
      float s[kAttBN];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(lane_base + s_col + ch * 32, u);
#pragma unroll
        for (int e = 0; e < 32; ++e) s[ch * 32 + e] = __uint_as_float(u[e]);
      }
      tmem_wait_ld();
      const int key0 = (j0 + j) * kAttBN;
      if (key0 + kAttBN > args.Skv || args.causal) {
        const int lim = args.causal ? min(args.Skv - 1, qpos + args.causal_offset) : args.Skv - 1;
#pragma unroll
        for (int e = 0; e < kAttBN; ++e)
          if (key0 + e > lim) s[e] = -INFINITY;
      }
      // row maximum: eight independent chains of three-input max, then a tree
      float m8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float* v = s + 16 * i;
        float m = fmax3(v[0], v[1], v[2]);
#pragma unroll
        for (int k = 3; k < 15; k += 2) m = fmax3(m, v[k], v[k + 1]);
        m8[i] = fmaxf(m, v[15]);
      }
      const float mx =
          fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
      const float m_blk = mx * c;  // -inf stays -inf (c > 0)
      const float m_new = fmaxf(m_run, m_blk);
      bool need = false;
      if (j == 0 || l_run == 0.0f) {
        // nothing accumulated yet (O is rewritten by the first PV or holds 0)
        m_run = m_new;
      } else {
        need = m_new - m_run > kRescaleLog2;
      }
      if (__any_sync(0xffffffffu, need)) {
        // O_t(j-1) is complete: S_t(j) was issued after PV_t(j-1).
        const float alpha = need ? ex2_approx(m_run - m_new) : 1.0f;
        if (need) {
          l_run *= alpha;
          m_run = m_new;
        }
#pragma unroll 1
        for (int ch = 0; ch < D / 32; ++ch) {
          uint32_t u[32];
          tmem_ld_32x32b_x32(lane_base + o_col + ch * 32, u);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
          tmem_st_32x32b_x32(lane_base + o_col + ch * 32, u);
        }
      }
      const float m_use = m_run == -INFINITY ? 0.0f : m_run;
      // P = 2^(S c - m) with the arguments and the row sum on packed f32
      // pairs (one f32x2 instruction per two keys). Measured on cfg 3: 281.7
      // -> 275.6 us; evaluating one pair in four on the FMA pipe instead of
      // the special-function unit (Cody-Waite + degree-3 polynomial) on top
      // of it measured 293.9 us, and the three-input max tree alone 283.7 us.
      const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(-m_use, -m_use);
      uint64_t acc2[2] = {0ull, 0ull};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const uint64_t x2 = f2_fma(f2_pack(s[h * 64 + 2 * e], s[h * 64 + 2 * e + 1]), c2, nm2);
          float a, b;
          f2_unpack(x2, a, b);
          const float p0 = ex2_approx(a), p1 = ex2_approx(b);
          acc2[e & 1] = f2_add(acc2[e & 1], f2_pack(p0, p1));
          pk[e] = pack_half2(p0, p1);
        }
        tmem_st_32x32b_x32(lane_base + p_col + h * 32, pk);
      }
      float sa, sb, sc2, sd;
      f2_unpack(acc2[0], sa, sb);
      f2_unpack(acc2[1], sc2, sd);
      l_run += (sa + sb) + (sc2 + sd);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    // -------------------------------------------------------- epilogue
    bool have = ok && n_kv > 0;
    if (have) have = mbar_wait(o_full, 0, fs);
    const bool all_have = __all_sync(0xffffffffu, have);
    if (all_have) tc_fence_after();
    const float inv = (all_have && l_run > 0.0f) ? 1.0f / l_run : 0.0f;
    const long long qhead = (long long)bh * args.group + qrow / args.q_len;
    __half* orow = args.O + (qhead / args.o_hpr * args.q_len + qpos) * args.ldo +
                   qhead % args.o_hpr * D;
    // (a tile the block does not run leaves its rows to the next block)
    const bool write = t < n_tiles && (ok || n_kv == 0) && qrow < args.Sq;
    const bool partial = args.kv_splits > 1;
    // split keys: this CTA's normalised O and log2-sum-exp2 of its row
    const size_t pidx = (size_t)blockIdx.x * args.part_rows + (t * kAttBM + r);
    if (partial && write)
      args.part_lse[pidx] = (all_have && l_run > 0.0f) ? m_run + log2f(l_run) : -INFINITY;
#pragma unroll 1
    for (int ch = 0; ch < D / 32; ++ch) {
      uint32_t u[32];
      if (all_have) {
        tmem_ld_32x32b_x32(lane_base + o_col + ch * 32, u);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) u[e] = 0u;
      }
      if (partial) {
        if (write) {
          float4* po = reinterpret_cast<float4*>(args.part_o + pidx * D + ch * 32);
#pragma unroll
          for (int v = 0; v < 8; ++v)
            po[v] = make_float4(__uint_as_float(u[v * 4 + 0]) * inv,
                                __uint_as_float(u[v * 4 + 1]) * inv,
                                __uint_as_float(u[v * 4 + 2]) * inv,
                                __uint_as_float(u[v * 4 + 3]) * inv);
        }
      } else if (write) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 o;
          o.x = pack_half2(__uint_as_float(u[v * 8 + 0]) * inv, __uint_as_float(u[v * 8 + 1]) * inv);
          o.y = pack_half2(__uint_as_float(u[v * 8 + 2]) * inv, __uint_as_float(u[v * 8 + 3]) * inv);
          o.z = pack_half2(__uint_as_float(u[v * 8 + 4]) * inv, __uint_as_float(u[v * 8 + 5]) * inv);
          o.w = pack_half2(__uint_as_float(u[v * 8 + 6]) * inv, __uint_as_float(u[v * 8 + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + ch * 32 + v * 8) = o;
        }
      }
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ---------------------------------------------------------------- decode
// Attention of at most 16 query rows per CTA head (decode: the query heads
// of one KV head times a few positions) with head dimension 128. The
// 128-row tile of attention_fwd_kernel would be nearly all padding there,
// and each of its threads would evaluate 128 exponentials per key block for
// one live row. Here the keys sit on the TMEM lanes instead:
//   S^T[key, q] = K Q^T   (tcgen05, M = 128 keys, N = 16 rows, K = D)
//   thread = key: its 16 scores, 16 exp2 per block, P^T to shared memory
//   O^T[d, q] += V^T P^T   (M = 128 = D from the MN-major V tile, N = 16)
// The running maximum of every row is shared by the 128 key threads; it is
// only recomputed (a warp-shuffle and shared-memory reduction) when some
// score exceeds it by more than 2^8, as in attention_fwd_kernel. Row sums
// stay per thread until the end. Partial results of split keys use the same
// layout as attention_fwd_kernel, so attention_combine_kernel merges them.
constexpr int kDecRows = 16;     // query rows per CTA head (MMA N)
constexpr int kDecSlots = 3;     // K/V ring slots (two CTAs per SM)
constexpr int kDecThreads = 256; // warp 0 TMA, warp 1 MMA + TMEM, warps 4-7 keys
constexpr int kDecTmemCols = 32; // S^T in [0, 16), O^T in [16, 32)

struct DecSmem {
  static constexpr int kTileBytes = 128 * 128 * 2;  // one K or V tile, two boxes
  static constexpr int kRowsBox = kDecRows * 128;   // one [16 rows x 64] f16 box
  static constexpr int kOffKV = 0;
  static constexpr int kOffQ = kOffKV + kDecSlots * kTileBytes;
  static constexpr int kOffP = kOffQ + 2 * kRowsBox;   // P^T as [16 rows][128 keys]
  static constexpr int kOffRed = kOffP + 2 * kRowsBox; // [4 warps][16] floats + votes
  static constexpr int kOffBar = kOffRed + 512;
  // q_full, kv_full[slots], kv_empty[slots], s_full, p_full, o_full, drain,
  // ksync (the key threads' bounded barrier)
  static constexpr int kNumBars = 1 + 2 * kDecSlots + 5;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

// K-major 128B-swizzled [16 rows x 128] operand (two [16 x 64] boxes): the
// descriptor of its 16-element K step kk.
__device__ __forceinline__ uint64_t rows16_desc(uint32_t base, int kk) {
  return make_smem_desc(base + (kk >> 2) * DecSmem::kRowsBox + (kk & 3) * 32, 16, 1024,
                        kLayoutSwizzle128);
}

__global__ void __launch_bounds__(kDecThreads, 2)
    attention_decode_kernel(const __grid_constant__ CUtensorMap tmQ,
                            const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const AttArgs args) {
  using L = DecSmem;
  constexpr int D = 128;
  constexpr uint32_t kIdescS = make_idesc_f16(128, kDecRows, 0, 0);
  constexpr uint32_t kIdescO = make_idesc_f16(128, kDecRows, 1, 0);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + kDecSlots;
  uint64_t* s_full = kv_empty + kDecSlots;
  uint64_t* p_full = s_full + 1;
  uint64_t* o_full = p_full + 1;
  uint64_t* drain = o_full + 1;
  uint64_t* ksync = drain + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  float* red = reinterpret_cast<float*>(smem + L::kOffRed);               // [4][16]
  volatile int* vote = reinterpret_cast<volatile int*>(smem + L::kOffRed + 256);  // [4]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x % args.kv_splits;
  const int bh = blockIdx.x / args.kv_splits;  // one query block per head (Sq <= 16)
  const int qx = (bh % args.q_hpr) * D, qy = bh / args.q_hpr;
  const int kx = (bh % args.kv_hpr) * D, ky = bh / args.kv_hpr;
  const int visible = kv_blocks_for(args, 0);
  const int j0 = split * args.split_blocks;
  const int n_kv = args.kv_splits == 1 ? visible : max(0, min(visible - j0, args.split_blocks));
  const FailState fs{abort_flag, args.status};

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kDecSlots; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    mbar_init(ksync, 128);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kDecTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_trigger();
  pdl_wait();

  if (warp == 0 && n_kv > 0) {
    // ------------------------------------------------------------ producer
    // Q: the warp copies the head's Sq rows into the K-major swizzled image
    // (rows past Sq are zero); a TMA box of 16 rows could reach past the end
    // of a Q matrix of fewer rows
    // (lanes 1-31, while lane 0 already streams K and V)
    if (lane != 0) {
      const __half* qsrc = args.Q + (long long)qy * args.Sq * args.ldq + qx;
      for (int idx = lane - 1; idx < kDecRows * 16; idx += 31) {
        const int r = idx >> 4, ch = idx & 15;
        const int box = ch >> 3, cc = ch & 7;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < args.Sq) v = *reinterpret_cast<const uint4*>(qsrc + (long long)r * args.ldq + ch * 8);
        *reinterpret_cast<uint4*>(smem + L::kOffQ + box * L::kRowsBox + r * 128 +
                                  ((cc ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      __syncwarp(0xfffffffeu);
      if (lane == 1) mbar_arrive(q_full);
    } else {
      Cursor<kDecSlots> c;
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        for (int which = 0; which < 2; ++which) {  // K_j then V_j
          if (!mbar_wait(&kv_empty[c.slot], c.phase ^ 1, fs)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[c.slot], L::kTileBytes);
          const CUtensorMap* map = which ? &tmV : &tmK;
          for (int b = 0; b < 2; ++b)
            tma_load_2d(smem + L::kOffKV + c.slot * L::kTileBytes + b * kAttBoxBytes, map,
                        &kv_full[c.slot], kx + 64 * b,
                        (int)(ky * args.kv_stride) + (j0 + j) * kAttBN);
          c.advance();
          ++issued;
        }
      }
      // bounded wait for the copies still landing (complete on the normal path)
      const unsigned long long t0 = globaltimer_ns();
      while (!mbar_try_wait(q_full, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
      for (int i = 0; i < issued && i < kDecSlots; ++i) {
        if (c.slot == 0) {
          c.slot = kDecSlots - 1;
          c.phase ^= 1u;
        } else {
          --c.slot;
        }
        const unsigned long long t1 = globaltimer_ns();
        while (!mbar_try_wait(&kv_full[c.slot], c.phase) &&
               globaltimer_ns() - t1 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_kv > 0) {
      bool ok = mbar_wait(q_full, 0, fs);
      bool issued_any = false;
      Cursor<kDecSlots> c;
      const uint32_t q_addr = smem_u32(smem + L::kOffQ);
      const uint32_t p_addr = smem_u32(smem + L::kOffP);
      const uint32_t kv_addr = smem_u32(smem + L::kOffKV);
      const uint32_t s_tmem = tmem_base, o_tmem = tmem_base + kDecRows;
      int kslot = c.slot;
      if (ok) ok = mbar_wait(&kv_full[kslot], c.phase, fs);
      c.advance();
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16_ss(s_tmem, kmajor_desc(kv_addr + kslot * L::kTileBytes, kk),
                      rows16_desc(q_addr, kk), kIdescS, kk != 0);
        umma_commit(s_full);
        umma_commit(&kv_empty[kslot]);
        issued_any = true;
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const int vslot = c.slot;
        if (!mbar_wait(&kv_full[vslot], c.phase, fs)) { ok = false; break; }
        c.advance();
        const bool has_next = j + 1 < n_kv;
        if (has_next) {
          kslot = c.slot;
          if (!mbar_wait(&kv_full[kslot], c.phase, fs)) { ok = false; break; }
          c.advance();
        }
        if (!mbar_wait(p_full, (uint32_t)(j & 1), fs)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kAttBN / 16; ++kk)
          umma_f16_ss(o_tmem, vmajor_desc(kv_addr + vslot * L::kTileBytes, kk),
                      rows16_desc(p_addr, kk), kIdescO, (j | kk) != 0);
        if (has_next) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16_ss(s_tmem, kmajor_desc(kv_addr + kslot * L::kTileBytes, kk),
                        rows16_desc(q_addr, kk), kIdescS, kk != 0);
          umma_commit(s_full);
        }
        umma_commit(&kv_empty[vslot]);
        if (has_next) umma_commit(&kv_empty[kslot]);
      }
      if (ok) {
        umma_commit(o_full);
      } else if (issued_any) {
        umma_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------- key threads: softmax, epilogue
    const int quarter = warp & 3;
    const int kl = quarter * 32 + lane;  // key of the block (S^T lane), d of O^T
    const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const float c = args.c;
    float m_run[kDecRows], l_part[kDecRows];
#pragma unroll
    for (int q = 0; q < kDecRows; ++q) {
      m_run[q] = -INFINITY;
      l_part[q] = 0.0f;
    }
    uint8_t* p_smem = smem + L::kOffP;
    // barrier of the 128 key threads with a bounded wait (a thread that gave
    // up on a wait stops arriving, and the others then give up too)
    uint32_t kphase = 0;
    auto key_sync = [&]() -> bool {
      mbar_arrive(ksync);
      const bool r = mbar_wait(ksync, kphase, fs);
      kphase ^= 1u;
      return __all_sync(0xffffffffu, r);
    };
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const bool ready = mbar_wait(s_full, (uint32_t)(j & 1), fs);
      if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
      tc_fence_after();
      uint32_t u[kDecRows];
      tmem_ld_32x32b_x16(lane_base, u);
      tmem_wait_ld();
      const int key = (j0 + j) * kAttBN + kl;
      float x[kDecRows];
      bool need = false;
#pragma unroll
      for (int q = 0; q < kDecRows; ++q) {
        const int lim = args.causal ? min(args.Skv - 1, q % args.q_len + args.causal_offset)
                                    : args.Skv - 1;
        x[q] = (q < args.Sq && key <= lim) ? __uint_as_float(u[q]) * c : -INFINITY;
        need |= x[q] > m_run[q] + kRescaleLog2;
      }
      need = __any_sync(0xffffffffu, need);
      if (lane == 0) vote[quarter] = need ? 1 : 0;
      if (!key_sync()) { ok = false; break; }
      const bool any_need = (vote[0] | vote[1] | vote[2] | vote[3]) != 0;
      if (any_need) {
        // the block maximum of every row over the 128 keys
        float mx[kDecRows];
#pragma unroll
        for (int q = 0; q < kDecRows; ++q) {
          mx[q] = x[q];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mx[q] = fmaxf(mx[q], __shfl_xor_sync(0xffffffffu, mx[q], o));
        }
        if (lane < kDecRows) {
          float v = mx[0];
#pragma unroll
          for (int q = 1; q < kDecRows; ++q) v = lane == q ? mx[q] : v;
          red[quarter * kDecRows + lane] = v;
        }
        if (!key_sync()) { ok = false; break; }
        float alpha[kDecRows];
#pragma unroll
        for (int q = 0; q < kDecRows; ++q) {
          const float m_blk = fmaxf(fmaxf(red[q], red[kDecRows + q]),
                                    fmaxf(red[2 * kDecRows + q], red[3 * kDecRows + q]));
          const float m_new = fmaxf(m_run[q], m_blk);
          alpha[q] = m_run[q] == -INFINITY ? 0.0f : ex2_approx(m_run[q] - m_new);
          l_part[q] *= alpha[q];
          m_run[q] = m_new;
        }
        // O^T(j-1) is complete: S^T(j) was issued after PV(j-1)
        if (j > 0) {
          uint32_t o[kDecRows];
          tmem_ld_32x32b_x16(lane_base + kDecRows, o);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < kDecRows; ++q) o[q] = __float_as_uint(__uint_as_float(o[q]) * alpha[q]);
          tmem_st_32x32b_x16(lane_base + kDecRows, o);
          tmem_wait_st();
        }
        // every thread has read `red` before the next block may rewrite it
        if (!key_sync()) { ok = false; break; }
      }
      // P^T[key kl][q] into the K-major [16 rows][128 keys] image of P
      const int box = kl >> 6, kc = kl & 63;
#pragma unroll
      for (int q = 0; q < kDecRows; ++q) {
        const float m_use = m_run[q] == -INFINITY ? 0.0f : m_run[q];
        const float pv = ex2_approx(x[q] - m_use);
        l_part[q] += pv;
        *reinterpret_cast<__half*>(p_smem + box * L::kRowsBox + q * 128 +
                                   ((((kc >> 3) ^ (q & 7))) << 4) + (kc & 7) * 2) =
            __float2half_rn(pv);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // ------------------------------------------------------------ epilogue
    bool have = ok && n_kv > 0;
    if (have) have = mbar_wait(o_full, 0, fs);
    const bool all_have = __all_sync(0xffffffffu, have);
    // row sums over the 128 key threads
#pragma unroll
    for (int q = 0; q < kDecRows; ++q)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l_part[q] += __shfl_xor_sync(0xffffffffu, l_part[q], o);
    bool synced = ok && key_sync();  // `red` is free
    if (synced && lane < kDecRows) {
      float v = l_part[0];
#pragma unroll
      for (int q = 1; q < kDecRows; ++q) v = lane == q ? l_part[q] : v;
      red[quarter * kDecRows + lane] = v;
    }
    if (synced) synced = key_sync();
    uint32_t o[kDecRows];
    if (all_have) {
      tc_fence_after();
      tmem_ld_32x32b_x16(lane_base + kDecRows, o);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int q = 0; q < kDecRows; ++q) o[q] = 0u;
    }
    const bool write_ok = synced && (ok || n_kv == 0);
    const bool partial = args.kv_splits > 1;
#pragma unroll
    for (int q = 0; q < kDecRows; ++q) {
      if (q >= args.Sq || !write_ok) continue;
      const float l = red[q] + red[kDecRows + q] + red[2 * kDecRows + q] + red[3 * kDecRows + q];
      const float inv = (all_have && l > 0.0f) ? 1.0f / l : 0.0f;
      const float v = __uint_as_float(o[q]) * inv;
      if (partial) {
        const size_t pidx = (size_t)blockIdx.x * args.part_rows + q;
        if (kl == 0)
          args.part_lse[pidx] = (all_have && l > 0.0f) ? m_run[q] + log2f(l) : -INFINITY;
        args.part_o[pidx * D + kl] = v;
      } else {
        const long long qhead = (long long)bh * args.group + q / args.q_len;
        __half* orow = args.O + (qhead / args.o_hpr * args.q_len + q % args.q_len) * args.ldo +
                       qhead % args.o_hpr * D;
        orow[kl] = __float2half_rn(v);
      }
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kDecTmemCols);
  }
}

// Split keys: one warp per (CTA head, query row) merges the kv_splits
// partial results of the row, each a normalised O_i with its log2-sum-exp2
// L_i: O = sum_i 2^(L_i - M) O_i / sum_i 2^(L_i - M), M = max_i L_i. A row
// whose partials are all -inf (no visible key) is 0.
template <int D>
__global__ void __launch_bounds__(256)
    attention_combine_kernel(const AttArgs args, int heads) {
  pdl_wait();
  pdl_trigger();
  constexpr int kPer = D / 32;  // O elements per lane
  const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (long long)heads * args.Sq) return;
  const int bh = (int)(gw / args.Sq), qrow = (int)(gw % args.Sq);
  const int qb = qrow / args.q_rows, prow = qrow % args.q_rows;
  const size_t unit0 = ((size_t)bh * args.q_blocks + qb) * args.kv_splits;
  const int S = args.kv_splits;
  // lane-parallel: the row maximum of the splits' log2-sum-exp2
  float mx = -INFINITY;
  for (int sp = lane; sp < S; sp += 32)
    mx = fmaxf(mx, args.part_lse[(unit0 + sp) * args.part_rows + prow]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float acc[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) acc[e] = 0.0f;
  float wsum = 0.0f;
  if (mx != -INFINITY) {
    for (int base = 0; base < S; base += 32) {
      // lane l holds the weight of split base + l; the partial rows are
      // loaded four splits at a time, so a row costs few memory round trips
      const int n = min(32, S - base);
      const float l2 =
          lane < n ? args.part_lse[(unit0 + base + lane) * args.part_rows + prow] : -INFINITY;
      const float w = ex2_approx(l2 - mx);  // 0 for -inf
      wsum += w;
      for (int j = 0; j < n; j += 4) {
        float o[4][kPer];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const size_t idx = (unit0 + base + min(j + u, n - 1)) * args.part_rows + prow;
          const float* po = args.part_o + idx * D + lane * kPer;
          if constexpr (kPer == 4) {
            const float4 v = *reinterpret_cast<const float4*>(po);
            o[u][0] = v.x, o[u][1] = v.y, o[u][2] = v.z, o[u][3] = v.w;
          } else {
            const float2 v = *reinterpret_cast<const float2*>(po);
            o[u][0] = v.x, o[u][1] = v.y;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float wu = j + u < n ? __shfl_sync(0xffffffffu, w, j + u) : 0.0f;
#pragma unroll
          for (int e = 0; e < kPer; ++e) acc[e] = fmaf(wu, o[u][e], acc[e]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  }
  const float inv = wsum > 0.0f ? 1.0f / wsum : 0.0f;
  const long long qhead = (long long)bh * args.group + qrow / args.q_len;
  __half* orow = args.O + (qhead / args.o_hpr * args.q_len + qrow % args.q_len) * args.ldo +
                 qhead % args.o_hpr * D + lane * kPer;
  if constexpr (kPer == 4) {
    uint2 v;
    v.x = pack_half2(acc[0] * inv, acc[1] * inv);
    v.y = pack_half2(acc[2] * inv, acc[3] * inv);
    *reinterpret_cast<uint2*>(orow) = v;
  } else {
    *reinterpret_cast<uint32_t*>(orow) = pack_half2(acc[0] * inv, acc[1] * inv);
  }
}

// 2-D map over a row-major [rows, ld] f16 matrix read in [box_rows x 64]
// boxes (128-byte swizzle).
hxb_status_t make_rows_map(CUtensorMap* m, const void* base, int64_t rows, int64_t ld,
                           uint32_t box_rows = 128) {
  const uint64_t dims[2] = {(uint64_t)ld, (uint64_t)rows};
  const uint64_t strides[1] = {(uint64_t)ld * 2};
  const uint32_t box[2] = {64, box_rows};
  return encode_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
}

// Operand layout of one attention launch (see AttArgs for the mapping).
struct AttLayout {
  const void *Q, *K, *V;
  void* O;
  int64_t ldq, ldk, ldv, ldo;  // row pitches (elements)
  int64_t heads;               // CTA heads: batch x KV heads
  int64_t q_hpr, kv_hpr;       // Q and K/V heads per row
  int64_t group;               // query heads per KV head
  int64_t q_len;               // query positions per query head
  int64_t Skv;                 // keys attended per head
  int64_t kv_stride;           // K/V rows per head (>= Skv)
  int64_t o_hpr;               // O heads per row
  int64_t D;
  int64_t q_pos0;              // causal: key j is visible to position i iff j <= q_pos0 + i
  void* workspace;             // split-key partials (null: no split)
  size_t workspace_bytes;
};

// How the keys of one query block are split across CTAs: for short queries
// (one query tile per CTA: decode, speculative or chunked steps) enough
// splits to fill one wave of the SMs when the query blocks alone do not, with
// at least one key block per split. Longer queries run unsplit.
struct SplitPlan {
  int splits = 1, split_blocks = 0, part_rows = 0;
  size_t bytes = 0;  // workspace the partials need (0 without a split)
};

// CTAs that run at once: the decode kernel (1-16 rows per head, D = 128)
// fits two per SM, the others one.
bool uses_decode_kernel(int64_t Sq, int64_t D) { return D == 128 && Sq >= 1 && Sq <= kDecRows; }
int split_units(int64_t Sq, int64_t D, int num_sms) {
  return uses_decode_kernel(Sq, D) ? 2 * num_sms : num_sms;
}

SplitPlan plan_splits(int64_t ctas, int64_t Sq, int64_t Skv, int64_t D, int num_sms) {
  SplitPlan p;
  const int64_t blocks = (Skv + kAttBN - 1) / kAttBN;
  p.split_blocks = (int)blocks;
  const int64_t want = ctas > 0 ? num_sms / ctas : 0;
  if (want < 2 || blocks < 2 || Sq > kAttBM) return p;
  const int64_t per = (blocks + std::min(want, blocks) - 1) / std::min(want, blocks);
  const int64_t splits = (blocks + per - 1) / per;
  if (splits < 2) return p;
  p.splits = (int)splits;
  p.split_blocks = (int)per;
  p.part_rows = (int)std::min<int64_t>(kAttTiles * kAttBM, Sq);
  const size_t rows = (size_t)(ctas * splits) * (size_t)p.part_rows;
  p.bytes = (rows * sizeof(float) + 15) / 16 * 16 + rows * (size_t)D * sizeof(float);
  return p;
}

template <int D>
hxb_status_t launch_d(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                      const AttArgs& args, int64_t heads, int ordinal, cudaStream_t stream) {
  static bool configured[64] = {};
  if (!configured[ordinal]) {
    // the kernel's register split assumes this launch count; with fewer
    // registers at launch its increase could never be granted
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, attention_fwd_kernel<D>);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncGetAttributes(attention)");
    if (fa.numRegs != kAttRegsLaunch)
      return fail(HXB_STATUS_UNSUPPORTED, "attention kernel built with %d registers per thread, "
                  "its register split needs %d", fa.numRegs, kAttRegsLaunch);
    e = cudaFuncSetAttribute(attention_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             AttSmem<D>::kAlloc);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(attention)");
    configured[ordinal] = true;
  }
  const int64_t ctas = heads * args.q_blocks * args.kv_splits;
  hxb_status_t s = launch_pdl(attention_fwd_kernel<D>, dim3((unsigned)ctas), dim3(kAttThreads),
                              AttSmem<D>::kAlloc, stream, "attention launch", tmQ, tmK, tmV, args);
  if (s != HXB_OK || args.kv_splits == 1) return s;
  const int64_t warps = heads * args.Sq;
  return launch_pdl(attention_combine_kernel<D>, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0,
                    stream, "attention combine launch", args, (int)heads);
}

// The keys-on-lanes kernel for at most 16 query rows per head (D = 128).
hxb_status_t launch_decode(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                           const AttArgs& args, int64_t heads, int ordinal, cudaStream_t stream) {
  static bool configured[64] = {};
  if (!configured[ordinal]) {
    cudaError_t e = cudaFuncSetAttribute(attention_decode_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         DecSmem::kAlloc);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(attention decode)");
    // all of the unified L1 as shared memory: two CTAs per SM
    e = cudaFuncSetAttribute(attention_decode_kernel,
                             cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(attention decode carveout)");
    configured[ordinal] = true;
  }
  const int64_t ctas = heads * args.kv_splits;
  hxb_status_t s = launch_pdl(attention_decode_kernel, dim3((unsigned)ctas), dim3(kDecThreads),
                              DecSmem::kAlloc, stream, "attention decode launch", tmQ, tmK, tmV,
                              args);
  if (s != HXB_OK || args.kv_splits == 1) return s;
  const int64_t warps = heads * args.Sq;
  return launch_pdl(attention_combine_kernel<128>, dim3((unsigned)((warps + 7) / 8)), dim3(256),
                    0, stream, "attention combine launch", args, (int)heads);
}

hxb_status_t attention_run(const AttLayout& a, float scale, int causal, cudaStream_t stream) {
  const int64_t D = a.D;
  if (a.heads < 1 || a.q_len < 1 || a.Skv < 1 || a.group < 1 || a.q_hpr < 1 || a.kv_hpr < 1 ||
      a.o_hpr < 1)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: batch, heads, Sq, Skv must be >= 1");
  if (D != 64 && D != 128)
    return fail(HXB_STATUS_UNSUPPORTED,
                "attention: head dim %lld not supported (D = 64 or 128)", (long long)D);
  if (!a.Q || !a.K || !a.V || !a.O)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: null operand");
  if (!aligned16(a.Q) || !aligned16(a.K) || !aligned16(a.V) || !aligned16(a.O))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: Q/K/V/O must be 16-byte aligned");
  if (a.ldq % 8 || a.ldk % 8 || a.ldv % 8 || a.ldo % 8)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "attention: row pitches must be multiples of 8 elements (16 bytes)");
  if (a.ldq < a.q_hpr * D || a.ldk < a.kv_hpr * D || a.ldv < a.kv_hpr * D ||
      a.ldo < a.o_hpr * D)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: row pitch smaller than the heads it holds");
  if (causal && (a.q_pos0 < -(int64_t)(1 << 30) || a.q_pos0 > (int64_t)(1 << 30)))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: query position out of range");
  if (a.kv_stride < a.Skv)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: kv_len %lld exceeds the %lld cache rows",
                (long long)a.Skv, (long long)a.kv_stride);
  if (a.heads % a.q_hpr || a.heads % a.kv_hpr || (a.heads * a.group) % a.o_hpr ||
      (a.group > 1 && a.q_hpr != 1))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: inconsistent head layout");
  if (!(scale > 0.0f) || !isfinite(scale))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: scale must be finite and > 0");
  if (a.q_len > (1 << 30) || a.Skv > (1 << 30) || a.group > (1 << 20) ||
      a.group * a.q_len > (1 << 30))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: extent too large");
  const int64_t Sq = a.group * a.q_len;
  const int64_t rows_q = a.heads / a.q_hpr * Sq, rows_kv = a.heads / a.kv_hpr * a.kv_stride;
  if (rows_q > INT32_MAX || rows_kv > INT32_MAX)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: extent too large");
  DeviceInfo* dev = nullptr;
  hxb_status_t s = current_device(&dev);
  if (s != HXB_OK) return s;
  // Query blocks of two 128-row tiles (the tiles take turns on the tensor
  // core), or of one tile when two-tile blocks would leave SMs idle (a
  // prefill of a few hundred rows: twice the CTAs, half the longest causal
  // walk).
  int64_t q_rows = kAttTiles * kAttBM;
  if (Sq > kAttBM && (Sq + q_rows - 1) / q_rows * a.heads < dev->num_sms) q_rows = kAttBM;
  const int64_t q_blocks = (Sq + q_rows - 1) / q_rows;
  if (q_blocks * a.heads > INT32_MAX / 1024)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: too many query tiles");
  SplitPlan plan = plan_splits(q_blocks * a.heads, Sq, a.Skv, D, split_units(Sq, D, dev->num_sms));
  if (plan.splits > 1 && (!a.workspace || a.workspace_bytes < plan.bytes ||
                          (reinterpret_cast<uintptr_t>(a.workspace) & 15u))) {
    plan = SplitPlan{};  // no room for partials: one CTA walks all the keys
    plan.split_blocks = (int)((a.Skv + kAttBN - 1) / kAttBN);
  }
  // 1 to 16 query rows per head (decode, grouped-query decode, short steps):
  // the keys-on-lanes kernel. With two CTAs per SM it also beats
  // attention_fwd_kernel on a single row per head (multi-head decode: the
  // cfg 4 decode step 95.4 -> 93.6 us on one B200).
  const bool decode = uses_decode_kernel(Sq, D);
  const int q_box = (int)std::min<int64_t>(kAttBM, (Sq + 7) / 8 * 8);
  CUtensorMap tmQ, tmK, tmV;
  if ((s = make_rows_map(&tmQ, a.Q, rows_q, a.ldq, (uint32_t)q_box)) != HXB_OK) return s;
  if ((s = make_rows_map(&tmK, a.K, rows_kv, a.ldk)) != HXB_OK) return s;
  if ((s = make_rows_map(&tmV, a.V, rows_kv, a.ldv)) != HXB_OK) return s;

  AttArgs args{};
  args.Sq = (int)Sq;
  args.Skv = (int)a.Skv;
  args.q_hpr = (int)a.q_hpr;
  args.kv_hpr = (int)a.kv_hpr;
  args.q_len = (int)a.q_len;
  args.group = (int)a.group;
  args.o_hpr = (int)a.o_hpr;
  args.kv_stride = a.kv_stride;
  args.ldo = a.ldo;
  args.q_rows = (int)q_rows;
  args.q_blocks = (int)q_blocks;
  args.q_box = q_box;
  args.kv_splits = plan.splits;
  args.split_blocks = plan.split_blocks;
  args.part_rows = plan.part_rows;
  if (plan.splits > 1) {
    args.part_lse = static_cast<float*>(a.workspace);
    const size_t lse_bytes = ((size_t)q_blocks * a.heads * plan.splits * plan.part_rows *
                                  sizeof(float) + 15) / 16 * 16;
    args.part_o = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + lse_bytes);
  }
  args.causal = causal ? 1 : 0;
  args.causal_offset = (int)a.q_pos0;
  args.c = (float)((double)scale * 1.4426950408889634);  // scale * log2(e)
  args.O = static_cast<__half*>(a.O);
  args.Q = static_cast<const __half*>(a.Q);
  args.ldq = a.ldq;
  args.status = dev->status_word;
  if (decode) return launch_decode(tmQ, tmK, tmV, args, a.heads, dev->ordinal, stream);
  return D == 64 ? launch_d<64>(tmQ, tmK, tmV, args, a.heads, dev->ordinal, stream)
                 : launch_d<128>(tmQ, tmK, tmV, args, a.heads, dev->ordinal, stream);
}

}  // namespace

// Dynamic shared memory (bytes) and threads per CTA of the attention kernel
// (the executable library's export attributes): the larger of the two
// head-dimension instances.
size_t attention_smem_bytes() {
  return AttSmem<128>::kAlloc > AttSmem<64>::kAlloc ? AttSmem<128>::kAlloc : AttSmem<64>::kAlloc;
}
int attention_threads() { return kAttThreads; }

// Shared launcher: B batches x H heads; hpr heads per matrix row (see AttArgs).
hxb_status_t attention_launch(const void* Q, int64_t ldq, const void* K, int64_t ldk,
                              const void* V, int64_t ldv, void* O, int64_t ldo, int64_t B,
                              int64_t H, int64_t hpr, int64_t Sq, int64_t Skv, int64_t D,
                              float scale, int causal, cudaStream_t stream) {
  if (B < 1 || H < 1)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: batch, heads, Sq, Skv must be >= 1");
  AttLayout a{};
  a.Q = Q, a.K = K, a.V = V, a.O = O;
  a.ldq = ldq, a.ldk = ldk, a.ldv = ldv, a.ldo = ldo;
  a.heads = B * H;
  a.q_hpr = a.kv_hpr = a.o_hpr = hpr;
  a.group = 1;
  a.q_len = Sq;
  a.Skv = a.kv_stride = Skv;
  a.D = D;
  a.q_pos0 = Skv - Sq;
  return attention_run(a, scale, causal, stream);
}

// Grouped-query attention over the first kv_len rows of a KV cache.
hxb_status_t attention_gqa_launch(const void* Q, const void* K, const void* V, void* O,
                                  int64_t batch, int64_t q_heads, int64_t kv_heads,
                                  int64_t q_len, int64_t q_pos0, int64_t kv_len,
                                  int64_t kv_rows, int64_t D, float scale, int causal,
                                  int out_layout, void* workspace, size_t workspace_bytes,
                                  cudaStream_t stream) {
  if (batch < 1 || q_heads < 1 || kv_heads < 1)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: batch and heads must be >= 1");
  if (q_heads % kv_heads)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "attention: %lld query heads are not a multiple of %lld KV heads",
                (long long)q_heads, (long long)kv_heads);
  if (out_layout != HXB_ATTN_OUT_BHSD && out_layout != HXB_ATTN_OUT_BSHD)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: unknown output layout %d", out_layout);
  if (batch > INT32_MAX || q_heads > INT32_MAX)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: extent too large");
  const bool bshd = out_layout == HXB_ATTN_OUT_BSHD;
  AttLayout a{};
  a.Q = Q, a.K = K, a.V = V, a.O = O;
  a.ldq = a.ldk = a.ldv = D;
  a.ldo = bshd ? q_heads * D : D;
  a.heads = batch * kv_heads;
  a.q_hpr = a.kv_hpr = 1;
  a.o_hpr = bshd ? q_heads : 1;
  a.group = q_heads / kv_heads;
  a.q_len = q_len;
  a.Skv = kv_len;
  a.kv_stride = kv_rows;
  a.D = D;
  a.q_pos0 = q_pos0;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return attention_run(a, scale, causal, stream);
}

// Upper bound of the split-key workspace of any call with Sq query rows per
// CTA head on the current device, whatever the number of keys: the splits
// never make more CTAs than can run at once.
size_t attention_split_bound(int64_t Sq, int64_t D) {
  DeviceInfo* dev = nullptr;
  if (Sq < 1 || Sq > kAttBM || current_device(&dev) != HXB_OK) return 0;
  const size_t rows = (size_t)split_units(Sq, D, dev->num_sms) * (size_t)Sq;
  return (rows * sizeof(float) + 15) / 16 * 16 + rows * (size_t)D * sizeof(float);
}

// Self-attention of new rows against a KV cache: Q is [batch * seq, ldq]
// with head h at columns [h*D, +D) (a fused QKV output), K/V caches are
// [batch, heads, cache_rows, D], keys [0, kv_len) attended causally from
// position q_pos0; O is [batch * seq, ldo] in the layout of Q.
hxb_status_t attention_cached_launch(const void* Q, int64_t ldq, const void* k_cache,
                                     const void* v_cache, int64_t cache_rows, void* O,
                                     int64_t ldo, int64_t batch, int64_t heads, int64_t seq,
                                     int64_t kv_len, int64_t q_pos0, int64_t D, float scale,
                                     void* workspace, size_t workspace_bytes,
                                     cudaStream_t stream) {
  if (batch < 1 || heads < 1)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: batch and heads must be >= 1");
  AttLayout a{};
  a.Q = Q, a.K = k_cache, a.V = v_cache, a.O = O;
  a.ldq = ldq, a.ldk = a.ldv = D, a.ldo = ldo;
  a.heads = batch * heads;
  a.q_hpr = a.o_hpr = heads;
  a.kv_hpr = 1;
  a.group = 1;
  a.q_len = seq;
  a.Skv = kv_len;
  a.kv_stride = cache_rows;
  a.D = D;
  a.q_pos0 = q_pos0;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return attention_run(a, scale, 1, stream);
}

// Workspace the split-key plan of a GQA call needs on the current device (0:
// the call does not split, or the shape or device is invalid).
size_t attention_gqa_workspace(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t q_len,
                               int64_t kv_len, int64_t D) {
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || q_len < 1 || kv_len < 1 ||
      q_heads % kv_heads || (D != 64 && D != 128) || batch > INT32_MAX || q_heads > INT32_MAX ||
      q_len > (1 << 30) || kv_len > (1 << 30) || (q_heads / kv_heads) * q_len > (1 << 30))
    return 0;
  DeviceInfo* dev = nullptr;
  if (current_device(&dev) != HXB_OK) return 0;
  const int64_t Sq = q_heads / kv_heads * q_len;
  const int64_t q_blocks = (Sq + kAttTiles * kAttBM - 1) / (kAttTiles * kAttBM);
  return plan_splits(q_blocks * batch * kv_heads, Sq, kv_len, D,
                     split_units(Sq, D, dev->num_sms)).bytes;
}

}  // namespace hxb

extern "C" hxb_status_t hxb_attention_f16(const void* Q, const void* K, const void* V,
                                          void* O, int64_t BH, int64_t Sq, int64_t Skv,
                                          int64_t D, float scale, int causal,
                                          void* stream) {
  return hxb::attention_launch(Q, D, K, D, V, D, O, D, BH, 1, 1, Sq, Skv, D, scale, causal,
                               static_cast<cudaStream_t>(stream));
}

extern "C" hxb_status_t hxb_attention_f16_bshd(const void* Q, int64_t ldq, const void* K,
                                               int64_t ldk, const void* V, int64_t ldv, void* O,
                                               int64_t ldo, int64_t batch, int64_t heads,
                                               int64_t Sq, int64_t Skv, int64_t D, float scale,
                                               int causal, void* stream) {
  return hxb::attention_launch(Q, ldq, K, ldk, V, ldv, O, ldo, batch, heads, heads, Sq, Skv, D,
                               scale, causal, static_cast<cudaStream_t>(stream));
}

extern "C" hxb_status_t hxb_attention_gqa_f16(const void* Q, const void* K, const void* V,
                                              void* O, int64_t batch, int64_t q_heads,
                                              int64_t kv_heads, int64_t q_len, int64_t q_pos0,
                                              int64_t kv_len, int64_t kv_rows, int64_t D,
                                              float scale, int causal, int out_layout,
                                              void* workspace, size_t workspace_bytes,
                                              void* stream) {
  return hxb::attention_gqa_launch(Q, K, V, O, batch, q_heads, kv_heads, q_len, q_pos0, kv_len,
                                   kv_rows, D, scale, causal, out_layout, workspace,
                                   workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" size_t hxb_attention_gqa_workspace_bytes(int64_t batch, int64_t q_heads,
                                                    int64_t kv_heads, int64_t q_len,
                                                    int64_t kv_len, int64_t D) {
  return hxb::attention_gqa_workspace(batch, q_heads, kv_heads, q_len, kv_len, D);
}
