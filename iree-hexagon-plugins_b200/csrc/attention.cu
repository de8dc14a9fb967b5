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

#include "runtime_common.h"
#include "sm100.cuh"

namespace hxb {
namespace {

constexpr int kAttD = 128;       // head dimension
constexpr int kAttBM = 128;      // query rows per tile
constexpr int kAttTiles = 2;     // query tiles per CTA
constexpr int kAttBN = 128;      // keys per block
constexpr int kAttSlots = 4;     // K/V ring slots
constexpr int kAttTileBytes = 128 * kAttD * 2;  // one [128 x 128] f16 tile
constexpr int kAttBoxBytes = 128 * 64 * 2;      // one TMA box: 128 rows x 64 f16
constexpr float kRescaleLog2 = 8.0f;
constexpr int kAttThreads = 384;

struct AttSmem {
  static constexpr int kOffQ = 0;
  static constexpr int kOffKV = kOffQ + kAttTiles * kAttTileBytes;
  static constexpr int kOffBar = kOffKV + kAttSlots * kAttTileBytes;
  // q_full, kv_full[slots], kv_empty[slots], s_full[2], p_full[2], o_full, drain
  static constexpr int kNumBars = 1 + 2 * kAttSlots + 2 * kAttTiles + 2;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

// Q, K, V and O are row-major matrices of B*S rows; head h of batch b
// occupies rows [b*S, (b+1)*S) and columns [(h % hpr) * 128, +128) with
// hpr heads per row: hpr = 1 is the contiguous [B*H, S, D] layout,
// hpr = H the [B, S, H*D] layout (e.g. the Q/K/V column blocks of a fused QKV
// projection output). Rows of a tile past S belong to the next head or batch
// (or lie outside the matrix and read as zeros): their keys are masked and
// their query rows are not stored.
struct AttArgs {
  int Sq, Skv;
  int hpr;            // heads per row
  long long ldo;      // O row pitch (elements)
  int q_blocks;       // CTAs per head: ceil(Sq / 256)
  int causal;
  int causal_offset;  // Skv - Sq: key j is visible to query i iff j <= i + offset
  float c;            // scale * log2(e)
  __half* O;
  int* status;
};

// Number of key blocks CTA rows [q0, q0+256) may see.
__device__ __forceinline__ int kv_blocks_for(const AttArgs& a, int q0) {
  int last_key = a.Skv - 1;
  if (a.causal) {
    const int last_row = min(q0 + kAttTiles * kAttBM, a.Sq) - 1;
    last_key = min(last_key, last_row + a.causal_offset);
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

__global__ void __launch_bounds__(kAttThreads, 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const AttArgs args) {
  using L = AttSmem;
  constexpr uint32_t kIdescQK = make_idesc_f16(kAttBM, kAttBN, 0, 0);
  constexpr uint32_t kIdescPV = make_idesc_f16(kAttBM, kAttD, 0, 1);

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
  const int qb = blockIdx.x % args.q_blocks;
  const int bh = blockIdx.x / args.q_blocks;
  const int hx = (bh % args.hpr) * kAttD;  // column of this head
  const int hb = bh / args.hpr;            // row block (batch) of this head
  const int q0 = qb * kAttTiles * kAttBM;
  const int n_kv = kv_blocks_for(args, q0);
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

  if (warp == 0) {
    // -------------------------------------------------------- TMA producer
    if (lane == 0 && n_kv > 0) {
      mbar_arrive_expect_tx(q_full, kAttTiles * kAttTileBytes);
      for (int t = 0; t < kAttTiles; ++t)
        for (int b = 0; b < 2; ++b)
          tma_load_2d(smem + L::kOffQ + t * kAttTileBytes + b * kAttBoxBytes, &tmQ, q_full,
                      hx + 64 * b, hb * args.Sq + q0 + t * kAttBM);
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
          for (int b = 0; b < 2; ++b)
            tma_load_2d(smem + L::kOffKV + c.slot * kAttTileBytes + b * kAttBoxBytes, map,
                        &kv_full[c.slot], hx + 64 * b, hb * args.Skv + j * kAttBN);
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
      const uint32_t q_addr = smem_u32(smem + L::kOffQ);
      const uint32_t kv_addr = smem_u32(smem + L::kOffKV);
      // S_t(0) = Q_t K_0^T
      int kslot = c.slot;
      if (ok) ok = mbar_wait(&kv_full[kslot], c.phase, fs);
      c.advance();
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < kAttTiles; ++t) {
#pragma unroll
          for (int kk = 0; kk < kAttD / 16; ++kk)
            umma_f16_ss(tmem_base + t * 128, kmajor_desc(q_addr + t * kAttTileBytes, kk),
                        kmajor_desc(kv_addr + kslot * kAttTileBytes, kk), kIdescQK, kk != 0);
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
        for (int t = 0; t < kAttTiles && ok; ++t) {
          if (!mbar_wait(&p_full[t], (uint32_t)(j & 1), fs)) { ok = false; break; }
          tc_fence_after();
          const uint32_t o_tmem = tmem_base + 256 + t * 128;
          const uint32_t p_tmem = tmem_base + t * 128 + 64;
#pragma unroll
          for (int kk = 0; kk < kAttBN / 16; ++kk)
            umma_f16_ts(o_tmem, p_tmem + kk * 8, vmajor_desc(kv_addr + vslot * kAttTileBytes, kk),
                        kIdescPV, (j | kk) != 0);
          if (has_next) {
#pragma unroll
            for (int kk = 0; kk < kAttD / 16; ++kk)
              umma_f16_ss(tmem_base + t * 128, kmajor_desc(q_addr + t * kAttTileBytes, kk),
                          kmajor_desc(kv_addr + kslot * kAttTileBytes, kk), kIdescQK, kk != 0);
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
  } else if (warp >= 4) {
    // -------------------------------------------------------- softmax
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qrow = q0 + t * kAttBM + r;
    const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const uint32_t s_col = t * 128, p_col = t * 128 + 64, o_col = 256 + t * 128;
    const float c = args.c;
    float m_run = -INFINITY;  // running max of S*c (log2 domain)
    float l_run = 0.0f;       // running sum of P against m_run
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
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
      const int key0 = j * kAttBN;
      if (key0 + kAttBN > args.Skv || args.causal) {
        const int lim = args.causal ? min(args.Skv - 1, qrow + args.causal_offset) : args.Skv - 1;
#pragma unroll
        for (int e = 0; e < kAttBN; ++e)
          if (key0 + e > lim) s[e] = -INFINITY;
      }
      float mx = s[0];
#pragma unroll
      for (int e = 1; e < kAttBN; ++e) mx = fmaxf(mx, s[e]);
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
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t u[32];
          tmem_ld_32x32b_x32(lane_base + o_col + ch * 32, u);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
          tmem_st_32x32b_x32(lane_base + o_col + ch * 32, u);
        }
      }
      const float m_use = m_run == -INFINITY ? 0.0f : m_run;
      float sum = 0.0f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float p0 = ex2_approx(fmaf(s[h * 64 + 2 * e], c, -m_use));
          const float p1 = ex2_approx(fmaf(s[h * 64 + 2 * e + 1], c, -m_use));
          sum += p0 + p1;
          pk[e] = pack_half2(p0, p1);
        }
        tmem_st_32x32b_x32(lane_base + p_col + h * 32, pk);
      }
      l_run += sum;
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
    __half* orow = args.O + ((long long)hb * args.Sq + qrow) * args.ldo + hx;
    const bool write = (ok || n_kv == 0) && qrow < args.Sq;
#pragma unroll 1
    for (int ch = 0; ch < 4; ++ch) {
      uint32_t u[32];
      if (all_have) {
        tmem_ld_32x32b_x32(lane_base + o_col + ch * 32, u);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) u[e] = 0u;
      }
      if (write) {
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

// 2-D map over a row-major [rows, ld] f16 matrix read in [128 rows x 64]
// boxes (128-byte swizzle).
hxb_status_t make_rows_map(CUtensorMap* m, const void* base, int64_t rows, int64_t ld) {
  const uint64_t dims[2] = {(uint64_t)ld, (uint64_t)rows};
  const uint64_t strides[1] = {(uint64_t)ld * 2};
  const uint32_t box[2] = {64, 128};
  return encode_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

// Dynamic shared memory (bytes) and threads per CTA of the attention kernel
// (the executable library's export attributes).
size_t attention_smem_bytes() { return AttSmem::kAlloc; }
int attention_threads() { return kAttThreads; }

// Shared launcher: B batches x H heads; hpr heads per matrix row (see AttArgs).
hxb_status_t attention_launch(const void* Q, int64_t ldq, const void* K, int64_t ldk,
                              const void* V, int64_t ldv, void* O, int64_t ldo, int64_t B,
                              int64_t H, int64_t hpr, int64_t Sq, int64_t Skv, int64_t D,
                              float scale, int causal, cudaStream_t stream) {
  if (B < 1 || H < 1 || Sq < 1 || Skv < 1)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: batch, heads, Sq, Skv must be >= 1");
  if (D != kAttD)
    return fail(HXB_STATUS_UNSUPPORTED, "attention: head dim %lld not supported (D = 128 only)",
                (long long)D);
  if (!Q || !K || !V || !O)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: null operand");
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: Q/K/V/O must be 16-byte aligned");
  if (ldq % 8 || ldk % 8 || ldv % 8 || ldo % 8)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "attention: row pitches must be multiples of 8 elements (16 bytes)");
  if (ldq < hpr * D || ldk < hpr * D || ldv < hpr * D || ldo < hpr * D)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: row pitch smaller than the heads it holds");
  if (!(scale > 0.0f) || !isfinite(scale))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: scale must be finite and > 0");
  const int64_t BH = B * H;
  const int64_t rows_q = BH / hpr * Sq, rows_kv = BH / hpr * Skv;
  if (Sq > (1 << 30) || Skv > (1 << 30) || rows_q > INT32_MAX || rows_kv > INT32_MAX)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: extent too large");
  const int64_t q_blocks = (Sq + kAttTiles * kAttBM - 1) / (kAttTiles * kAttBM);
  if (q_blocks * BH > INT32_MAX)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "attention: too many query tiles");

  DeviceInfo* dev = nullptr;
  hxb_status_t s = current_device(&dev);
  if (s != HXB_OK) return s;
  CUtensorMap tmQ, tmK, tmV;
  if ((s = make_rows_map(&tmQ, Q, rows_q, ldq)) != HXB_OK) return s;
  if ((s = make_rows_map(&tmK, K, rows_kv, ldk)) != HXB_OK) return s;
  if ((s = make_rows_map(&tmV, V, rows_kv, ldv)) != HXB_OK) return s;

  AttArgs args{};
  args.Sq = (int)Sq;
  args.Skv = (int)Skv;
  args.hpr = (int)hpr;
  args.ldo = ldo;
  args.q_blocks = (int)q_blocks;
  args.causal = causal ? 1 : 0;
  args.causal_offset = (int)(Skv - Sq);
  args.c = (float)((double)scale * 1.4426950408889634);  // scale * log2(e)
  args.O = static_cast<__half*>(O);
  args.status = dev->status_word;

  static bool configured[64] = {};
  if (!configured[dev->ordinal]) {
    cudaError_t e = cudaFuncSetAttribute(attention_fwd_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         AttSmem::kAlloc);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(attention)");
    configured[dev->ordinal] = true;
  }
  attention_fwd_kernel<<<(unsigned)(q_blocks * BH), kAttThreads, AttSmem::kAlloc, stream>>>(
      tmQ, tmK, tmV, args);
  return cuda_status(cudaGetLastError(), "attention launch");
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
