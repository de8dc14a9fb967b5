// Host launchers for the tcgen05 GEMM dispatches (f16 and int8-weight).
#include <string.h>

#include "gemm_sm100.cuh"
#include "gemm_splitk_sm100.cuh"
#include "gemm_w8_sm100.cuh"
#include "gemv_w8_sk_sm100.cuh"
#include "gemv_w8_sm100.cuh"
#include "planner.h"
#include "runtime_common.h"

namespace hxb {

namespace {

template <int BN, int STAGES, int BMODE, int OUT>
hxb_status_t launch_gemm(const DeviceInfo& dev, const CUtensorMap& tmA,
                         const CUtensorMap& tmB, const GemmArgs& args,
                         cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES, BMODE>;
  auto kernel = gemm_sm100_kernel<BN, STAGES, BMODE, OUT>;
  // Per-device attribute: set once per (device, instantiation).
  static bool configured[64] = {};
  if (!configured[dev.ordinal]) {
    cudaError_t e = cudaFuncSetAttribute(
        kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm)");
    configured[dev.ordinal] = true;
  }
  const int tiles = args.tiles_m * args.tiles_n;
  const int grid = tiles < dev.num_sms ? tiles : dev.num_sms;
  return launch_pdl(kernel, dim3(grid), dim3(GemmShape<BN, BMODE>::kThreads), L::kAlloc, stream,
                    "gemm launch", tmA, tmB, args);
}

// CTA pairs (gemm_sm100_kernel<..., PAIR = 2>): a cluster of two CTAs per
// 256 x BN tile, persistent over tiles. The grid holds as many pairs as can be
// resident at once (a GPC whose free SM count is odd leaves one SM out), so
// every pair starts in the first wave.
template <int BN, int STAGES, int BMODE, int OUT>
hxb_status_t launch_gemm_pair(const DeviceInfo& dev, const CUtensorMap& tmA,
                              const CUtensorMap& tmB, const GemmArgs& args,
                              cudaStream_t stream) {
  using L = GemmSmem<BN / 2, STAGES, BMODE>;
  auto kernel = gemm_sm100_kernel<BN, STAGES, BMODE, OUT, 2>;
  static int max_pairs[64] = {};
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(GemmShape<BN, BMODE>::kThreads);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!max_pairs[dev.ordinal]) {
    cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm pair)");
    cfg.gridDim = dim3(2 * (dev.num_sms / 2));
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
    if (e != cudaSuccess) return cuda_status(e, "cudaOccupancyMaxActiveClusters(gemm pair)");
    if (n < 1) return fail(HXB_STATUS_UNSUPPORTED, "gemm pair: no CTA pair fits an SM pair");
    max_pairs[dev.ordinal] = n;
  }
  const int tiles = args.tiles_m * args.tiles_n;
  const int pairs = tiles < max_pairs[dev.ordinal] ? tiles : max_pairs[dev.ordinal];
  cfg.gridDim = dim3(2 * pairs);
  cfg.numAttrs = 2;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, tmA, tmB, args), "gemm pair launch");
}

// One cluster of SPLIT CTAs per output tile (gemm_splitk_sm100.cuh),
// launched with programmatic stream serialization like the persistent kernel.
template <int BN, int STAGES, int BMODE, int OUT, int SPLIT>
hxb_status_t launch_splitk(const DeviceInfo& dev, const CUtensorMap& tmA, const CUtensorMap& tmB,
                           const GemmArgs& args, cudaStream_t stream) {
  using L = SplitSmem<BN, STAGES>;
  auto kernel = gemm_splitk_sm100_kernel<BN, STAGES, BMODE, OUT, SPLIT>;
  static bool configured[64] = {};
  if (!configured[dev.ordinal]) {
    cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm split-k)");
    configured[dev.ordinal] = true;
  }
  const int tiles = args.tiles_m * args.tiles_n;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(SPLIT, tiles);
  cfg.blockDim = dim3(GemmShape<BN, BMODE>::kThreads);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = SPLIT;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, tmA, tmB, args), "gemm split-k launch");
}

template <int BMODE, int OUT, int SPLIT>
hxb_status_t launch_split_bn(const GemmPlan& plan, const DeviceInfo& dev, const CUtensorMap& tmA,
                             const CUtensorMap& tmB, const GemmArgs& args, cudaStream_t stream) {
  switch (plan.block_n) {
    case 256: return launch_splitk<256, 4, BMODE, OUT, SPLIT>(dev, tmA, tmB, args, stream);
    case 128: return launch_splitk<128, 6, BMODE, OUT, SPLIT>(dev, tmA, tmB, args, stream);
    case 64: return launch_splitk<64, 8, BMODE, OUT, SPLIT>(dev, tmA, tmB, args, stream);
    default: break;
  }
  return fail(HXB_STATUS_UNSUPPORTED, "no split-k kernel for block_n=%d", plan.block_n);
}

template <int BMODE, int OUT>
hxb_status_t launch_planned(const GemmPlan& plan, const DeviceInfo& dev,
                            const CUtensorMap& tmA, const CUtensorMap& tmB,
                            const GemmArgs& args, cudaStream_t stream) {
  if (plan.pair == 2) {
    if (plan.split != 1)
      return fail(HXB_STATUS_UNSUPPORTED, "no CTA-pair kernel with split_k=%d", plan.split);
    switch (plan.block_n) {
      case 512: return launch_gemm_pair<512, 4, BMODE, OUT>(dev, tmA, tmB, args, stream);
      case 256: return launch_gemm_pair<256, 6, BMODE, OUT>(dev, tmA, tmB, args, stream);
      case 128: return launch_gemm_pair<128, 8, BMODE, OUT>(dev, tmA, tmB, args, stream);
      default: break;
    }
    return fail(HXB_STATUS_UNSUPPORTED, "no CTA-pair kernel for block_n=%d", plan.block_n);
  }
  switch (plan.split) {
    case 1: break;
    case 2: return launch_split_bn<BMODE, OUT, 2>(plan, dev, tmA, tmB, args, stream);
    case 4: return launch_split_bn<BMODE, OUT, 4>(plan, dev, tmA, tmB, args, stream);
    case 8: return launch_split_bn<BMODE, OUT, 8>(plan, dev, tmA, tmB, args, stream);
    default:
      return fail(HXB_STATUS_UNSUPPORTED, "no kernel for split_k=%d", plan.split);
  }
  // Stage counts fill ~192-208 KB of shared memory per CTA.
  switch (plan.block_n) {
    case 256: return launch_gemm<256, 4, BMODE, OUT>(dev, tmA, tmB, args, stream);
    case 128: return launch_gemm<128, 6, BMODE, OUT>(dev, tmA, tmB, args, stream);
    case 64: return launch_gemm<64, 8, BMODE, OUT>(dev, tmA, tmB, args, stream);
    default: break;
  }
  return fail(HXB_STATUS_UNSUPPORTED, "no kernel for block_n=%d", plan.block_n);
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// Bytes of re-pitched copy needed for an operand of `rows` x `cols` f16
// elements whose pitch or base is not TMA-compatible (0 if it is).
size_t repitch_bytes(const void* p, int64_t ld, int64_t rows, int64_t cols) {
  if (aligned16(p) && (ld * 2) % 16 == 0) return 0;
  return (size_t)(rows * round_up(cols, 8) * 2 + 256);
}

hxb_status_t make_a_map(CUtensorMap* m, const void* A, int64_t lda, int64_t M,
                        int64_t K) {
  const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
  const uint64_t strides[1] = {(uint64_t)lda * 2};
  const uint32_t box[2] = {64, 128};
  return encode_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, dims,
                           strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

hxb_status_t gemm_f16_launch(const void* A, int64_t lda, const void* B, int64_t ldb,
                             int transpose_b, const void* C_init, void* C, int64_t ldc,
                             hxb_dtype_t c_dtype, int64_t M, int64_t N, int64_t K,
                             void* workspace, size_t workspace_bytes, void* const* replicas,
                             int nreplicas, cudaStream_t stream, const GemmPlan* forced = nullptr) {
  if (M < 1 || N < 1 || K < 1)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul: M, N, K must be >= 1 (got %lld, %lld, %lld)",
                (long long)M, (long long)N, (long long)K);
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul: dimensions exceed 2^31-1");
  if (!A || !B || !C) return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul: null operand");
  if (lda < K) return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul: lda < K");
  if (ldb < (transpose_b ? K : N)) return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul: ldb too small");
  if (ldc < N) return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul: ldc < N");
  if (c_dtype != HXB_DTYPE_F16 && c_dtype != HXB_DTYPE_F32)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul: C dtype must be f16 or f32");

  DeviceInfo* dev = nullptr;
  hxb_status_t s = current_device(&dev);
  if (s != HXB_OK) return s;

  // Operands whose pitch breaks the 16-byte TMA stride rule are re-pitched
  // into the workspace (the B200 counterpart of HMX's pack into padded tiles,
  // hmx.c:60-92): a 2-D copy to an 8-element-aligned pitch. The tensor map
  // keeps the true extent, so TMA zero-fills beyond it.
  const int64_t b_rows = transpose_b ? N : K, b_cols = transpose_b ? K : N;
  const size_t need_a = repitch_bytes(A, lda, M, K);
  const size_t need_b = repitch_bytes(B, ldb, b_rows, b_cols);
  if (need_a + need_b > 0) {
    if (!workspace || workspace_bytes < need_a + need_b)
      return fail(HXB_STATUS_INVALID_ARGUMENT,
                  "matmul: operands need %zu bytes of workspace for re-pitching, got %zu",
                  need_a + need_b, workspace_bytes);
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (ws) ws = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  if (need_a) {
    const int64_t p = round_up(K, 8);
    cudaError_t e = cudaMemcpy2DAsync(ws, p * 2, A, lda * 2, K * 2, M,
                                      cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return cuda_status(e, "re-pitch A");
    A = ws;
    lda = p;
    ws += round_up(M * p * 2, 256);
  }
  if (need_b) {
    const int64_t p = round_up(b_cols, 8);
    cudaError_t e = cudaMemcpy2DAsync(ws, p * 2, B, ldb * 2, b_cols * 2, b_rows,
                                      cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return cuda_status(e, "re-pitch B");
    B = ws;
    ldb = p;
  }

  const int bmode = transpose_b ? kBF16RowMajorNK : kBF16RowMajorKN;
  GemmPlan plan = forced ? *forced : plan_gemm((int)M, (int)N, (int)K, bmode, dev->num_sms);
  // The all-gather epilogue lives in the persistent kernels only, and runs on
  // one CTA per tile: with peer stores in the epilogue the CTA-pair form
  // measured slower on B200 (cfg 5 split over 2 GPUs: 4.04-4.08 ms fused
  // against 3.85 ms one-CTA, while the pair is faster without peers). Both
  // forms give the same bits.
  if (nreplicas > 0) {
    plan.split = 1;
    plan.pair = 1;
    if (plan.block_n > 256) plan.block_n = 256;
  }
  if ((plan.pair != 1 && (plan.pair != 2 || plan.split != 1 || plan.block_n < 128)) ||
      (plan.block_n > 256 && plan.pair != 2))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "matmul: a CTA pair (256-row tiles) needs block_n 128, 256 or 512 and no split_k; "
                "block_n 512 only on a pair");
  if (plan.split > 1 && (plan.split > 8 || (plan.split & (plan.split - 1)) ||
                         (K + kBK - 1) / kBK < plan.split))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "matmul: split_k %d needs a power of two <= 8 and at least that many "
                "64-deep K-blocks",
                plan.split);
  const int64_t tile_rows = (int64_t)kBM * plan.pair;
  const int64_t tiles_m = (M + tile_rows - 1) / tile_rows;
  if (plan.group_m < 1) plan.group_m = 1;
  if (plan.group_m > tiles_m) plan.group_m = (int)tiles_m;

  CUtensorMap tmA, tmB;
  if ((s = make_a_map(&tmA, A, lda, M, K)) != HXB_OK) return s;
  if (transpose_b) {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)ldb * 2};
    // a CTA of a pair loads half of the tile's B rows
    // one box per MMA chunk (at most 256 columns) and CTA
    const uint32_t box[2] = {64, (uint32_t)((plan.block_n > 256 ? 256 : plan.block_n) /
                                            plan.pair)};
    s = encode_tensor_map(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, dims,
                          strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t strides[1] = {(uint64_t)ldb * 2};
    const uint32_t box[2] = {64, 64};
    s = encode_tensor_map(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, dims,
                          strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (s != HXB_OK) return s;

  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.C = C;
  args.ldc = ldc;
  args.C_init = C_init;
  args.scale = nullptr;
  args.status = dev->status_word;
  args.tiles_m = (int)tiles_m;
  args.tiles_n = (int)((N + plan.block_n - 1) / plan.block_n);
  args.group_m = plan.group_m;
  const int esz = c_dtype == HXB_DTYPE_F16 ? 2 : 4;
  args.vec_ok = aligned16(C) && (ldc * esz) % 16 == 0 &&
                (!C_init || aligned16(C_init));
  args.ndests = nreplicas > 0 ? nreplicas + 1 : 0;
  args.dests[0] = C;
  for (int i = 0; i < nreplicas; ++i) {
    args.dests[i + 1] = const_cast<void*>(replicas[i]);
    args.vec_ok = args.vec_ok && aligned16(replicas[i]);
  }

  if (c_dtype == HXB_DTYPE_F16) {
    return transpose_b
               ? launch_planned<kBF16RowMajorNK, kOutF16>(plan, *dev, tmA, tmB, args, stream)
               : launch_planned<kBF16RowMajorKN, kOutF16>(plan, *dev, tmA, tmB, args, stream);
  }
  return transpose_b
             ? launch_planned<kBF16RowMajorNK, kOutF32>(plan, *dev, tmA, tmB, args, stream)
             : launch_planned<kBF16RowMajorKN, kOutF32>(plan, *dev, tmA, tmB, args, stream);
}

// M <= 16: the bandwidth-bound GEMV (gemv_w8_sm100.cuh).
template <int MROWS>
hxb_status_t launch_gemv(const DeviceInfo& dev, const GemvArgs& p, cudaStream_t stream) {
  auto kernel = gemv_w8_kernel<MROWS>;
  static bool configured[64] = {};
  if (!configured[dev.ordinal]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         GemvSmem::kBytes);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemv_w8)");
    configured[dev.ordinal] = true;
  }
  const unsigned grid = (unsigned)((p.N + kGemvBN - 1) / kGemvBN);
  kernel<<<grid, kGemvThreads, GemvSmem::kBytes, stream>>>(p);
  return cuda_status(cudaGetLastError(), "gemv_w8 launch");
}

hxb_status_t gemm_f16_impl(const void* A, int64_t lda, const void* B,
                           int64_t ldb, int transpose_b, const void* C_init,
                           void* C, int64_t ldc, hxb_dtype_t c_dtype, int64_t M,
                           int64_t N, int64_t K, void* workspace,
                           size_t workspace_bytes, cudaStream_t stream) {
  return gemm_f16_launch(A, lda, B, ldb, transpose_b, C_init, C, ldc, c_dtype, M, N, K,
                         workspace, workspace_bytes, nullptr, 0, stream);
}

namespace {

// [G, M, n] -> [M, G*n] (column block g of the destination = source block g),
// 16-byte vectors; the layout step after an NCCL all-gather of column shards.
__global__ void gather_column_blocks_kernel(const uint4* __restrict__ src, __half* __restrict__ dst,
                                            long long M, int n, int G, long long ldd) {
  const long long vec_per_row = n / 8;
  const long long total = (long long)G * M * vec_per_row;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long v = i % vec_per_row;
    const long long gm = i / vec_per_row;
    const long long m = gm % M;
    const int g = (int)(gm / M);
    *reinterpret_cast<uint4*>(dst + m * ldd + (long long)g * n + v * 8) = src[i];
  }
}

}  // namespace

hxb_status_t gemv_w8_impl(const void* A, int64_t lda, const void* W, int64_t ldw,
                          const void* scale, const void* R, void* C, int64_t ldc, int64_t M,
                          int64_t N, int64_t K, cudaStream_t stream) {
  DeviceInfo* dev = nullptr;
  hxb_status_t s = current_device(&dev);
  if (s != HXB_OK) return s;
  GemvArgs p{};
  p.X = static_cast<const __half*>(A);
  p.W = static_cast<const int8_t*>(W);
  p.scale = static_cast<const __half*>(scale);
  p.C = static_cast<__half*>(C);
  p.R = static_cast<const __half*>(R);
  p.ldx = lda;
  p.ldw = ldw;
  p.ldc = ldc;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  return M <= 8 ? launch_gemv<8>(*dev, p, stream) : launch_gemv<16>(*dev, p, stream);
}

// M <= 16 over every SM (gemv_w8_sk_sm100.cuh), with the stream-K workspace
// for the cross-SM partial sums. Returns HXB_STATUS_UNSUPPORTED (nothing
// launched) when the workspace is missing or too small.
hxb_status_t gemv_w8_sk_impl(const void* A, int64_t lda, const void* W, int64_t ldw,
                             const void* scale, const void* R, void* C, int64_t ldc, int64_t M,
                             int64_t N, int64_t K, void* ws, size_t ws_bytes,
                             cudaStream_t stream) {
  DeviceInfo* dev = nullptr;
  hxb_status_t s = current_device(&dev);
  if (s != HXB_OK) return s;
  const int64_t strips = (N + kGsBN - 1) / kGsBN, kc = (K + kGsBK - 1) / kGsBK;
  const int64_t tiles = strips * kc;
  const int ctas = (int)(tiles < dev->num_sms ? tiles : dev->num_sms);
  if (!ws || !aligned16(ws) || tiles > INT32_MAX / 1024 || ctas > (int)(kW8FlagBytes / 4) ||
      ws_bytes < kW8FlagBytes + (size_t)ctas * kGsPartialFloats * sizeof(float))
    return HXB_STATUS_UNSUPPORTED;
  CUtensorMap tmW, tmX;
  {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t strides[1] = {(uint64_t)ldw};
    const uint32_t box[2] = {128, kGsBK};
    if ((s = encode_tensor_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, W, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B)) != HXB_OK)
      return s;
  }
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)lda * 2};
    const uint32_t box[2] = {kGsBK, 16};
    if ((s = encode_tensor_map(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B)) != HXB_OK)
      return s;
  }
  GsArgs g{};
  g.scale = static_cast<const __half*>(scale);
  g.C = static_cast<__half*>(C);
  g.R = static_cast<const __half*>(R);
  g.ldc = ldc;
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.kc = (int)kc;
  g.tiles = (int)tiles;
  g.ctas = ctas;
  g.flags = static_cast<int*>(ws);
  g.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kW8FlagBytes);
  g.status = dev->status_word;
  auto kernel = M <= 8 ? gemv_w8_sk_kernel<1> : gemv_w8_sk_kernel<2>;
  static bool configured[2][64] = {};
  bool& done = configured[M <= 8 ? 0 : 1][dev->ordinal];
  if (!done) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         GsSmem::kAlloc);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemv_w8_sk)");
    done = true;
  }
  return launch_pdl(kernel, dim3(ctas), dim3(kGsThreads), GsSmem::kAlloc, stream,
                    "gemv_w8_sk launch", tmW, tmX, g);
}

// Largest dynamic shared memory (bytes) and threads per CTA of the f16 GEMM
// and the int8-weight matmul kernels (the executable library's export
// attributes).
size_t gemm_f16_max_smem_bytes() {
  size_t m = GemmSmem<256, 4, kBF16RowMajorKN>::kAlloc;
  if (GemmSmem<128, 6, kBF16RowMajorKN>::kAlloc > m) m = GemmSmem<128, 6, kBF16RowMajorKN>::kAlloc;
  if (GemmSmem<64, 8, kBF16RowMajorKN>::kAlloc > m) m = GemmSmem<64, 8, kBF16RowMajorKN>::kAlloc;
  return m;
}
int gemm_f16_threads() { return GemmShape<256, kBF16RowMajorKN>::kThreads; }
size_t w8_max_smem_bytes() {
  size_t m = W8Smem::kAlloc;
  if ((size_t)GemvSmem::kBytes > m) m = GemvSmem::kBytes;
  if ((size_t)GsSmem::kAlloc > m) m = GsSmem::kAlloc;
  return m;
}
int w8_threads() { return kW8Threads; }

// Stream-K workspace of the int8-weight GEMM for `ctas` CTAs: flags, then one
// f32 partial accumulator per CTA.
size_t w8_streamk_workspace_bytes(int ctas) {
  return kW8FlagBytes + (size_t)ctas * kW8PartialFloats * sizeof(float);
}
int w8_streamk_flag_ints() { return (int)(kW8FlagBytes / sizeof(int)); }

// Cost of the stream-K fix-up in K-blocks of one CTA's main loop: a
// contributor's partial write holds the single accumulator (~3 us), the
// finaliser adds the partials it waited for (~4 us for two) and the shares
// walk tiles in an order that shares less L2 between the CTAs running at
// once, which costs more the more tiles a share spans. Fitted on B200 against
// the data-parallel schedule (us, data-parallel / stream-K): 512 x 4096 x
// 4096 33.1 / 28.6, 512 x 11008 x 4096 76.0 / 49.1, 512 x 4096 x 12288
// 62.4 / 52.4, 512 x 4096 x 22016 91.7 / 93.7, 1024 x 4096 x 4096
// 32.4 / 37.3, 4096 x 4096 x 11008 313.6 / 333.9 (M x K x N).
constexpr long long kW8StreamKFixupKb = 28;
constexpr long long kW8StreamKFixupWaveKb = 8;
// The same for stream-K over the last partial wave only: its short shares
// cut each tile into about three pieces, so a finaliser adds two or three
// partials (fitted on B200, us, data-parallel / all stream-K / tail stream-K:
// 512 x 4096 x 22016 89.8 / 92.7 / 87.0, 512 x 4096 x 12288 61.2 / 51.8 /
// 55.8, 4096 x 4096 x 11008 308.8 / 323.2 / 308.7).
constexpr long long kW8StreamKTailFixupKb = 40;

// Schedule of the W8 GEMM for `tiles` output tiles of `num_kb` K-blocks on
// `units` CTAs that run at once, chosen by the estimated K-blocks of the
// busiest CTA: data-parallel (whole tiles, `waves` rounds), stream-K over all
// tiles (even shares plus the fix-up), or whole-tile waves followed by
// stream-K over the last partial wave only.
struct W8Plan {
  int grid = 0;      // CTAs to launch
  int streamk = 0;   // 1: stream-K over the tiles from dp_tiles on
  int dp_tiles = 0;  // tiles dealt whole before the stream-K part
};

W8Plan w8_plan(int tiles, long long num_kb, int units) {
  W8Plan plan;
  plan.grid = tiles < units ? tiles : units;
  const long long total = (long long)tiles * num_kb;
  const int waves = (tiles + units - 1) / units;
  const double fill = (double)tiles / ((double)waves * units);
  long long best = (long long)waves * num_kb;
  // stream-K over all tiles: fewer tiles than units (spread them over more
  // units), or several waves evened out over all units
  const long long g = total / kW8MinShare < units ? total / kW8MinShare : units;
  if (fill < 0.92 && (g > tiles || (tiles > units && g == units)) && g > 0) {
    const long long cost =
        (total + g - 1) / g + kW8StreamKFixupKb + kW8StreamKFixupWaveKb * (waves - 1);
    if (cost < best) {
      best = cost;
      plan.grid = (int)g;
      plan.streamk = 1;
      plan.dp_tiles = 0;
    }
  }
  // whole-tile waves, then the last partial wave split over all units
  if (waves >= 2) {
    const int dp_tiles = (waves - 1) * units;
    const long long tail = (long long)(tiles - dp_tiles) * num_kb;
    if (tail >= (long long)units * kW8MinShare) {
      const long long cost =
          (long long)(waves - 1) * num_kb + (tail + units - 1) / units + kW8StreamKTailFixupKb;
      if (cost < best) {
        best = cost;
        plan.grid = units;
        plan.streamk = 1;
        plan.dp_tiles = dp_tiles;
      }
    }
  }
  return plan;
}

hxb_status_t gemm_w8_impl(const void* A, int64_t lda, const void* W,
                          int64_t ldw, const void* scale, const void* R, void* C, int64_t ldc,
                          int64_t M, int64_t N, int64_t K, void* sk_ws, size_t sk_ws_bytes,
                          cudaStream_t stream, void* const* replicas = nullptr,
                          int nreplicas = 0) {
  DeviceInfo* dev = nullptr;
  hxb_status_t s = current_device(&dev);
  if (s != HXB_OK) return s;
  CUtensorMap tmA, tmW;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)lda * 2};
    const uint32_t box[2] = {64, (uint32_t)kW8BM};
    if ((s = encode_tensor_map(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B)) != HXB_OK)
      return s;
  }
  {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t strides[1] = {(uint64_t)ldw};
    const uint32_t box[2] = {(uint32_t)kW8BN, 64};
    if ((s = encode_tensor_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, W, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B)) != HXB_OK)
      return s;
  }
  CUtensorMap tmC;
  {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)ldc * 2};
    const uint32_t box[2] = {64, (uint32_t)kW8BM};
    if ((s = encode_tensor_map(&tmC, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, C, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B)) != HXB_OK)
      return s;
  }
  // The residual (same shape and leading dimension as C, 16-byte aligned like
  // it) comes in by TMA into the output staging tile.
  CUtensorMap tmR = tmC;
  if (R) {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)ldc * 2};
    const uint32_t box[2] = {64, (uint32_t)kW8BM};
    if ((s = encode_tensor_map(&tmR, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, R, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B)) != HXB_OK)
      return s;
  }
  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.C = C;
  args.ldc = ldc;
  args.C_init = R;
  args.scale = static_cast<const __half*>(scale);
  args.status = dev->status_word;
  args.tiles_m = (int)((M + kW8BM - 1) / kW8BM);
  args.tiles_n = (int)((N + kW8BN - 1) / kW8BN);
  // consecutive tiles sweep all m-tiles of one weight column block, so the
  // CTAs running at the same time share that int8 block in L2
  args.group_m = args.tiles_m;
  args.vec_ok = 0;
  // all-gather epilogue: the staged tiles also go to the other ranks' outputs
  args.ndests = nreplicas > 0 ? nreplicas + 1 : 0;
  args.dests[0] = C;
  for (int i = 0; i < nreplicas; ++i) args.dests[i + 1] = const_cast<void*>(replicas[i]);
  const int tiles = args.tiles_m * args.tiles_n;
  const int sms = dev->num_sms;
  int grid = tiles < sms ? tiles : sms;
  // Stream-K (when the caller gave the workspace) if whole tiles would leave
  // SMs idle in the last wave: every SM then gets the same share of K-blocks
  // of all tiles, or of the last partial wave's.
  if (sk_ws && sms <= kW8MaxStreamKCtas && sk_ws_bytes >= w8_streamk_workspace_bytes(sms)) {
    const W8Plan plan = w8_plan(tiles, (K + kBK - 1) / kBK, sms);
    if (plan.streamk) {
      grid = plan.grid;
      args.streamk = 1;
      args.sk_dp_tiles = plan.dp_tiles;
      args.sk_flags = static_cast<int*>(sk_ws);
      args.sk_partials =
          reinterpret_cast<float*>(static_cast<uint8_t*>(sk_ws) + kW8FlagBytes);
    }
  }
  static bool configured[64] = {};
  if (!configured[dev->ordinal]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_w8_sm100_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         W8Smem::kAlloc);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm_w8)");
    configured[dev->ordinal] = true;
  }
  gemm_w8_sm100_kernel<<<grid, kW8Threads, W8Smem::kAlloc, stream>>>(tmA, tmW, tmC, tmR, args);
  return cuda_status(cudaGetLastError(), "gemm_w8 launch");
}

}  // namespace hxb

extern "C" size_t hxb_matmul_f16_workspace_bytes(const void* A, int64_t lda,
                                                 const void* B, int64_t ldb,
                                                 int transpose_b, int64_t M,
                                                 int64_t N, int64_t K) {
  const int64_t b_rows = transpose_b ? N : K, b_cols = transpose_b ? K : N;
  return hxb::repitch_bytes(A, lda, M, K) + hxb::repitch_bytes(B, ldb, b_rows, b_cols);
}

extern "C" hxb_status_t hxb_matmul_f16(const void* A, int64_t lda, const void* B,
                                       int64_t ldb, int transpose_b,
                                       const void* C_init, void* C, int64_t ldc,
                                       hxb_dtype_t c_dtype, int64_t M, int64_t N,
                                       int64_t K, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  return hxb::gemm_f16_impl(A, lda, B, ldb, transpose_b, C_init, C, ldc, c_dtype,
                            M, N, K, workspace, workspace_bytes,
                            static_cast<cudaStream_t>(stream));
}

namespace hxb {
namespace {
// dests[d][r, c] = src[r, c] for r < M, c < N (f16, leading dimension ld,
// 8-column chunks): the all-gather step of the GEMV path, whose output is a
// few rows.
struct Dests {
  void* p[kMaxDests];
  int n;
};
__global__ void replicate_block_kernel(const __half* __restrict__ src, long long ld, int M,
                                       int N, Dests dests) {
  pdl_wait();
  const int chunks = N / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
       i < (long long)M * chunks; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / chunks, c = (i % chunks) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(src + r * ld + c);
    for (int d = 0; d < dests.n; ++d)
      *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(dests.p[d]) + r * ld + c) = v;
  }
  __threadfence_system();  // peer stores performed system-wide before the kernel ends
}
}  // namespace

hxb_status_t matmul_w8a16_impl(const void* A, int64_t lda, const void* W, int64_t ldw,
                               const void* scale, const void* R, void* C, int64_t ldc,
                               int64_t M, int64_t N, int64_t K, void* sk_ws,
                               size_t sk_ws_bytes, cudaStream_t stream,
                               void* const* replicas = nullptr, int nreplicas = 0) {
  if (M < 1 || N < 1 || K < 1)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_w8a16: M, N, K must be >= 1");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_w8a16: dimensions exceed 2^31-1");
  if (!A || !W || !scale || !C)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_w8a16: null operand");
  if (lda < K || ldw < N || ldc < N)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_w8a16: leading dimension too small");
  if (lda % 8 || ldw % 16 || ldc % 8 || !aligned16(A) || !aligned16(W) ||
      !aligned16(C) || !aligned16(scale) || (R && !aligned16(R)))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "matmul_w8a16: A/W/C/scale/R must be 16-byte aligned with lda%%8 == 0, "
                "ldw%%16 == 0, ldc%%8 == 0");
  if (M <= kGemvRows) {
    hxb_status_t s = HXB_STATUS_UNSUPPORTED;
    if (sk_ws)
      s = gemv_w8_sk_impl(A, lda, W, ldw, scale, R, C, ldc, M, N, K, sk_ws, sk_ws_bytes, stream);
    if (s == HXB_STATUS_UNSUPPORTED)
      s = gemv_w8_impl(A, lda, W, ldw, scale, R, C, ldc, M, N, K, stream);
    if (s != HXB_OK || nreplicas == 0) return s;
    // a few output rows: copy the block to the other ranks in one small
    // programmatically launched kernel after the GEMV
    Dests d{};
    d.n = nreplicas;
    for (int i = 0; i < nreplicas; ++i) d.p[i] = const_cast<void*>(replicas[i]);
    const long long work = M * (N / 8);
    const int blocks = (int)((work + 255) / 256);
    return launch_pdl(replicate_block_kernel, dim3(blocks), dim3(256), 0, stream,
                      "replicate launch", static_cast<const __half*>(C), (long long)ldc, (int)M,
                      (int)N, d);
  }
  if (sk_ws && !aligned16(sk_ws))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_w8a16: workspace must be 16-byte aligned");
  return gemm_w8_impl(A, lda, W, ldw, scale, R, C, ldc, M, N, K, sk_ws, sk_ws_bytes, stream,
                      replicas, nreplicas);
}
}  // namespace hxb

extern "C" hxb_status_t hxb_matmul_w8a16_allgather(const void* A, int64_t lda, const void* W,
                                                   int64_t ldw, const void* scale, void* C,
                                                   void* const* replicas, int nreplicas,
                                                   int64_t ldc, int64_t M, int64_t N, int64_t K,
                                                   void* workspace, size_t workspace_bytes,
                                                   void* stream) {
  using namespace hxb;
  if (nreplicas < 0 || nreplicas > kMaxDests - 1)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_w8a16_allgather: 0..%d replicas",
                kMaxDests - 1);
  if (nreplicas > 0 && !replicas)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_w8a16_allgather: null replica list");
  if (N % 8)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "matmul_w8a16_allgather: the shard width N (%lld) must be a multiple of 8",
                (long long)N);
  for (int i = 0; i < nreplicas; ++i)
    if (!replicas[i] || !aligned16(replicas[i]))
      return fail(HXB_STATUS_INVALID_ARGUMENT,
                  "matmul_w8a16_allgather: replica %d is null or not 16-byte aligned", i);
  return matmul_w8a16_impl(A, lda, W, ldw, scale, nullptr, C, ldc, M, N, K, workspace,
                           workspace_bytes, static_cast<cudaStream_t>(stream), replicas,
                           nreplicas);
}

extern "C" hxb_status_t hxb_matmul_w8a16(const void* A, int64_t lda, const void* W,
                                         int64_t ldw, const void* scale, void* C,
                                         int64_t ldc, int64_t M, int64_t N, int64_t K,
                                         void* stream) {
  return hxb::matmul_w8a16_impl(A, lda, W, ldw, scale, nullptr, C, ldc, M, N, K, nullptr, 0,
                                static_cast<cudaStream_t>(stream));
}

extern "C" hxb_status_t hxb_matmul_w8a16_residual(const void* A, int64_t lda, const void* W,
                                                  int64_t ldw, const void* scale, const void* R,
                                                  void* C, int64_t ldc, int64_t M, int64_t N,
                                                  int64_t K, void* stream) {
  if (!R) return hxb::fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_w8a16_residual: null residual");
  return hxb::matmul_w8a16_impl(A, lda, W, ldw, scale, R, C, ldc, M, N, K, nullptr, 0,
                                static_cast<cudaStream_t>(stream));
}

extern "C" hxb_status_t hxb_plan_matmul_w8a16(int64_t M, int64_t N, int64_t K, int num_sms,
                                             int* grid, int* dp_tiles, int32_t* pieces,
                                             int64_t cap, int64_t* count) {
  using namespace hxb;
  if (M <= kGemvRows || N < 1 || K < 1 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "plan_matmul_w8a16: M > %d, N, K >= 1 required",
                kGemvRows);
  if (num_sms < 1 || num_sms > kW8MaxStreamKCtas || !grid || !dp_tiles || (pieces && cap < 0))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "plan_matmul_w8a16: bad arguments");
  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.tiles_m = (int)((M + kW8BM - 1) / kW8BM);
  args.tiles_n = (int)((N + kW8BN - 1) / kW8BN);
  const int tiles = args.tiles_m * args.tiles_n;
  const W8Plan plan = w8_plan(tiles, (K + kBK - 1) / kBK, num_sms);
  args.streamk = plan.streamk;
  args.sk_dp_tiles = plan.dp_tiles;
  *grid = plan.grid;
  *dp_tiles = plan.streamk ? plan.dp_tiles : tiles;
  int64_t n = 0;
  for (int u = 0; u < plan.grid; ++u) {
    W8Work work;
    work.init(args, u, plan.grid);
    long long pos = work.first();
    W8Seg sg;
    while (work.next(pos, sg)) {
      int c_lo, c_hi;
      work.contributors(sg, &c_lo, &c_hi);
      if (pieces && n < cap) {
        int32_t* r = pieces + 5 * n;
        r[0] = u, r[1] = sg.tile, r[2] = sg.k0, r[3] = sg.k1, r[4] = c_hi - c_lo;
      }
      ++n;
    }
  }
  if (count) *count = n;
  return HXB_OK;
}

extern "C" size_t hxb_matmul_w8a16_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  (void)M;
  (void)N;
  (void)K;
  hxb::DeviceInfo* dev = nullptr;
  if (hxb::current_device(&dev) != HXB_OK) return 0;
  return hxb::w8_streamk_workspace_bytes(dev->num_sms);
}

extern "C" hxb_status_t hxb_matmul_w8a16_streamk(const void* A, int64_t lda, const void* W,
                                                 int64_t ldw, const void* scale, const void* R,
                                                 void* C, int64_t ldc, int64_t M, int64_t N,
                                                 int64_t K, void* workspace,
                                                 size_t workspace_bytes, void* stream) {
  if (!workspace)
    return hxb::fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_w8a16_streamk: null workspace");
  return hxb::matmul_w8a16_impl(A, lda, W, ldw, scale, R, C, ldc, M, N, K, workspace,
                                workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" hxb_status_t hxb_matmul_f16_allgather(const void* A, int64_t lda, const void* B,
                                                 int64_t ldb, int transpose_b, void* C,
                                                 void* const* replicas, int nreplicas,
                                                 int64_t ldc, int64_t M, int64_t N, int64_t K,
                                                 void* stream) {
  using namespace hxb;
  if (nreplicas < 0 || nreplicas > kMaxDests - 1)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_f16_allgather: 0..%d replicas",
                kMaxDests - 1);
  if (nreplicas > 0 && !replicas)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_f16_allgather: null replica list");
  for (int i = 0; i < nreplicas; ++i)
    if (!replicas[i])
      return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_f16_allgather: null replica %d", i);
  if (!aligned16(A) || !aligned16(B) || (lda * 2) % 16 || (ldb * 2) % 16)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "matmul_f16_allgather: A and B need 16-byte aligned rows (no re-pitching)");
  return gemm_f16_launch(A, lda, B, ldb, transpose_b, nullptr, C, ldc, HXB_DTYPE_F16, M, N, K,
                         nullptr, 0, replicas, nreplicas, static_cast<cudaStream_t>(stream));
}

extern "C" hxb_status_t hxb_gather_column_blocks_f16(const void* src, void* dst, int64_t G,
                                                     int64_t M, int64_t n, int64_t ldd,
                                                     void* stream) {
  using namespace hxb;
  if (!src || !dst || G < 1 || M < 1 || n < 8 || n % 8 || ldd < G * n || ldd % 8 ||
      !aligned16(src) || !aligned16(dst))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "gather_column_blocks: need n %% 8 == 0, ldd >= G*n, 16-byte alignment");
  DeviceInfo* dev = nullptr;
  hxb_status_t s = current_device(&dev);
  if (s != HXB_OK) return s;
  const unsigned grid = (unsigned)(dev->num_sms * 8);
  gather_column_blocks_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<__half*>(dst), M, (int)n, (int)G, ldd);
  return cuda_status(cudaGetLastError(), "gather_column_blocks launch");
}

extern "C" hxb_status_t hxb_matmul_f16_tiled(const void* A, int64_t lda, const void* B,
                                             int64_t ldb, int transpose_b, void* C, int64_t ldc,
                                             hxb_dtype_t c_dtype, int64_t M, int64_t N, int64_t K,
                                             int block_n, int group_m, int split_k,
                                             int cta_pair, void* stream) {
  using namespace hxb;
  if (block_n != 64 && block_n != 128 && block_n != 256 && !(block_n == 512 && cta_pair == 2))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "matmul_f16_tiled: block_n must be 64, 128 or 256 (512 on a CTA pair)");
  if (split_k != 1 && split_k != 2 && split_k != 4 && split_k != 8)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_f16_tiled: split_k must be 1, 2, 4 or 8");
  if (cta_pair != 1 && (cta_pair != 2 || split_k != 1 || block_n == 64))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "matmul_f16_tiled: cta_pair must be 1, or 2 with split_k 1 and block_n 128 or "
                "256");
  if (!aligned16(A) || !aligned16(B) || (lda * 2) % 16 || (ldb * 2) % 16)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "matmul_f16_tiled: A and B need 16-byte aligned rows (no re-pitching)");
  const GemmPlan plan{block_n, group_m, split_k, cta_pair};
  return gemm_f16_launch(A, lda, B, ldb, transpose_b, nullptr, C, ldc, c_dtype, M, N, K,
                         nullptr, 0, nullptr, 0, static_cast<cudaStream_t>(stream), &plan);
}

extern "C" hxb_status_t hxb_plan_matmul_f16(int64_t M, int64_t N, int64_t K, int transpose_b,
                                            int num_sms, int* block_n, int* group_m,
                                            int* split_k, int* cta_pair) {
  using namespace hxb;
  if (M < 1 || N < 1 || K < 1 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX ||
      num_sms < 1 || !block_n || !group_m)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "plan_matmul_f16: bad arguments");
  const GemmPlan p = plan_gemm((int)M, (int)N, (int)K,
                               transpose_b ? kBF16RowMajorNK : kBF16RowMajorKN, num_sms);
  *block_n = p.block_n;
  *group_m = p.group_m;
  if (split_k) *split_k = p.split;
  if (cta_pair) *cta_pair = p.pair;
  return HXB_OK;
}
