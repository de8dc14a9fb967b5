// Llama-style decoder block with int8-weight linears (BASELINE configuration
// 4) built from the dispatch kernels of this library:
//
//   h   = RMSNorm(x) * attn_norm                          rmsnorm_kernel
//   qkv = h . Wqkv * s_qkv                                W8 GEMM  [S, 3*hidden]
//   q,k = RoPE(q), RoPE(k)   (in place inside qkv)        rope_kernel
//        (with a KV cache: rope_cache_kernel, which also writes the new
//        rows' k and v into the caches)
//   att = causal softmax(q k^T / sqrt(d)) v               attention, [B,S,H*D]
//   h2  = att . Wo * s_o + x                              W8 GEMM + residual
//   g,u = RMSNorm(h2) * ffn_norm . Wgu * s_gu             rmsnorm + W8 GEMM
//   a   = silu(g) * u                                     swiglu_kernel
//   out = a . Wd * s_d + h2                               W8 GEMM + residual
//
// Attention reads q, k and v straight out of the fused QKV output (column
// blocks of one row-major matrix) and writes its output in [S, H*D] order,
// the input layout of the O projection, so no transposes are needed. The
// reference has no such block (its full models come from Hugging Face
// checkpoints, integration_tests/models/meta-llama/*); the arithmetic follows
// the Hugging Face Llama modules those tests wrap: RMSNorm in f32 over the
// row, rounded to f16 and multiplied by the f16 weight; RoPE with
// inv_freq[i] = theta^(-2i/d) over the rotate-half pairs (i, i + d/2);
// silu(g) * u. Intermediates are f16 as in an f16 model.
#include <math.h>
#include <string.h>

#include "runtime_common.h"
#include "sm100.cuh"

namespace hxb {

hxb_status_t matmul_w8a16_impl(const void* A, int64_t lda, const void* W, int64_t ldw,
                               const void* scale, const void* R, void* C, int64_t ldc,
                               int64_t M, int64_t N, int64_t K, void* sk_ws,
                               size_t sk_ws_bytes, cudaStream_t stream,
                               void* const* replicas = nullptr, int nreplicas = 0);
size_t w8_streamk_workspace_bytes(int ctas);
int w8_streamk_flag_ints();
hxb_status_t attention_launch(const void* Q, int64_t ldq, const void* K, int64_t ldk,
                              const void* V, int64_t ldv, void* O, int64_t ldo, int64_t B,
                              int64_t H, int64_t hpr, int64_t Sq, int64_t Skv, int64_t D,
                              float scale, int causal, cudaStream_t stream);
hxb_status_t attention_cached_launch(const void* Q, int64_t ldq, const void* k_cache,
                                     const void* v_cache, int64_t cache_rows, void* O,
                                     int64_t ldo, int64_t batch, int64_t heads, int64_t seq,
                                     int64_t kv_len, int64_t q_pos0, int64_t D, float scale,
                                     void* workspace, size_t workspace_bytes,
                                     cudaStream_t stream);
size_t attention_split_bound(int64_t Sq, int64_t D);

namespace {

// One warp per row; 16-byte vector loads (cols % 8 == 0).
// `clear` (optional, nclear ints) is zeroed by block 0: the decoder block's
// first kernel resets the stream-K flags its W8 GEMMs use.
__global__ void rmsnorm_kernel(const __half* __restrict__ x, long long ldx,
                               const __half* __restrict__ gamma, __half* __restrict__ y,
                               long long ldy, int rows, int cols, float eps, int* clear,
                               int nclear) {
  pdl_wait();
  pdl_trigger();
  if (clear && blockIdx.x == 0)
    for (int i = threadIdx.x; i < nclear; i += blockDim.x) clear[i] = 0;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const __half* xr = x + (long long)warp * ldx;
  __half* yr = y + (long long)warp * ldy;
  float ss = 0.0f;
  for (int c = lane * 8; c < cols; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)cols + eps);
  for (int c = lane * 8; c < cols; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const uint4 g = *reinterpret_cast<const uint4*>(gamma + c);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
    const __half2* gh = reinterpret_cast<const __half2*>(&g);
    uint4 o;
    __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      oh[e] = __hmul2(__floats2half2_rn(f.x * r, f.y * r), gh[e]);
    }
    *reinterpret_cast<uint4*>(yr + c) = o;
  }
}

// The same normalisation with one 256-thread block per row, the row held in
// registers (cols <= 8192, cols % 8 == 0): for up to 1024 rows (decode steps,
// prefills of a few hundred tokens), where one warp per row leaves too few
// warps per SM to hide its 16 dependent vector loads. Only the order of the
// sum of squares differs from rmsnorm_kernel.
constexpr int kNormBlockThreads = 256;
constexpr int kNormBlockVecs = 4;  // 16-byte vectors of x per thread
constexpr int kNormBlockMaxCols = kNormBlockThreads * kNormBlockVecs * 8;
__global__ void __launch_bounds__(kNormBlockThreads)
    rmsnorm_block_kernel(const __half* __restrict__ x, long long ldx,
                         const __half* __restrict__ gamma, __half* __restrict__ y,
                         long long ldy, int rows, int cols, float eps, int* clear, int nclear) {
  __shared__ float part[kNormBlockThreads / 32];
  pdl_wait();
  pdl_trigger();
  if (clear && blockIdx.x == 0)
    for (int i = threadIdx.x; i < nclear; i += blockDim.x) clear[i] = 0;
  const __half* xr = x + (long long)blockIdx.x * ldx;
  __half* yr = y + (long long)blockIdx.x * ldy;
  uint4 v[kNormBlockVecs];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormBlockVecs; ++i) {
    const int c = (i * kNormBlockThreads + threadIdx.x) * 8;
    v[i] = c < cols ? *reinterpret_cast<const uint4*>(xr + c) : make_uint4(0, 0, 0, 0);
    const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kNormBlockThreads / 32; ++w) tot += part[w];
  const float r = rsqrtf(tot / (float)cols + eps);
#pragma unroll
  for (int i = 0; i < kNormBlockVecs; ++i) {
    const int c = (i * kNormBlockThreads + threadIdx.x) * 8;
    if (c >= cols) break;
    const uint4 g = *reinterpret_cast<const uint4*>(gamma + c);
    const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
    const __half2* gh = reinterpret_cast<const __half2*>(&g);
    uint4 o;
    __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      oh[e] = __hmul2(__floats2half2_rn(f.x * r, f.y * r), gh[e]);
    }
    *reinterpret_cast<uint4*>(yr + c) = o;
  }
}

// In-place rotary embedding of `heads` consecutive 128-wide heads at the
// start of every row (the q and k blocks of a fused QKV row). One warp per
// (row, head); lane l handles the rotate-half pairs (2l, 2l + 64) and
// (2l + 1, 2l + 65). Row r has position pos0 + r % seq.
// Rotates one 128-wide head in place at position `pos` (lane l: the pairs
// (2l, 2l + 64) and (2l + 1, 2l + 65), read and written as f16 pairs);
// `out`, if given, receives a copy of the rotated head.
__device__ __forceinline__ void rope_head(__half* v, float pos, float log2_theta, int lane,
                                          __half* out) {
  // lane l: dimensions i = 2l, 2l + 1 and their partners i + 64, as f16 pairs
  const __half2 x1 = *reinterpret_cast<const __half2*>(v + 2 * lane);
  const __half2 x2 = *reinterpret_cast<const __half2*>(v + 64 + 2 * lane);
  const float2 a = __half22float2(x1), b = __half22float2(x2);
  float ra[2], rb[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = 2 * lane + k;
    const float inv_freq = exp2f(-(2.0f * (float)i / 128.0f) * log2_theta);
    float sn, cs;
    sincosf(pos * inv_freq, &sn, &cs);
    const float ai = k ? a.y : a.x, bi = k ? b.y : b.x;
    ra[k] = ai * cs - bi * sn;
    rb[k] = bi * cs + ai * sn;
  }
  const __half2 ya = __halves2half2(__float2half_rn(ra[0]), __float2half_rn(ra[1]));
  const __half2 yb = __halves2half2(__float2half_rn(rb[0]), __float2half_rn(rb[1]));
  *reinterpret_cast<__half2*>(v + 2 * lane) = ya;
  *reinterpret_cast<__half2*>(v + 64 + 2 * lane) = yb;
  if (out) {
    *reinterpret_cast<__half2*>(out + 2 * lane) = ya;
    *reinterpret_cast<__half2*>(out + 64 + 2 * lane) = yb;
  }
}

__global__ void rope_kernel(__half* __restrict__ x, long long ldx, int rows, int heads, int seq,
                            int pos0, float log2_theta) {
  pdl_wait();
  pdl_trigger();
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= rows * heads) return;
  const int row = wid / heads, head = wid - row * heads;
  rope_head(x + (long long)row * ldx + head * 128, (float)(pos0 + row % seq), log2_theta, lane,
            nullptr);
}

// RoPE of the q and k heads of fused QKV rows fused with the KV-cache update:
// one warp per (row, slot); slots [0, heads) rotate q in place, [heads,
// 2 heads) rotate k in place and copy it to k_cache, [2 heads, 3 heads) copy
// v to v_cache (row b * seq + t goes to cache row pos0 + t of batch b).
__global__ void rope_cache_kernel(__half* __restrict__ qkv, long long ld, int rows, int heads,
                                  int seq, int pos0, float log2_theta, __half* __restrict__ k_cache,
                                  __half* __restrict__ v_cache, long long cache_rows) {
  pdl_wait();
  pdl_trigger();
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (long long)rows * 3 * heads) return;
  const int row = (int)(wid / (3 * heads)), slot = (int)(wid - (long long)row * 3 * heads);
  const int b = row / seq, t = row - b * seq;
  __half* src = qkv + (long long)row * ld + slot * 128;
  const int h = slot % heads;
  const long long crow = (((long long)b * heads + h) * cache_rows + pos0 + t) * 128;
  if (slot < 2 * heads) {
    rope_head(src, (float)(pos0 + t), log2_theta, lane, slot < heads ? nullptr : k_cache + crow);
  } else {
    *reinterpret_cast<uint2*>(v_cache + crow + 4 * lane) =
        *reinterpret_cast<const uint2*>(src + 4 * lane);
  }
}

// a[r, j] = silu(gu[r, j]) * gu[r, F + j], 8 columns per thread (F % 8 == 0).
__global__ void swiglu_kernel(const __half* __restrict__ gu, long long ldgu, __half* __restrict__ a,
                              long long lda, int rows, int F) {
  pdl_wait();
  pdl_trigger();
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = F / 8;
  if (idx >= (long long)rows * per_row) return;
  const int r = (int)(idx / per_row), c = (int)(idx - (long long)r * per_row) * 8;
  const uint4 g = *reinterpret_cast<const uint4*>(gu + (long long)r * ldgu + c);
  const uint4 u = *reinterpret_cast<const uint4*>(gu + (long long)r * ldgu + F + c);
  const __half2* gh = reinterpret_cast<const __half2*>(&g);
  const __half2* uh = reinterpret_cast<const __half2*>(&u);
  uint4 o;
  __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 gf = __half22float2(gh[e]), uf = __half22float2(uh[e]);
    const float s0 = gf.x / (1.0f + expf(-gf.x)), s1 = gf.y / (1.0f + expf(-gf.y));
    oh[e] = __floats2half2_rn(s0 * uf.x, s1 * uf.y);
  }
  *reinterpret_cast<uint4*>(a + (long long)r * lda + c) = o;
}

// KV-cache update: cache[b, h, begin + t, :] = src[b * n + t, h*D : (h+1)*D]
// for the K (blockIdx.y 0) and V (1) blocks of a fused projection output;
// one thread per 8 halves, coalesced on both sides.
__global__ void kv_cache_write_kernel(const __half* __restrict__ k_src,
                                      const __half* __restrict__ v_src, long long ld_src,
                                      __half* __restrict__ k_cache, __half* __restrict__ v_cache,
                                      int n, int heads, int D, int begin, long long cache_rows,
                                      long long vectors) {
  pdl_wait();
  pdl_trigger();
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= vectors) return;
  const __half* src = blockIdx.y ? v_src : k_src;
  __half* cache = blockIdx.y ? v_cache : k_cache;
  const int per_row = heads * D / 8;
  const long long r = idx / per_row;  // source row b * n + t
  const int c = (int)(idx - r * per_row) * 8;
  const int h = c / D, d = c - h * D;
  const long long b = r / n, t = r - b * n;
  const uint4 v = *reinterpret_cast<const uint4*>(src + r * ld_src + c);
  *reinterpret_cast<uint4*>(cache + ((b * heads + h) * cache_rows + begin + t) * D + d) = v;
}

hxb_status_t launch_kv_cache_write(const void* k_src, const void* v_src, int64_t ld_src,
                                   void* k_cache, void* v_cache, int64_t batch, int64_t heads,
                                   int64_t n, int64_t begin, int64_t cache_rows, int64_t D,
                                   cudaStream_t stream) {
  const long long vectors = (long long)batch * n * heads * D / 8;
  const int threads = 256;
  const dim3 grid((unsigned)((vectors + threads - 1) / threads), 2);
  return launch_pdl(kv_cache_write_kernel, grid, dim3(threads), 0, stream,
                    "kv cache write launch", static_cast<const __half*>(k_src),
                    static_cast<const __half*>(v_src), (long long)ld_src,
                    static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), (int)n,
                    (int)heads, (int)D, (int)begin, (long long)cache_rows, vectors);
}

hxb_status_t check_kv_cache_write(const void* k_src, const void* v_src, int64_t ld_src,
                                  const void* k_cache, const void* v_cache, int64_t batch,
                                  int64_t heads, int64_t n, int64_t begin, int64_t cache_rows,
                                  int64_t D) {
  if (!k_src || !v_src || !k_cache || !v_cache)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "kv cache write: null pointer");
  if (!aligned16(k_src) || !aligned16(v_src) || !aligned16(k_cache) || !aligned16(v_cache) ||
      ld_src % 8 || D % 8 || D < 8)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "kv cache write: 16-byte aligned rows and head_dim %% 8 == 0 required");
  if (batch < 1 || heads < 1 || n < 1 || begin < 0 || ld_src < heads * D)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "kv cache write: bad extents");
  if (begin + n > cache_rows)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "kv cache write: rows [%lld, %lld) exceed the %lld cache rows", (long long)begin,
                (long long)(begin + n), (long long)cache_rows);
  if (batch * n * heads * D / 8 > ((int64_t)1 << 40) || n > INT32_MAX || begin > INT32_MAX ||
      heads * D > INT32_MAX)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "kv cache write: extent too large");
  return HXB_OK;
}

hxb_status_t launch_rmsnorm(const void* x, int64_t ldx, const void* gamma, void* y, int64_t ldy,
                            int64_t rows, int64_t cols, float eps, cudaStream_t stream,
                            int* clear = nullptr, int nclear = 0) {
  // a block per row while one warp per row would leave the SMs with too few
  // warps to hide the row's load latency
  if (rows <= 1024 && cols <= kNormBlockMaxCols)
    return launch_pdl(rmsnorm_block_kernel, dim3((unsigned)rows), dim3(kNormBlockThreads), 0,
                      stream, "rmsnorm launch", static_cast<const __half*>(x), (long long)ldx,
                      static_cast<const __half*>(gamma), static_cast<__half*>(y),
                      (long long)ldy, (int)rows, (int)cols, eps, clear, nclear);
  const int threads = 256;
  const long long blocks = (rows * 32 + threads - 1) / threads;
  return launch_pdl(rmsnorm_kernel, dim3((unsigned)blocks), dim3(threads), 0, stream,
                    "rmsnorm launch", static_cast<const __half*>(x), (long long)ldx,
                    static_cast<const __half*>(gamma), static_cast<__half*>(y), (long long)ldy,
                    (int)rows, (int)cols, eps, clear, nclear);
}

// The RoPE kernels move f16 pairs (lane l rotates dimensions 2l, 2l + 1), so
// every row base must be 4-byte aligned: an even leading dimension and a
// 4-byte aligned base pointer.
inline bool pair_aligned(const void* p, int64_t ld) {
  return (reinterpret_cast<uintptr_t>(p) & 3u) == 0 && (ld & 1) == 0;
}

hxb_status_t launch_rope(void* x, int64_t ldx, int64_t rows, int64_t heads, int64_t seq,
                         int64_t pos0, float theta, cudaStream_t stream) {
  if (!pair_aligned(x, ldx))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "rope: the base must be 4-byte aligned and ldx (%lld) even (f16-pair accesses)",
                (long long)ldx);
  const int threads = 256;
  const long long blocks = (rows * heads * 32 + threads - 1) / threads;
  return launch_pdl(rope_kernel, dim3((unsigned)blocks), dim3(threads), 0, stream, "rope launch",
                    static_cast<__half*>(x), (long long)ldx, (int)rows, (int)heads, (int)seq,
                    (int)pos0, log2f(theta));
}

hxb_status_t launch_rope_cache(void* qkv, int64_t ld, int64_t rows, int64_t heads, int64_t seq,
                               int64_t pos0, float theta, void* k_cache, void* v_cache,
                               int64_t cache_rows, cudaStream_t stream) {
  if (!pair_aligned(qkv, ld) || !pair_aligned(k_cache, 2) || !pair_aligned(v_cache, 2))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "rope + kv cache: bases must be 4-byte aligned and ld (%lld) even (f16-pair "
                "accesses)",
                (long long)ld);
  const int threads = 256;
  const long long blocks = (rows * 3 * heads * 32 + threads - 1) / threads;
  return launch_pdl(rope_cache_kernel, dim3((unsigned)blocks), dim3(threads), 0, stream,
                    "rope + kv cache launch", static_cast<__half*>(qkv), (long long)ld, (int)rows,
                    (int)heads, (int)seq, (int)pos0, log2f(theta), static_cast<__half*>(k_cache),
                    static_cast<__half*>(v_cache), (long long)cache_rows);
}

hxb_status_t launch_swiglu(const void* gu, int64_t ldgu, void* a, int64_t lda, int64_t rows,
                           int64_t F, cudaStream_t stream) {
  const int threads = 256;
  const long long blocks = (rows * (F / 8) + threads - 1) / threads;
  return launch_pdl(swiglu_kernel, dim3((unsigned)blocks), dim3(threads), 0, stream,
                    "swiglu launch", static_cast<const __half*>(gu), (long long)ldgu,
                    static_cast<__half*>(a), (long long)lda, (int)rows, (int)F);
}

size_t round256(size_t b) { return (b + 255) & ~size_t(255); }

struct DecoderBuffers {
  size_t sk, sk_bytes, att_ws, att_ws_bytes, h, qkv, att, h2, gu, a, total;
};

// Stream-K scratch of the W8 GEMMs (flags, then partial accumulators) first,
// then (with a KV cache) the key-split partials of the attention, then the
// activations.
DecoderBuffers decoder_layout(const hxb_decoder_w8_t* w, int64_t rows, int64_t seq = 0) {
  DecoderBuffers b{};
  size_t off = 0;
  DeviceInfo* dev = nullptr;
  b.sk_bytes = current_device(&dev) == HXB_OK ? w8_streamk_workspace_bytes(dev->num_sms) : 0;
  b.sk = off;  off += round256(b.sk_bytes);
  b.att_ws_bytes = seq > 0 ? attention_split_bound(seq, w->head_dim) : 0;
  b.att_ws = off; off += round256(b.att_ws_bytes);
  b.h = off;   off += round256((size_t)rows * w->hidden * 2);
  b.qkv = off; off += round256((size_t)rows * 3 * w->hidden * 2);
  b.att = off; off += round256((size_t)rows * w->hidden * 2);
  b.h2 = off;  off += round256((size_t)rows * w->hidden * 2);
  b.gu = off;  off += round256((size_t)rows * 2 * w->ffn * 2);
  b.a = off;   off += round256((size_t)rows * w->ffn * 2);
  b.total = off + 256;  // alignment slack
  return b;
}

hxb_status_t check_decoder(const hxb_decoder_w8_t* w, int64_t batch, int64_t seq) {
  if (!w) return fail(HXB_STATUS_INVALID_ARGUMENT, "decoder: null weights");
  if (w->head_dim != 128)
    return fail(HXB_STATUS_UNSUPPORTED, "decoder: head_dim must be 128");
  if (w->heads < 1 || w->hidden != w->heads * w->head_dim)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "decoder: hidden must equal heads * head_dim");
  if (w->ffn < 8 || w->ffn % 8)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "decoder: ffn must be a positive multiple of 8");
  if (batch < 1 || seq < 1 || batch * seq > INT32_MAX)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "decoder: bad batch / seq");
  if (!w->attn_norm || !w->w_qkv || !w->s_qkv || !w->w_o || !w->s_o || !w->ffn_norm ||
      !w->w_gate_up || !w->s_gate_up || !w->w_down || !w->s_down)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "decoder: null weight pointer");
  if (!(w->rope_theta > 1.0f) || !(w->rms_eps >= 0.0f))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "decoder: bad rope_theta / rms_eps");
  return HXB_OK;
}

}  // namespace
}  // namespace hxb

extern "C" hxb_status_t hxb_rmsnorm_f16(const void* x, int64_t ldx, const void* gamma, void* y,
                                        int64_t ldy, int64_t rows, int64_t cols, float eps,
                                        void* stream) {
  using namespace hxb;
  if (!x || !gamma || !y || rows < 1 || cols < 8 || cols % 8 || ldx % 8 || ldy % 8 ||
      ldx < cols || ldy < cols || !aligned16(x) || !aligned16(y) || !aligned16(gamma) ||
      rows > INT32_MAX / 32)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "rmsnorm: need cols %% 8 == 0, 16-byte aligned rows, ld >= cols");
  return launch_rmsnorm(x, ldx, gamma, y, ldy, rows, cols, eps, static_cast<cudaStream_t>(stream));
}

extern "C" hxb_status_t hxb_rope_f16(void* x, int64_t ldx, int64_t rows, int64_t heads,
                                     int64_t head_dim, int64_t seq, int64_t pos0, float theta,
                                     void* stream) {
  using namespace hxb;
  if (head_dim != 128) return fail(HXB_STATUS_UNSUPPORTED, "rope: head_dim must be 128");
  if (!x || rows < 1 || heads < 1 || seq < 1 || ldx < heads * 128 || !(theta > 1.0f) ||
      rows * heads > INT32_MAX / 32 || pos0 < 0 || pos0 + seq > (1 << 24))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "rope: bad arguments");
  return launch_rope(x, ldx, rows, heads, seq, pos0, theta, static_cast<cudaStream_t>(stream));
}

extern "C" hxb_status_t hxb_swiglu_f16(const void* gu, int64_t ldgu, void* a, int64_t lda,
                                       int64_t rows, int64_t ffn, void* stream) {
  using namespace hxb;
  if (!gu || !a || rows < 1 || ffn < 8 || ffn % 8 || ldgu % 8 || lda % 8 || ldgu < 2 * ffn ||
      lda < ffn || !aligned16(gu) || !aligned16(a))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "swiglu: need ffn %% 8 == 0, 16-byte aligned rows, ldgu >= 2*ffn");
  return launch_swiglu(gu, ldgu, a, lda, rows, ffn, static_cast<cudaStream_t>(stream));
}

namespace hxb {
namespace {

struct KvCache {
  void *k, *v;
  int64_t rows;
};

// The block's dispatch sequence; with `cache` the new K/V rows go into the
// cache at pos0 and attention reads keys [0, pos0 + seq) from it.
hxb_status_t decoder_run(const hxb_decoder_w8_t* w, const void* x, void* out, int64_t batch,
                         int64_t seq, int64_t pos0, const KvCache* cache, void* workspace,
                         size_t workspace_bytes, cudaStream_t stream) {
  hxb_status_t s = check_decoder(w, batch, seq);
  if (s != HXB_OK) return s;
  if (!x || !out || !aligned16(x) || !aligned16(out))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "decoder: x / out must be 16-byte aligned");
  if (pos0 < 0 || pos0 + seq > (1 << 24))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "decoder: positions out of range");
  const int64_t rows = batch * seq, H = w->hidden, F = w->ffn;
  const DecoderBuffers b = decoder_layout(w, rows, cache ? seq : 0);
  if (!workspace || workspace_bytes < b.total)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "decoder: workspace needs %zu bytes, got %zu",
                b.total, workspace_bytes);
  // the cache side of the K/V write (its sources are this block's own qkv rows,
  // aligned like x)
  if (cache && (s = check_kv_cache_write(x, x, 3 * H, cache->k, cache->v, batch, w->heads, seq,
                                         pos0, cache->rows, w->head_dim)) != HXB_OK)
    return s;
  uint8_t* ws = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  __half* h = reinterpret_cast<__half*>(ws + b.h);
  __half* qkv = reinterpret_cast<__half*>(ws + b.qkv);
  __half* att = reinterpret_cast<__half*>(ws + b.att);
  __half* h2 = reinterpret_cast<__half*>(ws + b.h2);
  __half* gu = reinterpret_cast<__half*>(ws + b.gu);
  __half* a = reinterpret_cast<__half*>(ws + b.a);

  void* sk = b.sk_bytes ? ws + b.sk : nullptr;
  const size_t skb = b.sk_bytes;
  const float scale = 1.0f / sqrtf((float)w->head_dim);

  if ((s = launch_rmsnorm(x, H, w->attn_norm, h, H, rows, H, w->rms_eps, stream,
                          static_cast<int*>(sk), sk ? w8_streamk_flag_ints() : 0)) != HXB_OK)
    return s;
  if ((s = matmul_w8a16_impl(h, H, w->w_qkv, 3 * H, w->s_qkv, nullptr, qkv, 3 * H, rows, 3 * H, H,
                             sk, skb, stream)) != HXB_OK)
    return s;
  if (cache) {
    // RoPE of q and k with the new rows' k and v written into the caches
    if ((s = launch_rope_cache(qkv, 3 * H, rows, w->heads, seq, pos0, w->rope_theta, cache->k,
                               cache->v, cache->rows, stream)) != HXB_OK)
      return s;
    if ((s = attention_cached_launch(qkv, 3 * H, cache->k, cache->v, cache->rows, att, H, batch,
                                     w->heads, seq, pos0 + seq, pos0, w->head_dim, scale,
                                     b.att_ws_bytes ? ws + b.att_ws : nullptr, b.att_ws_bytes,
                                     stream)) != HXB_OK)
      return s;
  } else {
    // q and k are the first 2 * heads heads of every qkv row
    if ((s = launch_rope(qkv, 3 * H, rows, 2 * w->heads, seq, pos0, w->rope_theta, stream)) !=
        HXB_OK)
      return s;
    if ((s = attention_launch(qkv, 3 * H, qkv + H, 3 * H, qkv + 2 * H, 3 * H, att, H, batch,
                              w->heads, w->heads, seq, seq, w->head_dim, scale, 1, stream)) !=
        HXB_OK)
      return s;
  }
  if ((s = matmul_w8a16_impl(att, H, w->w_o, H, w->s_o, x, h2, H, rows, H, H, sk, skb, stream)) !=
      HXB_OK)
    return s;
  if ((s = launch_rmsnorm(h2, H, w->ffn_norm, h, H, rows, H, w->rms_eps, stream)) != HXB_OK) return s;
  if ((s = matmul_w8a16_impl(h, H, w->w_gate_up, 2 * F, w->s_gate_up, nullptr, gu, 2 * F, rows,
                             2 * F, H, sk, skb, stream)) != HXB_OK)
    return s;
  if ((s = launch_swiglu(gu, 2 * F, a, F, rows, F, stream)) != HXB_OK) return s;
  return matmul_w8a16_impl(a, F, w->w_down, H, w->s_down, h2, out, H, rows, H, F, sk, skb, stream);
}

}  // namespace
}  // namespace hxb

extern "C" size_t hxb_decoder_block_workspace_bytes(const hxb_decoder_w8_t* w, int64_t batch,
                                                    int64_t seq) {
  if (hxb::check_decoder(w, batch, seq) != HXB_OK) return 0;
  return hxb::decoder_layout(w, batch * seq).total;
}

extern "C" hxb_status_t hxb_decoder_block_w8a16(const hxb_decoder_w8_t* w, const void* x,
                                                void* out, int64_t batch, int64_t seq,
                                                int64_t pos0, void* workspace,
                                                size_t workspace_bytes, void* stream) {
  return hxb::decoder_run(w, x, out, batch, seq, pos0, nullptr, workspace, workspace_bytes,
                          static_cast<cudaStream_t>(stream));
}

extern "C" size_t hxb_decoder_block_cached_workspace_bytes(const hxb_decoder_w8_t* w,
                                                           int64_t batch, int64_t seq) {
  if (hxb::check_decoder(w, batch, seq) != HXB_OK) return 0;
  return hxb::decoder_layout(w, batch * seq, seq).total;
}

extern "C" hxb_status_t hxb_decoder_block_w8a16_cached(const hxb_decoder_w8_t* w, const void* x,
                                                       void* out, int64_t batch, int64_t seq,
                                                       int64_t pos0, void* k_cache,
                                                       void* v_cache, int64_t cache_rows,
                                                       void* workspace, size_t workspace_bytes,
                                                       void* stream) {
  const hxb::KvCache c{k_cache, v_cache, cache_rows};
  return hxb::decoder_run(w, x, out, batch, seq, pos0, &c, workspace, workspace_bytes,
                          static_cast<cudaStream_t>(stream));
}

extern "C" hxb_status_t hxb_kv_cache_write_f16(const void* k_src, const void* v_src,
                                               int64_t ld_src, void* k_cache, void* v_cache,
                                               int64_t batch, int64_t kv_heads, int64_t n,
                                               int64_t begin, int64_t cache_rows,
                                               int64_t head_dim, void* stream) {
  using namespace hxb;
  hxb_status_t s = check_kv_cache_write(k_src, v_src, ld_src, k_cache, v_cache, batch, kv_heads,
                                        n, begin, cache_rows, head_dim);
  if (s != HXB_OK) return s;
  return launch_kv_cache_write(k_src, v_src, ld_src, k_cache, v_cache, batch, kv_heads, n, begin,
                               cache_rows, head_dim, static_cast<cudaStream_t>(stream));
}
