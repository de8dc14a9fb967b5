// The executable library of this dispatch library (include/hxb200_hal.h,
// part 1): a versioned query function and an export table of dispatch
// functions with the reference's dispatch signature
// (plugins/runtime/hexagon/dsp/rt/executable_library.h:163-177), each
// reading its operands from the binding pointers and its shape from the push
// constants and launching the whole dispatch on the environment's stream.
// Argument errors are returned as hxb_status_t values before anything is
// launched.
#include <math.h>
#include <string.h>

#include "hxb200_hal.h"
#include "runtime_common.h"

namespace hxb {

size_t gemm_f16_max_smem_bytes();
int gemm_f16_threads();
size_t w8_max_smem_bytes();
int w8_threads();
size_t attention_smem_bytes();
int attention_threads();

namespace {

// Leading bytes of the environment's scratch that hold the stream-K flags.
constexpr uint64_t kScratchFlagBytes = 4096;

// a * b (+ overflow check into *ok)
uint64_t mulc(uint64_t a, uint64_t b, bool* ok) {
  if (a != 0 && b > UINT64_MAX / a) {
    *ok = false;
    return 0;
  }
  return a * b;
}

// Binding i is present and at least `bytes` long.
hxb_status_t need(const hxb_executable_dispatch_state_t* ds, int i, uint64_t bytes,
                  const char* what) {
  if (!ds->binding_ptrs[i])
    return fail(HXB_STATUS_INVALID_ARGUMENT, "%s: binding %d is null", what, i);
  if (ds->binding_lengths && (uint64_t)ds->binding_lengths[i] < bytes)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "%s: binding %d holds %llu bytes, needs %llu",
                what, i, (unsigned long long)ds->binding_lengths[i],
                (unsigned long long)bytes);
  return HXB_OK;
}

hxb_status_t check_state(const hxb_executable_environment_t* env,
                         const hxb_executable_dispatch_state_t* ds, int min_bindings,
                         int max_bindings, const char* what) {
  if (!env || !ds || !ds->constants || !ds->binding_ptrs)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "%s: null environment or dispatch state", what);
  if (ds->binding_count < min_bindings || ds->binding_count > max_bindings)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "%s: %d bindings, expected %d..%d", what,
                (int)ds->binding_count, min_bindings, max_bindings);
  return HXB_OK;
}

float f32_bits(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// bindings: A, B, C [, C_init]; constants: M, N, K, flags
// [, block_n, group_m, split_k, cta_pair]
int dispatch_matmul_f16(const hxb_executable_environment_t* env,
                        const hxb_executable_dispatch_state_t* ds,
                        const hxb_executable_workgroup_state_t*) {
  hxb_status_t s = check_state(env, ds, 3, 4, "matmul_f16");
  if (s != HXB_OK) return s;
  const uint64_t M = ds->constants[0], N = ds->constants[1], K = ds->constants[2];
  const uint32_t flags = ds->constants[3];
  const int tb = (int)(flags & 1u);
  const bool f32 = (flags & 2u) != 0;
  bool ok = true;
  const uint64_t a_bytes = mulc(mulc(M, K, &ok), 2, &ok);
  const uint64_t b_bytes = mulc(mulc(K, N, &ok), 2, &ok);
  const uint64_t c_bytes = mulc(mulc(M, N, &ok), f32 ? 4 : 2, &ok);
  if (!ok) return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_f16: extents overflow");
  if ((s = need(ds, 0, a_bytes, "matmul_f16")) != HXB_OK ||
      (s = need(ds, 1, b_bytes, "matmul_f16")) != HXB_OK ||
      (s = need(ds, 2, c_bytes, "matmul_f16")) != HXB_OK)
    return s;
  const void* init = nullptr;
  if (ds->binding_count == 4) {
    if ((s = need(ds, 3, c_bytes, "matmul_f16")) != HXB_OK) return s;
    init = ds->binding_ptrs[3];
  }
  const void* A = ds->binding_ptrs[0];
  const void* B = ds->binding_ptrs[1];
  void* C = ds->binding_ptrs[2];
  const int64_t ldb = tb ? (int64_t)K : (int64_t)N;
  const hxb_dtype_t dt = f32 ? HXB_DTYPE_F32 : HXB_DTYPE_F16;
  // dense operands whose pitches TMA cannot take are re-pitched in the
  // library's built-in scratch (the dispatch has no transient binding)
  if (hxb_matmul_f16_workspace_bytes(A, (int64_t)K, B, ldb, tb, (int64_t)M, (int64_t)N,
                                     (int64_t)K) != 0)
    return hxb_matmul_f16_noalloc(A, (int64_t)K, B, ldb, tb, init, C, (int64_t)N, dt,
                                  (int64_t)M, (int64_t)N, (int64_t)K, env->stream);
  // a tile plan the compiler baked into the push constants (block_n,
  // group_m, split_k, cta_pair; block_n 0 = plan at dispatch time)
  const uint32_t block_n = ds->constants[4], group_m = ds->constants[5];
  const uint32_t split_k = ds->constants[6] ? ds->constants[6] : 1u;
  const uint32_t cta_pair = ds->constants[7] ? ds->constants[7] : 1u;
  if (block_n != 0 && !init)
    return hxb_matmul_f16_tiled(A, (int64_t)K, B, ldb, tb, C, (int64_t)N, dt, (int64_t)M,
                                (int64_t)N, (int64_t)K, (int)block_n, (int)group_m,
                                (int)split_k, (int)cta_pair, env->stream);
  return hxb_matmul_f16(A, (int64_t)K, B, ldb, tb, init, C, (int64_t)N, dt, (int64_t)M,
                        (int64_t)N, (int64_t)K, nullptr, 0, env->stream);
}

// bindings: A, W, scale, C [, residual]; constants: M, N, K
int dispatch_matmul_w8a16(const hxb_executable_environment_t* env,
                          const hxb_executable_dispatch_state_t* ds,
                          const hxb_executable_workgroup_state_t*) {
  hxb_status_t s = check_state(env, ds, 4, 5, "matmul_w8a16");
  if (s != HXB_OK) return s;
  const uint64_t M = ds->constants[0], N = ds->constants[1], K = ds->constants[2];
  bool ok = true;
  const uint64_t a_bytes = mulc(mulc(M, K, &ok), 2, &ok);
  const uint64_t w_bytes = mulc(K, N, &ok);
  const uint64_t c_bytes = mulc(mulc(M, N, &ok), 2, &ok);
  if (!ok) return fail(HXB_STATUS_INVALID_ARGUMENT, "matmul_w8a16: extents overflow");
  if ((s = need(ds, 0, a_bytes, "matmul_w8a16")) != HXB_OK ||
      (s = need(ds, 1, w_bytes, "matmul_w8a16")) != HXB_OK ||
      (s = need(ds, 2, 2 * N, "matmul_w8a16")) != HXB_OK ||
      (s = need(ds, 3, c_bytes, "matmul_w8a16")) != HXB_OK)
    return s;
  const void* R = nullptr;
  if (ds->binding_count == 5) {
    if ((s = need(ds, 4, c_bytes, "matmul_w8a16")) != HXB_OK) return s;
    R = ds->binding_ptrs[4];
  }
  void* const* p = ds->binding_ptrs;
  if (env->scratch)
    return hxb_matmul_w8a16_streamk(p[0], (int64_t)K, p[1], (int64_t)N, p[2], R, p[3],
                                    (int64_t)N, (int64_t)M, (int64_t)N, (int64_t)K,
                                    env->scratch, (size_t)env->scratch_bytes, env->stream);
  if (R)
    return hxb_matmul_w8a16_residual(p[0], (int64_t)K, p[1], (int64_t)N, p[2], R, p[3],
                                     (int64_t)N, (int64_t)M, (int64_t)N, (int64_t)K,
                                     env->stream);
  return hxb_matmul_w8a16(p[0], (int64_t)K, p[1], (int64_t)N, p[2], p[3], (int64_t)N,
                          (int64_t)M, (int64_t)N, (int64_t)K, env->stream);
}

// bindings: Q, K, V, O; constants: BH, Sq, Skv, D, causal, scale bits
int dispatch_attention_f16(const hxb_executable_environment_t* env,
                           const hxb_executable_dispatch_state_t* ds,
                           const hxb_executable_workgroup_state_t*) {
  hxb_status_t s = check_state(env, ds, 4, 4, "attention_f16");
  if (s != HXB_OK) return s;
  const uint64_t BH = ds->constants[0], Sq = ds->constants[1], Skv = ds->constants[2],
                 D = ds->constants[3];
  const int causal = ds->constants[4] != 0;
  float scale = f32_bits(ds->constants[5]);
  if (ds->constants[5] == 0u && D > 0) scale = 1.0f / sqrtf((float)D);
  bool ok = true;
  const uint64_t q_bytes = mulc(mulc(mulc(BH, Sq, &ok), D, &ok), 2, &ok);
  const uint64_t kv_bytes = mulc(mulc(mulc(BH, Skv, &ok), D, &ok), 2, &ok);
  if (!ok) return fail(HXB_STATUS_INVALID_ARGUMENT, "attention_f16: extents overflow");
  if ((s = need(ds, 0, q_bytes, "attention_f16")) != HXB_OK ||
      (s = need(ds, 1, kv_bytes, "attention_f16")) != HXB_OK ||
      (s = need(ds, 2, kv_bytes, "attention_f16")) != HXB_OK ||
      (s = need(ds, 3, q_bytes, "attention_f16")) != HXB_OK)
    return s;
  void* const* p = ds->binding_ptrs;
  return hxb_attention_f16(p[0], p[1], p[2], p[3], (int64_t)BH, (int64_t)Sq, (int64_t)Skv,
                           (int64_t)D, scale, causal, env->stream);
}

// bindings: Q, K cache, V cache, O; constants: batch, q_heads, kv_heads, q_len,
// q_pos0 (i32), kv_len, kv_rows, D, causal, out_layout, scale bits
int dispatch_attention_gqa_f16(const hxb_executable_environment_t* env,
                               const hxb_executable_dispatch_state_t* ds,
                               const hxb_executable_workgroup_state_t*) {
  hxb_status_t s = check_state(env, ds, 4, 4, "attention_gqa_f16");
  if (s != HXB_OK) return s;
  const uint32_t* c = ds->constants;
  const uint64_t B = c[0], Hq = c[1], Hkv = c[2], q_len = c[3], kv_len = c[5], kv_rows = c[6],
                 D = c[7];
  const int32_t q_pos0 = (int32_t)c[4];
  float scale = f32_bits(c[10]);
  if (c[10] == 0u && D > 0) scale = 1.0f / sqrtf((float)D);
  bool ok = true;
  const uint64_t q_bytes = mulc(mulc(mulc(mulc(B, Hq, &ok), q_len, &ok), D, &ok), 2, &ok);
  const uint64_t kv_bytes = mulc(mulc(mulc(mulc(B, Hkv, &ok), kv_rows, &ok), D, &ok), 2, &ok);
  if (!ok) return fail(HXB_STATUS_INVALID_ARGUMENT, "attention_gqa_f16: extents overflow");
  if ((s = need(ds, 0, q_bytes, "attention_gqa_f16")) != HXB_OK ||
      (s = need(ds, 1, kv_bytes, "attention_gqa_f16")) != HXB_OK ||
      (s = need(ds, 2, kv_bytes, "attention_gqa_f16")) != HXB_OK ||
      (s = need(ds, 3, q_bytes, "attention_gqa_f16")) != HXB_OK)
    return s;
  void* const* p = ds->binding_ptrs;
  // the key split's partials go to the device scratch past the stream-K
  // flags, which they must not touch
  char* ws = nullptr;
  size_t ws_bytes = 0;
  if (env->scratch && env->scratch_bytes > kScratchFlagBytes) {
    ws = static_cast<char*>(env->scratch) + kScratchFlagBytes;
    ws_bytes = env->scratch_bytes - kScratchFlagBytes;
  }
  return hxb_attention_gqa_f16(p[0], p[1], p[2], p[3], (int64_t)B, (int64_t)Hq, (int64_t)Hkv,
                               (int64_t)q_len, (int64_t)q_pos0, (int64_t)kv_len,
                               (int64_t)kv_rows, (int64_t)D, scale, c[8] != 0, (int)c[9], ws,
                               ws_bytes, env->stream);
}

// bindings: x, out, attn_norm, w_qkv, s_qkv, w_o, s_o, ffn_norm, w_gate_up,
// s_gate_up, w_down, s_down, workspace; constants: batch, seq, pos0, hidden,
// heads, head_dim, ffn, rms_eps bits, rope_theta bits
int dispatch_decoder_block_w8a16(const hxb_executable_environment_t* env,
                                 const hxb_executable_dispatch_state_t* ds,
                                 const hxb_executable_workgroup_state_t*) {
  hxb_status_t s = check_state(env, ds, 13, 13, "decoder_block_w8a16");
  if (s != HXB_OK) return s;
  const uint32_t* c = ds->constants;
  void* const* p = ds->binding_ptrs;
  hxb_decoder_w8_t w;
  w.hidden = c[3];
  w.heads = c[4];
  w.head_dim = c[5];
  w.ffn = c[6];
  w.rms_eps = f32_bits(c[7]);
  w.rope_theta = f32_bits(c[8]);
  w.attn_norm = p[2];
  w.w_qkv = p[3];
  w.s_qkv = p[4];
  w.w_o = p[5];
  w.s_o = p[6];
  w.ffn_norm = p[7];
  w.w_gate_up = p[8];
  w.s_gate_up = p[9];
  w.w_down = p[10];
  w.s_down = p[11];
  const uint64_t batch = c[0], seq = c[1], H = c[3], F = c[6];
  bool ok = true;
  const uint64_t act = mulc(mulc(mulc(batch, seq, &ok), H, &ok), 2, &ok);
  const uint64_t bytes[11] = {act,
                              act,
                              2 * H,
                              mulc(H, 3 * H, &ok),
                              6 * H,
                              mulc(H, H, &ok),
                              2 * H,
                              2 * H,
                              mulc(H, 2 * F, &ok),
                              4 * F,
                              mulc(F, H, &ok)};
  if (!ok) return fail(HXB_STATUS_INVALID_ARGUMENT, "decoder_block_w8a16: extents overflow");
  for (int i = 0; i < 11; ++i)
    if ((s = need(ds, i, bytes[i], "decoder_block_w8a16")) != HXB_OK) return s;
  if ((s = need(ds, 11, 2 * H, "decoder_block_w8a16")) != HXB_OK) return s;
  const size_t ws = hxb_decoder_block_workspace_bytes(&w, (int64_t)batch, (int64_t)seq);
  if (ws == 0) return fail(HXB_STATUS_INVALID_ARGUMENT, "decoder_block_w8a16: bad shape");
  if ((s = need(ds, 12, ws, "decoder_block_w8a16")) != HXB_OK) return s;
  const size_t ws_len = ds->binding_lengths ? ds->binding_lengths[12] : ws;
  return hxb_decoder_block_w8a16(&w, p[0], p[1], (int64_t)batch, (int64_t)seq, (int64_t)c[2],
                                 p[12], ws_len, env->stream);
}

const hxb_executable_library_header_t kHeader = {HXB_EXECUTABLE_LIBRARY_VERSION_1};

const hxb_executable_dispatch_fn_t kPtrs[HXB_EXPORT_COUNT] = {
    dispatch_matmul_f16, dispatch_matmul_w8a16, dispatch_attention_f16,
    dispatch_decoder_block_w8a16, dispatch_attention_gqa_f16};

const char* const kNames[HXB_EXPORT_COUNT] = {"matmul_f16", "matmul_w8a16", "attention_f16",
                                              "decoder_block_w8a16", "attention_gqa_f16"};

struct Library {
  const hxb_executable_library_header_t* header;
  hxb_executable_import_table_t imports;
  hxb_executable_export_table_t exports;
  hxb_executable_dispatch_attrs_t attrs[HXB_EXPORT_COUNT];
};

Library* library() {
  static Library lib = [] {
    Library l{};
    l.header = &kHeader;
    l.imports = {0, nullptr};
    const uint64_t tc = HXB_DISPATCH_FLAG_RESOURCES_VALID | HXB_DISPATCH_FLAG_USES_TENSOR_CORE |
                        HXB_DISPATCH_FLAG_USES_TMEM;
    const size_t w8 = w8_max_smem_bytes();
    const size_t att = attention_smem_bytes();
    l.attrs[HXB_EXPORT_MATMUL_F16] = {tc, gemm_f16_max_smem_bytes(),
                                      (uint64_t)gemm_f16_threads()};
    l.attrs[HXB_EXPORT_MATMUL_W8A16] = {tc, w8, (uint64_t)w8_threads()};
    l.attrs[HXB_EXPORT_ATTENTION_F16] = {tc, att, (uint64_t)attention_threads()};
    l.attrs[HXB_EXPORT_ATTENTION_GQA_F16] = {tc, att, (uint64_t)attention_threads()};
    l.attrs[HXB_EXPORT_DECODER_BLOCK_W8A16] = {
        tc, w8 > att ? w8 : att,
        (uint64_t)(w8_threads() > attention_threads() ? w8_threads() : attention_threads())};
    l.exports = {HXB_EXPORT_COUNT, kPtrs, l.attrs, kNames};
    return l;
  }();
  return &lib;
}

}  // namespace
}  // namespace hxb

static_assert(sizeof(hxb_executable_dispatch_attrs_t) == 24, "dispatch attrs layout");
static_assert(offsetof(hxb::Library, header) == offsetof(hxb_executable_library_t, header) &&
                  offsetof(hxb::Library, imports) == offsetof(hxb_executable_library_t, imports) &&
                  offsetof(hxb::Library, exports) == offsetof(hxb_executable_library_t, exports),
              "the library starts with the public hxb_executable_library_t layout");

extern "C" const hxb_executable_library_header_t** hxb_executable_library_query(
    hxb_executable_library_version_t max_version, const hxb_executable_environment_t*) {
  if (max_version != HXB_EXECUTABLE_LIBRARY_VERSION_LATEST) return nullptr;
  return const_cast<const hxb_executable_library_header_t**>(&hxb::library()->header);
}
