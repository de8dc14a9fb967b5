/* hxb200_hal.h -- executable-library and HAL-runtime ABI of the B200
 * dispatch library: the same shapes the reference's runtime plugin uses, so a
 * driver or loader written against the reference finds them here.
 *
 * Part 1 mirrors the dispatch ABI between the reference's compiled
 * executables and its runtime (plugins/runtime/hexagon/dsp/rt/
 * executable_library.h:40-250): a versioned query function returning a
 * library with an export table of dispatch functions
 * `int fn(environment, dispatch_state, workgroup_state)` over binding
 * pointers and 32-bit push constants. On B200 a dispatch function is called
 * ONCE per dispatch and launches the whole CUDA grid on the environment's
 * stream; the workgroup state may be NULL and is not read.
 *
 * Part 2 mirrors the host HAL driver API (plugins/runtime/hexagon/api.h:
 * 55-114: driver and device options / create) and the pieces of the HAL a
 * driver exposes beneath it (device.c queue execute, command_buffer.c
 * dispatch recording, timeline semaphores). It is asynchronous where the
 * reference is synchronous (device.c:1068-1112): a command buffer is recorded
 * once, captured as a CUDA graph at end(), and each queue submission waits on
 * and signals timeline semaphores with stream memory operations, so the host
 * never blocks unless it waits on a semaphore.
 *
 * All functions return hxb_status_t (see hxb200.h) unless noted; the message
 * of the last error is hxb_last_error_message().
 */
#ifndef HXB200_HAL_H_
#define HXB200_HAL_H_

#include <stddef.h>
#include <stdint.h>

#include "hxb200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ===================================================== executable library */

/* 'HB' in the upper half, so the code cannot be confused with the reference's
 * 'HX' versions (executable_library.h:49-53). */
#define HXB_EXECUTABLE_LIBRARY_VERSION_1 0x48420001u
#define HXB_EXECUTABLE_LIBRARY_VERSION_LATEST HXB_EXECUTABLE_LIBRARY_VERSION_1
#define HXB_EXECUTABLE_LIBRARY_EXPORT_NAME "hxb_executable_library_query"

typedef uint32_t hxb_executable_library_version_t;

typedef struct hxb_executable_library_header_t {
  hxb_executable_library_version_t version;
} hxb_executable_library_header_t;

/* Environment shared by every dispatch of an executable
 * (executable_library.h:95-104). `stream` is the cudaStream_t the dispatch
 * launches on. `scratch` (may be NULL) is device memory the runtime owns for
 * the dispatches of one queue: with it the int8-weight exports use the
 * stream-K schedule (hxb_matmul_w8a16_streamk; its first 4096 bytes must be
 * zero when the runtime creates it) and the GQA attention export splits the
 * keys of short queries across SMs (its partials go past those 4096 bytes). */
typedef struct hxb_executable_environment_t {
  const uint32_t* constants;
  void* stream;
  void* scratch;
  uint64_t scratch_bytes;
} hxb_executable_environment_t;

/* Per-dispatch state (executable_library.h:106-133), same fields. On B200 the
 * workgroup size/count fields are informational (the grid is chosen by the
 * dispatch); `binding_lengths` are checked against the extents the constants
 * imply. */
typedef struct hxb_executable_dispatch_state_t {
  uint32_t workgroup_size_x;
  uint32_t workgroup_size_y;
  uint16_t workgroup_size_z;
  uint32_t workgroup_count_x;
  uint32_t workgroup_count_y;
  uint16_t workgroup_count_z;
  uint8_t binding_count;
  const uint32_t* constants;
  void* const* binding_ptrs;
  const size_t* binding_lengths;
  void* reserved;
} hxb_executable_dispatch_state_t;

/* Per-workgroup state (executable_library.h:135-160), same fields; not read
 * by the B200 dispatch functions (one call covers every workgroup). */
typedef struct hxb_executable_workgroup_state_t {
  uint32_t workgroup_id_x;
  uint32_t workgroup_id_y;
  uint16_t workgroup_id_z;
  uint16_t reserved;
  uint32_t processor_id;
  void* reserved_ptr;
} hxb_executable_workgroup_state_t;

/* Returns 0 on success, otherwise an hxb_status_t (executable_library.h:
 * 163-177: non-zero means the dispatch failed). */
typedef int (*hxb_executable_dispatch_fn_t)(
    const hxb_executable_environment_t* environment,
    const hxb_executable_dispatch_state_t* dispatch_state,
    const hxb_executable_workgroup_state_t* workgroup_state);

enum hxb_dispatch_flag_bits_e {
  HXB_DISPATCH_FLAG_NONE = 0,
  HXB_DISPATCH_FLAG_RESOURCES_VALID = 1u << 0, /* smem_bytes / threads are set */
  HXB_DISPATCH_FLAG_USES_TENSOR_CORE = 1u << 1,
  HXB_DISPATCH_FLAG_USES_TMEM = 1u << 2,
};

/* Resources of an export (executable_library.h:193-214: flags, VTCM bytes,
 * threads): here the largest dynamic shared memory a CTA of the dispatch
 * takes and its threads per CTA. 24 bytes, as in the reference. */
typedef struct hxb_executable_dispatch_attrs_t {
  uint64_t flags;
  uint64_t smem_bytes;
  uint64_t threads;
} hxb_executable_dispatch_attrs_t;

typedef struct hxb_executable_export_table_t {
  uint32_t count;
  const hxb_executable_dispatch_fn_t* ptrs;
  const hxb_executable_dispatch_attrs_t* attrs;
  const char* const* names;
} hxb_executable_export_table_t;

typedef struct hxb_executable_import_table_t {
  uint32_t count;
  const char* const* symbols;
} hxb_executable_import_table_t;

typedef struct hxb_executable_library_t {
  const hxb_executable_library_header_t* header;
  hxb_executable_import_table_t imports;
  hxb_executable_export_table_t exports;
} hxb_executable_library_t;

/* Returns the library (its header pointer; cast to hxb_executable_library_t)
 * or NULL if `max_version` is not the version the library was built with
 * (executable_library.h:61-72). `environment` is not read. */
const hxb_executable_library_header_t** hxb_executable_library_query(
    hxb_executable_library_version_t max_version,
    const hxb_executable_environment_t* environment);

/* Export ordinals and their bindings / push constants. All operands are
 * dense row-major; binding i must be at least the byte length given.
 *
 * HXB_EXPORT_MATMUL_F16 "matmul_f16"
 *   bindings: [0] A f16 [M,K], [1] B f16 [K,N] (or [N,K] if transposed),
 *             [2] C [M,N] (f16, or f32 with flag bit 1), optional [3] C_init
 *             (same type/shape as C, added to the product)
 *   constants: M, N, K, flags (bit 0: B transposed, bit 1: f32 output)
 * HXB_EXPORT_MATMUL_W8A16 "matmul_w8a16"
 *   bindings: [0] A f16 [M,K], [1] W int8 [K,N], [2] scale f16 [N],
 *             [3] C f16 [M,N], optional [4] residual f16 [M,N]
 *   constants: M, N, K
 * HXB_EXPORT_ATTENTION_F16 "attention_f16"
 *   bindings: [0] Q [BH,Sq,D], [1] K [BH,Skv,D], [2] V [BH,Skv,D],
 *             [3] O [BH,Sq,D], all f16
 *   constants: BH, Sq, Skv, D, causal, scale as f32 bits (0 = 1/sqrt(D))
 * HXB_EXPORT_DECODER_BLOCK_W8A16 "decoder_block_w8a16"
 *   bindings: [0] x f16 [B*S,hidden], [1] out f16 [B*S,hidden],
 *             [2] attn_norm, [3] w_qkv, [4] s_qkv, [5] w_o, [6] s_o,
 *             [7] ffn_norm, [8] w_gate_up, [9] s_gate_up, [10] w_down,
 *             [11] s_down, [12] workspace
 *             (hxb_decoder_block_workspace_bytes)
 *   constants: batch, seq, pos0, hidden, heads, head_dim, ffn,
 *              rms_eps as f32 bits, rope_theta as f32 bits
 * HXB_EXPORT_ATTENTION_GQA_F16 "attention_gqa_f16"
 *   bindings: [0] Q [B,Hq,q_len,D], [1] K cache [B,Hkv,kv_rows,D],
 *             [2] V cache [B,Hkv,kv_rows,D], [3] O ([B,Hq,q_len,D] or
 *             [B,q_len,Hq,D] by out_layout), all f16
 *   constants: batch, q_heads, kv_heads, q_len, q_pos0 (i32), kv_len,
 *              kv_rows, D, causal, out_layout (HXB_ATTN_OUT_*), scale as
 *              f32 bits (0 = 1/sqrt(D)); the arguments of
 *              hxb_attention_gqa_f16 in its order */
enum hxb_export_ordinal_e {
  HXB_EXPORT_MATMUL_F16 = 0,
  HXB_EXPORT_MATMUL_W8A16 = 1,
  HXB_EXPORT_ATTENTION_F16 = 2,
  HXB_EXPORT_DECODER_BLOCK_W8A16 = 3,
  HXB_EXPORT_ATTENTION_GQA_F16 = 4,
  HXB_EXPORT_COUNT = 5,
};

/* ===================================================== HAL runtime */

typedef struct hxb_hal_driver_s hxb_hal_driver_t;
typedef struct hxb_hal_device_s hxb_hal_device_t;
typedef struct hxb_hal_buffer_s hxb_hal_buffer_t;
typedef struct hxb_hal_semaphore_s hxb_hal_semaphore_t;
typedef struct hxb_hal_command_buffer_s hxb_hal_command_buffer_t;

/* Device options (api.h:40-63): which GPU, and the size of the device's
 * scratch arena (stream-K partials of the int8-weight dispatches and the
 * key-split partials of GQA attention; 0 = the stream-K size, which also
 * covers a decode step's key split). */
typedef struct hxb_hal_device_options_t {
  int32_t ordinal;
  uint64_t scratch_bytes;
} hxb_hal_device_options_t;

typedef struct hxb_hal_driver_options_t {
  hxb_hal_device_options_t default_device_options;
} hxb_hal_driver_options_t;

void hxb_hal_device_options_initialize(hxb_hal_device_options_t* out_options);
void hxb_hal_driver_options_initialize(hxb_hal_driver_options_t* out_options);

/* Creates a driver (api.h:98-111). `identifier` names the driver ("b200");
 * no GPU is touched. */
hxb_status_t hxb_hal_driver_create(const char* identifier,
                                   const hxb_hal_driver_options_t* options,
                                   hxb_hal_driver_t** out_driver);
/* Number of CUDA devices the driver can create devices on (0 without a GPU). */
hxb_status_t hxb_hal_driver_query_device_count(hxb_hal_driver_t* driver, int32_t* out_count);
void hxb_hal_driver_release(hxb_hal_driver_t* driver);

/* Creates a device on `options->ordinal` (or the driver's default options)
 * with its own queue stream and scratch arena (api.h:67-76). */
hxb_status_t hxb_hal_device_create(hxb_hal_driver_t* driver, const char* identifier,
                                   const hxb_hal_device_options_t* options,
                                   hxb_hal_device_t** out_device);
void hxb_hal_device_release(hxb_hal_device_t* device);
/* The cudaStream_t of the device's queue. */
void* hxb_hal_device_queue_stream(hxb_hal_device_t* device);

/* Device-local buffers. write/read are ordered on the device queue and
 * return when the copy is complete. */
hxb_status_t hxb_hal_buffer_allocate(hxb_hal_device_t* device, uint64_t byte_length,
                                     hxb_hal_buffer_t** out_buffer);
void* hxb_hal_buffer_device_pointer(hxb_hal_buffer_t* buffer);
uint64_t hxb_hal_buffer_byte_length(hxb_hal_buffer_t* buffer);
hxb_status_t hxb_hal_buffer_write(hxb_hal_buffer_t* buffer, uint64_t offset, const void* host,
                                  uint64_t byte_length);
hxb_status_t hxb_hal_buffer_read(hxb_hal_buffer_t* buffer, uint64_t offset, void* host,
                                 uint64_t byte_length);
void hxb_hal_buffer_release(hxb_hal_buffer_t* buffer);

/* Timeline semaphores: a 64-bit value that only grows. The device queue
 * waits for and signals values with stream memory operations; the host
 * signals by storing and waits by polling, bounded by `timeout_ns`
 * (HXB_STATUS_DEVICE_TIMEOUT when it runs out). */
hxb_status_t hxb_hal_semaphore_create(hxb_hal_device_t* device, uint64_t initial_value,
                                      hxb_hal_semaphore_t** out_semaphore);
hxb_status_t hxb_hal_semaphore_query(hxb_hal_semaphore_t* semaphore, uint64_t* out_value);
hxb_status_t hxb_hal_semaphore_signal(hxb_hal_semaphore_t* semaphore, uint64_t value);
hxb_status_t hxb_hal_semaphore_wait(hxb_hal_semaphore_t* semaphore, uint64_t value,
                                    uint64_t timeout_ns);
void hxb_hal_semaphore_release(hxb_hal_semaphore_t* semaphore);

/* A range of a buffer bound to a dispatch. */
typedef struct hxb_hal_buffer_ref_t {
  hxb_hal_buffer_t* buffer;
  uint64_t offset;
  uint64_t length;
} hxb_hal_buffer_ref_t;

/* Command buffers (command_buffer.c:586-726): begin, record dispatches of
 * this library's exports, end. end() checks every dispatch's arguments and
 * captures the recording as one CUDA graph; a command buffer may be executed
 * any number of times after that. */
hxb_status_t hxb_hal_command_buffer_create(hxb_hal_device_t* device,
                                           hxb_hal_command_buffer_t** out_command_buffer);
hxb_status_t hxb_hal_command_buffer_begin(hxb_hal_command_buffer_t* command_buffer);
hxb_status_t hxb_hal_command_buffer_dispatch(hxb_hal_command_buffer_t* command_buffer,
                                             uint32_t export_ordinal, const uint32_t* constants,
                                             uint32_t constant_count,
                                             const hxb_hal_buffer_ref_t* bindings,
                                             uint32_t binding_count);
hxb_status_t hxb_hal_command_buffer_end(hxb_hal_command_buffer_t* command_buffer);
void hxb_hal_command_buffer_release(hxb_hal_command_buffer_t* command_buffer);

/* Queue submission (device.c:1068-1112): after `wait_semaphore` reaches
 * `wait_value` (NULL: no wait), run `command_buffer`, then set
 * `signal_semaphore` to `signal_value` (NULL: no signal). Returns without
 * waiting for the device. */
hxb_status_t hxb_hal_device_queue_execute(hxb_hal_device_t* device,
                                          hxb_hal_semaphore_t* wait_semaphore,
                                          uint64_t wait_value,
                                          hxb_hal_command_buffer_t* command_buffer,
                                          hxb_hal_semaphore_t* signal_semaphore,
                                          uint64_t signal_value);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* HXB200_HAL_H_ */
