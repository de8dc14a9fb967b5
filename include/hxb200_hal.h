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
 *   constants: M, N, K, flags (bit 0: B transposed, bit 1: f32 output),
 *             optional block_n, group_m, split_k, cta_pair: a tile plan fixed at
 *             compile time (hxb_plan_matmul_f16; used when there is no C_init
 *             and no re-pitch; block_n 0 = plan at dispatch time)
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

/* ---- base types, shaped like IREE's (iree/base/string_view.h,
 * iree/base/allocator.h) so a driver written against the reference's
 * signatures maps 1:1. */

/* A non-owning string: `size` bytes at `data`, no terminator required. */
typedef struct hxb_string_view_t {
  const char* data;
  size_t size;
} hxb_string_view_t;

/* Host allocator: a control function and its state, as iree_allocator_t.
 * {NULL, NULL} is the C library's malloc / free. Every host object of the
 * HAL (driver, device, buffer, semaphore and command-buffer records) is
 * allocated and freed through the allocator given when it was created. */
typedef enum hxb_allocator_command_e {
  HXB_ALLOCATOR_COMMAND_MALLOC = 0,
  HXB_ALLOCATOR_COMMAND_CALLOC = 1,
  HXB_ALLOCATOR_COMMAND_REALLOC = 2,
  HXB_ALLOCATOR_COMMAND_FREE = 3,
} hxb_allocator_command_t;

typedef struct hxb_allocator_alloc_params_t {
  size_t byte_length;
} hxb_allocator_alloc_params_t;

/* MALLOC / CALLOC / REALLOC read `params` (hxb_allocator_alloc_params_t) and
 * store the block in *inout_ptr (REALLOC also reads the old block from it);
 * FREE releases *inout_ptr and ignores `params`. */
typedef hxb_status_t (*hxb_allocator_ctl_fn_t)(void* self, hxb_allocator_command_t command,
                                               const void* params, void** inout_ptr);

typedef struct hxb_allocator_t {
  void* self;
  hxb_allocator_ctl_fn_t ctl;
} hxb_allocator_t;

typedef struct hxb_hal_driver_s hxb_hal_driver_t;
typedef struct hxb_hal_device_s hxb_hal_device_t;
typedef struct hxb_hal_buffer_s hxb_hal_buffer_t;
typedef struct hxb_hal_semaphore_s hxb_hal_semaphore_t;
typedef struct hxb_hal_command_buffer_s hxb_hal_command_buffer_t;
typedef struct hxb_hal_driver_registry_s hxb_hal_driver_registry_t;

/* The CUDA device ordinal a device is created on: the B200 counterpart of the
 * reference's DSP domain id (iree_hal_hexagon_domain_id_t, api.h:31). */
typedef int hxb_hal_domain_id_t;

/* Default and largest bound on one device-side queue wait (see
 * hxb_hal_device_queue_execute). */
#define HXB_HAL_DEFAULT_QUEUE_WAIT_TIMEOUT_NS 10000000000ull /* 10 s */
#define HXB_HAL_MAX_QUEUE_WAIT_TIMEOUT_NS 60000000000ull     /* 60 s */

/* Device options (api.h:38-63): the size of the device's scratch arena
 * (stream-K partials of the int8-weight dispatches and the key-split partials
 * of GQA attention; 0 = the stream-K size, which also covers a decode step's
 * key split) and the bound on a queue submission's device-side wait for its
 * wait semaphore (0 = HXB_HAL_DEFAULT_QUEUE_WAIT_TIMEOUT_NS; at most
 * HXB_HAL_MAX_QUEUE_WAIT_TIMEOUT_NS). */
typedef struct hxb_hal_device_options_t {
  uint64_t scratch_bytes;
  uint64_t queue_wait_timeout_ns;
} hxb_hal_device_options_t;

typedef struct hxb_hal_driver_options_t {
  hxb_hal_device_options_t default_device_options;
} hxb_hal_driver_options_t;

/* Device creation parameters, the slot of iree_hal_device_create_params_t
 * (api.h:93-96). `flags` is reserved and must be 0; NULL means defaults. */
typedef struct hxb_hal_device_create_params_t {
  uint64_t flags;
} hxb_hal_device_create_params_t;

void hxb_hal_device_options_initialize(hxb_hal_device_options_t* out_options);
void hxb_hal_driver_options_initialize(hxb_hal_driver_options_t* out_options);

/* Creates a driver (iree_hal_hexagon_driver_create, api.h:108-111).
 * `identifier` names the driver (empty = "b200"); no GPU is touched.
 * Release with hxb_hal_driver_release. */
hxb_status_t hxb_hal_driver_create(hxb_string_view_t identifier,
                                   const hxb_hal_driver_options_t* options,
                                   hxb_allocator_t host_allocator,
                                   hxb_hal_driver_t** out_driver);
/* Number of CUDA devices the driver can create devices on (0 without a GPU). */
hxb_status_t hxb_hal_driver_query_device_count(hxb_hal_driver_t* driver, int32_t* out_count);

/* One device the driver can create (iree_hal_device_info_t): its id (the
 * CUDA ordinal), a path ("cuda:<ordinal>") and the device's name. */
typedef struct hxb_hal_device_info_t {
  uint64_t device_id;
  char path[32];
  char name[96];
} hxb_hal_device_info_t;

/* Fills up to `capacity` infos (infos may be NULL with capacity 0) and
 * stores the number of devices in *out_count. */
hxb_status_t hxb_hal_driver_query_available_devices(hxb_hal_driver_t* driver,
                                                    hxb_hal_device_info_t* infos,
                                                    int32_t capacity, int32_t* out_count);
/* Creates the device `device_id` with the driver's default device options
 * (the driver vtable's create_device_by_id). */
hxb_status_t hxb_hal_driver_create_device_by_id(
    hxb_hal_driver_t* driver, uint64_t device_id,
    const hxb_hal_device_create_params_t* create_params, hxb_allocator_t host_allocator,
    hxb_hal_device_t** out_device);
void hxb_hal_driver_release(hxb_hal_driver_t* driver);

/* Creates a device on CUDA device `domain_id` (iree_hal_hexagon_device_create,
 * api.h:93-96) with its own queue stream and scratch arena. Resolves every
 * per-device address of the dispatch library here, before any command buffer
 * is captured. */
hxb_status_t hxb_hal_device_create(hxb_string_view_t identifier, hxb_hal_domain_id_t domain_id,
                                   const hxb_hal_device_options_t* options,
                                   const hxb_hal_device_create_params_t* create_params,
                                   hxb_allocator_t host_allocator,
                                   hxb_hal_device_t** out_device);
/* Waits for the queue (bounded: every device-side wait of the queue is) and
 * frees the device. */
void hxb_hal_device_release(hxb_hal_device_t* device);
/* The cudaStream_t of the device's queue. */
void* hxb_hal_device_queue_stream(hxb_hal_device_t* device);
/* Non-zero once a queue wait of this device ran out (the device is lost:
 * later submissions return HXB_STATUS_DEVICE_TIMEOUT). */
int hxb_hal_device_is_lost(hxb_hal_device_t* device);

/* ---- driver registry and module (registration/driver_module.c:65-120) */

typedef struct hxb_hal_driver_info_t {
  hxb_string_view_t driver_name;
  hxb_string_view_t full_name;
} hxb_hal_driver_info_t;

/* A driver factory (iree_hal_driver_factory_t): lists the drivers it provides
 * and creates one by name; try_create returns HXB_STATUS_UNAVAILABLE for a
 * name it does not provide. */
typedef struct hxb_hal_driver_factory_t {
  void* self;
  hxb_status_t (*enumerate)(void* self, size_t* out_driver_info_count,
                            const hxb_hal_driver_info_t** out_driver_infos);
  hxb_status_t (*try_create)(void* self, hxb_string_view_t driver_name,
                             hxb_allocator_t host_allocator, hxb_hal_driver_t** out_driver);
} hxb_hal_driver_factory_t;

/* A registry of factories (iree_hal_driver_registry_t). The factory structs
 * must outlive the registry. */
hxb_status_t hxb_hal_driver_registry_create(hxb_allocator_t host_allocator,
                                            hxb_hal_driver_registry_t** out_registry);
void hxb_hal_driver_registry_release(hxb_hal_driver_registry_t* registry);
/* HXB_STATUS_ALREADY_EXISTS if the factory is registered already. */
hxb_status_t hxb_hal_driver_registry_register_factory(hxb_hal_driver_registry_t* registry,
                                                      const hxb_hal_driver_factory_t* factory);
/* Driver infos of every registered factory, in registration order. */
hxb_status_t hxb_hal_driver_registry_enumerate(hxb_hal_driver_registry_t* registry,
                                               hxb_hal_driver_info_t* infos, int32_t capacity,
                                               int32_t* out_count);
/* Asks each factory in turn; HXB_STATUS_UNAVAILABLE if none provides it. */
hxb_status_t hxb_hal_driver_registry_try_create(hxb_hal_driver_registry_t* registry,
                                                hxb_string_view_t driver_name,
                                                hxb_allocator_t host_allocator,
                                                hxb_hal_driver_t** out_driver);

/* Registers the "b200" driver factory
 * (iree_hal_hexagon_driver_module_register, driver_module.c:108-120). Where
 * the reference reads IREE tool flags into the driver options, its
 * try_create reads the environment: HXB_HAL_SCRATCH_BYTES and
 * HXB_HAL_QUEUE_WAIT_TIMEOUT_MS (decimal; a malformed or out-of-range value
 * is HXB_STATUS_INVALID_ARGUMENT, as the reference rejects bad flags). */
hxb_status_t hxb_hal_driver_module_register(hxb_hal_driver_registry_t* registry);

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
 * waits for values with a bounded device-side poll and signals them with a
 * store (see hxb_hal_device_queue_execute); the host signals by storing and
 * waits by polling, bounded by `timeout_ns` (HXB_STATUS_DEVICE_TIMEOUT when it
 * runs out). */
hxb_status_t hxb_hal_semaphore_create(hxb_hal_device_t* device, uint64_t initial_value,
                                      hxb_hal_semaphore_t** out_semaphore);
hxb_status_t hxb_hal_semaphore_query(hxb_hal_semaphore_t* semaphore, uint64_t* out_value);
hxb_status_t hxb_hal_semaphore_signal(hxb_hal_semaphore_t* semaphore, uint64_t value);
hxb_status_t hxb_hal_semaphore_wait(hxb_hal_semaphore_t* semaphore, uint64_t value,
                                    uint64_t timeout_ns);
void hxb_hal_semaphore_release(hxb_hal_semaphore_t* semaphore);

/* A range bound to a dispatch (iree_hal_buffer_ref_t): a buffer of the
 * device, or -- when `buffer` is NULL -- slot `buffer_slot` of the binding
 * table given at submission, `offset` bytes into that binding. */
typedef struct hxb_hal_buffer_ref_t {
  hxb_hal_buffer_t* buffer;
  uint64_t offset;
  uint64_t length;
  uint32_t buffer_slot;
  uint32_t reserved;
} hxb_hal_buffer_ref_t;

/* One binding-table entry (iree_hal_buffer_binding_t) and the table
 * (iree_hal_buffer_binding_table_t), as submitted with a command buffer. */
typedef struct hxb_hal_buffer_binding_t {
  hxb_hal_buffer_t* buffer;
  uint64_t offset;
  uint64_t length;
} hxb_hal_buffer_binding_t;

typedef struct hxb_hal_buffer_binding_table_t {
  uint32_t count;
  const hxb_hal_buffer_binding_t* bindings;
} hxb_hal_buffer_binding_table_t;

/* Command buffers (command_buffer.c:586-726): begin, record dispatches of
 * this library's exports, end. A command buffer created with
 * binding_capacity > 0 may record bindings that name table slots
 * (< binding_capacity); it is then captured when it is first submitted with
 * a table, and re-captured into the same executable graph
 * (cudaGraphExecUpdate) when a later table binds other addresses. Without
 * table slots, end() checks every dispatch's arguments and captures the
 * recording as one CUDA graph; a command buffer may be executed any number
 * of times after that. */
hxb_status_t hxb_hal_command_buffer_create(hxb_hal_device_t* device, uint32_t binding_capacity,
                                           hxb_hal_command_buffer_t** out_command_buffer);
hxb_status_t hxb_hal_command_buffer_begin(hxb_hal_command_buffer_t* command_buffer);
hxb_status_t hxb_hal_command_buffer_dispatch(hxb_hal_command_buffer_t* command_buffer,
                                             uint32_t export_ordinal, const uint32_t* constants,
                                             uint32_t constant_count,
                                             const hxb_hal_buffer_ref_t* bindings,
                                             uint32_t binding_count);
hxb_status_t hxb_hal_command_buffer_end(hxb_hal_command_buffer_t* command_buffer);
void hxb_hal_command_buffer_release(hxb_hal_command_buffer_t* command_buffer);

/* ---- channels and collectives (channel.c:37-56, command_buffer.c:560-584
 * return IREE_STATUS_UNIMPLEMENTED in the reference) ------------------------
 * A channel is a group of `count` devices, one per process (or thread), that
 * run collectives together; it is an NCCL communicator over NVLink /
 * NVSwitch, loaded at run time (libnccl.so.2; the one the process already
 * holds, e.g. PyTorch's, else the system's). Collectives are recorded into
 * command buffers next to dispatches and captured into the same CUDA graph.
 * Every rank must record and submit the same collectives in the same order. */
typedef struct hxb_hal_channel_s hxb_hal_channel_t;

#define HXB_HAL_CHANNEL_ID_BYTES 128

/* A fresh channel id (rank 0 makes it and passes it to the other ranks out of
 * band). Host only, no GPU needed. */
hxb_status_t hxb_hal_channel_id_create(uint8_t* out_id);

/* Joins the channel `id` as `rank` of `count` on `device`. Every rank must
 * call it; the call returns once all have joined, or fails with
 * HXB_STATUS_DEVICE_TIMEOUT after `timeout_ns` (the half-made communicator
 * is aborted). */
hxb_status_t hxb_hal_channel_create(hxb_hal_device_t* device, const uint8_t* id, int32_t rank,
                                    int32_t count, uint64_t timeout_ns,
                                    hxb_hal_channel_t** out_channel);
int32_t hxb_hal_channel_rank(hxb_hal_channel_t* channel);
int32_t hxb_hal_channel_count(hxb_hal_channel_t* channel);
void hxb_hal_channel_release(hxb_hal_channel_t* channel);

typedef enum hxb_hal_collective_op_e {
  /* recv[r * n .. (r + 1) * n) = send of rank r (n = element_count) */
  HXB_HAL_COLLECTIVE_ALL_GATHER = 0,
  /* recv = sum over ranks of send (n elements) */
  HXB_HAL_COLLECTIVE_ALL_REDUCE_SUM = 1,
  /* recv (n elements) = rank r's block of the sum of the ranks' send
   * (count * n elements) */
  HXB_HAL_COLLECTIVE_REDUCE_SCATTER_SUM = 2,
  /* recv = send of rank 0 (n elements) */
  HXB_HAL_COLLECTIVE_BROADCAST = 3,
} hxb_hal_collective_op_t;

/* Records a collective of `element_count` elements of `element_type`
 * (HXB_DTYPE_F16, HXB_DTYPE_F32 or HXB_DTYPE_I8) from `send` into `recv`
 * (buffer ranges or binding-table slots, like dispatch bindings). */
hxb_status_t hxb_hal_command_buffer_collective(hxb_hal_command_buffer_t* command_buffer,
                                               hxb_hal_channel_t* channel,
                                               hxb_hal_collective_op_t op,
                                               hxb_dtype_t element_type,
                                               hxb_hal_buffer_ref_t send,
                                               hxb_hal_buffer_ref_t recv,
                                               uint64_t element_count);

/* Queue submission (device.c:1068-1112): after `wait_semaphore` reaches
 * `wait_value` (NULL: no wait), run `command_buffer` (NULL: none) with
 * `binding_table` (NULL: none; required when the command buffer records
 * table slots), then set `signal_semaphore` to `signal_value` (NULL: no
 * signal). Returns without waiting for the device.
 * The wait is a one-thread kernel on the queue that polls the semaphore for
 * at most the device's queue_wait_timeout_ns. When it runs out, the kernel
 * ORs HXB_DEVICE_STATUS_TIMEOUT into the device status word and marks the
 * device lost: this submission's command buffer still runs (its inputs may
 * not be ready, so its results are void), its signal is NOT written, so
 * waiters on it time out in turn, and later submissions to the device return
 * HXB_STATUS_DEVICE_TIMEOUT. Release waits on the queue therefore always
 * end. */
hxb_status_t hxb_hal_device_queue_execute(hxb_hal_device_t* device,
                                          hxb_hal_semaphore_t* wait_semaphore,
                                          uint64_t wait_value,
                                          hxb_hal_command_buffer_t* command_buffer,
                                          const hxb_hal_buffer_binding_table_t* binding_table,
                                          hxb_hal_semaphore_t* signal_semaphore,
                                          uint64_t signal_value);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* HXB200_HAL_H_ */
