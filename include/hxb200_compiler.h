/* hxb200_compiler.h -- the compiler half of the B200 drop-in: a stand-in for
 * the IREE target plugin that turns linalg-on-tensors input into an
 * executable of B200 dispatches, and the runtime that loads and runs it.
 *
 * The reference's compiler plugin (plugins/compiler/hexagon) registers a
 * TargetBackend with IREE (PluginRegistration.cpp:9-12,
 * Target/HexagonTargetBackend.cpp:32-112) that forms dispatches, picks the
 * HMX strategy for eligible contractions
 * (CodeGen/Transforms/HexagonSpecializeHmxContractions.cpp:29-60,
 * CodeGen/Strategy/Planning/Strategies/ContractionStrategy.cpp:133-213),
 * searches VTCM tiles (VTCMPlanning.cpp:186-260) and serialises a
 * hal.executable.binary (Target/HexagonExecutableSerialization.cpp:622-635).
 * IREE itself is not available to this library, so the B200 target does the
 * same work on the textual MLIR the reference compiles
 * (examples/matmul/matmul.mlir, examples/attention_layer/attention_layer.mlir
 * and the int8-weight linalg.generic of BASELINE configuration 2):
 *
 *   1. parse the module's functions (func.func / util.func), their linalg,
 *      arith, tensor and hal.tensor ops;
 *   2. recognise each dispatch: a named or generic f16 contraction that the
 *      reference's HMX eligibility rules accept (one M, N and K dimension, at
 *      most one batch dimension, f16 inputs, f16 or f32 output, M before N in
 *      the output) -> the matmul export, its batch dimension tiled to one
 *      (one dispatch per batch); the int8-weight contraction with a
 *      per-output-channel scale and its f16 truncation -> the w8a16 export;
 *      the decomposed scaled-dot-product chain of attention_layer.mlir
 *      (extf, split scale on Q and K^T, batch_matmul, max, sub, exp, sum,
 *      div, fully-masked-row select, batch_matmul, truncf) -> the attention
 *      export. Anything else is a compile error naming the op and its line;
 *   3. choose the tile plan of every matmul dispatch at compile time (the
 *      offline sweep table, else the cost model) and bake it into the
 *      dispatch's push constants;
 *   4. serialise the executable: per function its argument and result
 *      tensors, the transient buffers between dispatches and the dispatch
 *      table (export ordinal, push constants, bindings).
 * The runtime part loads that executable onto a HAL device as one command
 * buffer per function whose bindings are binding-table slots (arguments,
 * results, transients), and invokes it with the caller's buffers.
 */
#ifndef HXB200_COMPILER_H_
#define HXB200_COMPILER_H_

#include <stddef.h>
#include <stdint.h>

#include "hxb200.h"
#include "hxb200_hal.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Format string and MIME type of the serialised executable (the
 * hal.executable.binary's format / mime_type). */
#define HXB_EXECUTABLE_FORMAT "cuda-sm100a-hxb-v1"
#define HXB_EXECUTABLE_MIME_TYPE "application/x-hxb200-dispatch-table"

typedef struct hxb_compiler_options_t {
  /* Dispatch kinds the target may form (non-zero = on); the reference's
   * --iree-hexagon-enable-hmx-matmul gate for contractions. */
  int32_t enable_matmul;
  int32_t enable_w8a16;
  int32_t enable_attention;
  /* SM count the tile plans are chosen for (0 = 148, a B200). */
  int32_t num_sms;
} hxb_compiler_options_t;

void hxb_compiler_options_initialize(hxb_compiler_options_t* out_options);

/* Compiles MLIR text (`length` bytes) into an executable. On success
 * *out_executable (size *out_size) holds the serialised executable; on any
 * status *out_log holds the compiler's decisions and diagnostics (one per
 * line: "accept", "reject" or "error" with the op and its source line), the
 * counterpart of the reference planner's decision trace. Both are allocated
 * by the library; free them with hxb_compiler_free. */
hxb_status_t hxb_compile_mlir(const char* text, size_t length,
                              const hxb_compiler_options_t* options,
                              void** out_executable, size_t* out_size,
                              char** out_log);
void hxb_compiler_free(void* p);

/* The executable wrapped as the MLIR the target's serializeExecutable
 * emits: `hal.executable.binary @<name> attributes {data = dense<[...]> :
 * vector<Nxi8>, format = HXB_EXECUTABLE_FORMAT, mime_type = ...}`.
 * Free with hxb_compiler_free. */
hxb_status_t hxb_executable_binary_mlir(const void* executable, size_t size,
                                        const char* symbol, char** out_text);

/* ---- loading and running a compiled executable ------------------------ */

/* Element types of argument / result tensors. */
typedef enum hxb_element_type_e {
  HXB_ELEMENT_F16 = 0,
  HXB_ELEMENT_F32 = 1,
  HXB_ELEMENT_I8 = 2,
} hxb_element_type_t;

#define HXB_MAX_RANK 8

typedef struct hxb_tensor_desc_t {
  int32_t element_type; /* hxb_element_type_t */
  int32_t rank;
  int64_t dims[HXB_MAX_RANK];
} hxb_tensor_desc_t;

typedef struct hxb_module_s hxb_module_t;

/* Loads an executable onto `device`: allocates the transient buffers of
 * every function and records each function as a command buffer over
 * binding-table slots. */
hxb_status_t hxb_module_load(hxb_hal_device_t* device, const void* executable,
                             size_t size, hxb_module_t** out_module);
void hxb_module_release(hxb_module_t* module);

/* Number of functions, and the name of function i (owned by the module). */
int32_t hxb_module_function_count(hxb_module_t* module);
const char* hxb_module_function_name(hxb_module_t* module, int32_t index);

/* Signature of the function `name`: *n_args / *n_results, and up to
 * `capacity` descriptors, the arguments first. */
hxb_status_t hxb_module_signature(hxb_module_t* module, const char* name,
                                  int32_t* n_args, int32_t* n_results,
                                  hxb_tensor_desc_t* descs, int32_t capacity);

/* Number of dispatches function `name` runs. */
int32_t hxb_module_dispatch_count(hxb_module_t* module, const char* name);

/* Runs function `name` on the module's device queue (the counterpart of
 * iree-run-module's invocation): `args` and `results` are device buffers
 * (each at least the bytes its descriptor implies), ordered after
 * `wait_semaphore` reaches `wait_value` and signalling `signal_semaphore`
 * with `signal_value` when done (either may be NULL). Returns without
 * waiting for the device. */
hxb_status_t hxb_module_invoke(hxb_module_t* module, const char* name,
                               const hxb_hal_buffer_binding_t* args, uint32_t n_args,
                               const hxb_hal_buffer_binding_t* results, uint32_t n_results,
                               hxb_hal_semaphore_t* wait_semaphore, uint64_t wait_value,
                               hxb_hal_semaphore_t* signal_semaphore, uint64_t signal_value);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* HXB200_COMPILER_H_ */
