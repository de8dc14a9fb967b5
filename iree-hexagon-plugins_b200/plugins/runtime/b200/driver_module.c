// IREE runtime driver module for the B200 target: the source a maintainer
// builds inside an IREE runtime checkout (it includes IREE's headers and is
// not compiled by this repository's build, which has no IREE). It mirrors
// plugins/runtime/hexagon/registration/driver_module.c:65-120 -- a driver
// factory with enumerate / try_create registered with IREE's driver
// registry, the driver options filled from tool flags -- and hands the work
// to the C ABI of include/hxb200_hal.h:
//
//   iree_hal_b200_driver_module_register   -> hxb_hal_driver_module_register
//                                             semantics (driver "b200")
//   factory try_create                     -> hxb_hal_driver_create
//   driver create_device_by_id             -> hxb_hal_driver_create_device_by_id
//   device queue_execute                   -> hxb_hal_device_queue_execute
//   executable (hal.executable.binary of format "cuda-sm100a-hxb-v1")
//                                          -> hxb_module_load
//   command-buffer dispatch of export i    -> the dispatch table of that
//                                             function, replayed through
//                                             hxb_hal_command_buffer_dispatch
//
// The IREE-side vtables (iree_hal_driver_vtable_t, iree_hal_device_vtable_t,
// ...) are thin: each wraps one hxb_hal_* object in an iree_hal_resource_t
// and converts hxb_status_t to iree_status_t with b200_status() below. Only
// the registration and driver creation are spelled out here; they are the
// part a tool (iree-run-module, iree-benchmark-module) reaches first.

#include <stdlib.h>

#include "hxb200_hal.h"
#include "iree/base/api.h"
#include "iree/base/tooling/flags.h"
#include "iree/hal/api.h"

IREE_FLAG(int64_t, b200_scratch_bytes, 0,
          "Bytes of the B200 device's scratch arena (stream-K partials, key-split\n"
          "partials). 0 selects the stream-K size.");
IREE_FLAG(int32_t, b200_queue_wait_timeout_ms, 10000,
          "Bound on one device-side queue wait for a semaphore, in ms (at most\n"
          "60000). A wait that runs out marks the device lost.");

// hxb_status_t -> iree_status_t, with the library's message.
static iree_status_t b200_status(hxb_status_t s) {
  if (s == HXB_OK) return iree_ok_status();
  iree_status_code_t code = IREE_STATUS_INTERNAL;
  switch (s) {
    case HXB_STATUS_INVALID_ARGUMENT: code = IREE_STATUS_INVALID_ARGUMENT; break;
    case HXB_STATUS_UNSUPPORTED: code = IREE_STATUS_UNIMPLEMENTED; break;
    case HXB_STATUS_RESOURCE_EXHAUSTED: code = IREE_STATUS_RESOURCE_EXHAUSTED; break;
    case HXB_STATUS_DEVICE_TIMEOUT: code = IREE_STATUS_DEADLINE_EXCEEDED; break;
    case HXB_STATUS_UNAVAILABLE: code = IREE_STATUS_UNAVAILABLE; break;
    case HXB_STATUS_ALREADY_EXISTS: code = IREE_STATUS_ALREADY_EXISTS; break;
    default: break;
  }
  return iree_make_status(code, "%s", hxb_last_error_message());
}

// iree_allocator_t and hxb_allocator_t have the same shape (self + control
// function over MALLOC / CALLOC / REALLOC / FREE with a byte-length params
// struct); the control function is called through a trampoline so the
// status types stay separate.
static hxb_status_t b200_allocator_ctl(void* self, hxb_allocator_command_t command,
                                       const void* params, void** inout_ptr) {
  const iree_allocator_t* a = (const iree_allocator_t*)self;
  iree_allocator_alloc_params_t p = {0};
  if (params) p.byte_length = ((const hxb_allocator_alloc_params_t*)params)->byte_length;
  iree_status_t st = a->ctl(a->self, (iree_allocator_command_t)command, params ? &p : NULL,
                            inout_ptr);
  if (iree_status_is_ok(st)) return HXB_OK;
  iree_status_ignore(st);
  return HXB_STATUS_RESOURCE_EXHAUSTED;
}

static iree_status_t iree_hal_b200_driver_factory_enumerate(
    void* self, iree_host_size_t* out_driver_info_count,
    const iree_hal_driver_info_t** out_driver_infos) {
  static const iree_hal_driver_info_t default_driver_info = {
      .driver_name = IREE_SVL("b200"),
      .full_name = IREE_SVL("NVIDIA B200 (sm_100a) CUDA driver"),
  };
  *out_driver_info_count = 1;
  *out_driver_infos = &default_driver_info;
  return iree_ok_status();
}

static iree_status_t iree_hal_b200_driver_factory_try_create(
    void* self, iree_string_view_t driver_name, iree_allocator_t host_allocator,
    iree_hal_driver_t** out_driver) {
  if (!iree_string_view_equal(driver_name, IREE_SV("b200"))) {
    return iree_make_status(IREE_STATUS_UNAVAILABLE,
                            "no driver '%.*s' is provided by this factory",
                            (int)driver_name.size, driver_name.data);
  }
  if (FLAG_b200_queue_wait_timeout_ms <= 0 || FLAG_b200_queue_wait_timeout_ms > 60000 ||
      FLAG_b200_scratch_bytes < 0) {
    return iree_make_status(IREE_STATUS_INVALID_ARGUMENT,
                            "b200_queue_wait_timeout_ms must be in (0, 60000] and "
                            "b200_scratch_bytes non-negative");
  }
  hxb_hal_driver_options_t options;
  hxb_hal_driver_options_initialize(&options);
  options.default_device_options.scratch_bytes = (uint64_t)FLAG_b200_scratch_bytes;
  options.default_device_options.queue_wait_timeout_ns =
      (uint64_t)FLAG_b200_queue_wait_timeout_ms * 1000000ull;

  // the allocator outlives the driver: it is the one the tool passed in
  iree_allocator_t* held = NULL;
  IREE_RETURN_IF_ERROR(iree_allocator_malloc(host_allocator, sizeof(*held), (void**)&held));
  *held = host_allocator;
  const hxb_allocator_t alloc = {held, b200_allocator_ctl};
  hxb_hal_driver_t* driver = NULL;
  iree_status_t status = b200_status(hxb_hal_driver_create(
      (hxb_string_view_t){driver_name.data, driver_name.size}, &options, alloc, &driver));
  if (!iree_status_is_ok(status)) {
    iree_allocator_free(host_allocator, held);
    return status;
  }
  // wrap in the IREE driver object (resource header + vtable over the
  // hxb_hal_driver_t; see the header comment)
  return iree_hal_b200_driver_wrap(driver, held, host_allocator, out_driver);
}

IREE_API_EXPORT iree_status_t
iree_hal_b200_driver_module_register(iree_hal_driver_registry_t* registry) {
  static const iree_hal_driver_factory_t factory = {
      .self = NULL,
      .enumerate = iree_hal_b200_driver_factory_enumerate,
      .try_create = iree_hal_b200_driver_factory_try_create,
  };
  return iree_hal_driver_registry_register_factory(registry, &factory);
}
