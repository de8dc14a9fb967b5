// HAL-shaped runtime over the B200 dispatch library (include/hxb200_hal.h,
// part 2): driver, device (a CUDA device with its own queue stream and
// scratch arena), buffers, timeline semaphores and command buffers.
//
// A command buffer records dispatches of the executable library's exports;
// end() runs every recorded dispatch function once under stream capture, so
// argument errors surface there and the recording becomes one CUDA graph.
// Queue submission is a graph launch on the device's stream, preceded by a
// stream wait on the wait semaphore's value and followed by a stream write of
// the signal value (CUDA stream memory operations on host-mapped memory), so
// submission never blocks the host. The reference's queue is synchronous
// (plugins/runtime/hexagon/device.c:1068-1112).
#include <string.h>

#include <chrono>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "hxb200_hal.h"
#include "runtime_common.h"

namespace hxb {
size_t w8_streamk_workspace_bytes(int ctas);
}

struct hxb_hal_driver_s {
  std::string identifier;
  hxb_hal_driver_options_t options;
};

struct hxb_hal_device_s {
  std::string identifier;
  int ordinal = 0;
  cudaStream_t queue = nullptr;
  void* scratch = nullptr;
  uint64_t scratch_bytes = 0;
  bool stream_mem_ops = false;
};

struct hxb_hal_buffer_s {
  hxb_hal_device_t* device = nullptr;
  void* ptr = nullptr;
  uint64_t bytes = 0;
};

struct hxb_hal_semaphore_s {
  hxb_hal_device_t* device = nullptr;
  uint64_t* host = nullptr;  // host-mapped pinned memory
  CUdeviceptr dev = 0;       // its device address
};

namespace {

struct Recorded {
  uint32_t ordinal;
  std::vector<uint32_t> constants;
  std::vector<void*> ptrs;
  std::vector<size_t> lengths;
};

enum CbState { kCbInitial, kCbRecording, kCbExecutable };

}  // namespace

struct hxb_hal_command_buffer_s {
  hxb_hal_device_t* device = nullptr;
  CbState state = kCbInitial;
  std::vector<Recorded> commands;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

namespace {

using hxb::cuda_status;
using hxb::fail;

typedef CUresult (*WriteValue64Fn)(CUstream, CUdeviceptr, cuuint64_t, unsigned int);
typedef CUresult (*WaitValue64Fn)(CUstream, CUdeviceptr, cuuint64_t, unsigned int);
typedef CUresult (*DeviceGetAttributeFn)(int*, CUdevice_attribute, CUdevice);

template <class Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion(name, &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

WriteValue64Fn write_value64() {
  static WriteValue64Fn f = driver_fn<WriteValue64Fn>("cuStreamWriteValue64");
  return f;
}
WaitValue64Fn wait_value64() {
  static WaitValue64Fn f = driver_fn<WaitValue64Fn>("cuStreamWaitValue64");
  return f;
}

// Sets the device for the calling thread; every HAL call that touches CUDA
// goes through this first.
hxb_status_t use_device(const hxb_hal_device_t* d) {
  return cuda_status(cudaSetDevice(d->ordinal), "cudaSetDevice");
}

uint64_t load_acquire(const uint64_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }

void destroy_graph(hxb_hal_command_buffer_t* cb) {
  if (cb->exec) cudaGraphExecDestroy(cb->exec);
  if (cb->graph) cudaGraphDestroy(cb->graph);
  cb->exec = nullptr;
  cb->graph = nullptr;
}

const hxb_executable_library_t* lib() {
  return reinterpret_cast<const hxb_executable_library_t*>(
      hxb_executable_library_query(HXB_EXECUTABLE_LIBRARY_VERSION_LATEST, nullptr));
}

}  // namespace

extern "C" {

void hxb_hal_device_options_initialize(hxb_hal_device_options_t* o) {
  if (!o) return;
  o->ordinal = 0;
  o->scratch_bytes = 0;
}

void hxb_hal_driver_options_initialize(hxb_hal_driver_options_t* o) {
  if (!o) return;
  hxb_hal_device_options_initialize(&o->default_device_options);
}

hxb_status_t hxb_hal_driver_create(const char* identifier, const hxb_hal_driver_options_t* options,
                                   hxb_hal_driver_t** out_driver) {
  if (!out_driver) return fail(HXB_STATUS_INVALID_ARGUMENT, "driver_create: null out_driver");
  *out_driver = nullptr;
  hxb_hal_driver_t* d = new (std::nothrow) hxb_hal_driver_s();
  if (!d) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "driver_create: out of host memory");
  d->identifier = identifier ? identifier : "b200";
  if (options)
    d->options = *options;
  else
    hxb_hal_driver_options_initialize(&d->options);
  *out_driver = d;
  return HXB_OK;
}

hxb_status_t hxb_hal_driver_query_device_count(hxb_hal_driver_t* driver, int32_t* out_count) {
  if (!driver || !out_count) return fail(HXB_STATUS_INVALID_ARGUMENT, "query_device_count: null");
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  *out_count = n;
  return HXB_OK;
}

void hxb_hal_driver_release(hxb_hal_driver_t* driver) { delete driver; }

hxb_status_t hxb_hal_device_create(hxb_hal_driver_t* driver, const char* identifier,
                                   const hxb_hal_device_options_t* options,
                                   hxb_hal_device_t** out_device) {
  if (!driver || !out_device) return fail(HXB_STATUS_INVALID_ARGUMENT, "device_create: null");
  *out_device = nullptr;
  const hxb_hal_device_options_t o = options ? *options : driver->options.default_device_options;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || o.ordinal < 0 || o.ordinal >= n) {
    cudaGetLastError();
    return fail(HXB_STATUS_INVALID_ARGUMENT, "device_create: no CUDA device %d (%d present)",
                (int)o.ordinal, n);
  }
  hxb_hal_device_t* d = new (std::nothrow) hxb_hal_device_s();
  if (!d) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "device_create: out of host memory");
  d->identifier = identifier ? identifier : driver->identifier;
  d->ordinal = o.ordinal;
  hxb_status_t s = use_device(d);
  hxb::DeviceInfo* info = nullptr;
  // resolve the per-device state of the dispatch library now, outside any
  // stream capture
  if (s == HXB_OK) s = hxb::current_device(&info);
  if (s == HXB_OK)
    s = cuda_status(cudaStreamCreateWithFlags(&d->queue, cudaStreamNonBlocking),
                    "cudaStreamCreate");
  if (s == HXB_OK) {
    d->scratch_bytes =
        o.scratch_bytes ? o.scratch_bytes : hxb::w8_streamk_workspace_bytes(info->num_sms);
    s = cuda_status(cudaMalloc(&d->scratch, d->scratch_bytes), "cudaMalloc(scratch)");
  }
  if (s == HXB_OK) s = cuda_status(cudaMemset(d->scratch, 0, d->scratch_bytes), "cudaMemset");
  if (s == HXB_OK) {
    auto attr = driver_fn<DeviceGetAttributeFn>("cuDeviceGetAttribute");
    int v = 0;
    d->stream_mem_ops = attr && write_value64() && wait_value64() &&
                        attr(&v, CU_DEVICE_ATTRIBUTE_CAN_USE_64_BIT_STREAM_MEM_OPS,
                             (CUdevice)d->ordinal) == CUDA_SUCCESS &&
                        v != 0;
  }
  if (s != HXB_OK) {
    hxb_hal_device_release(d);
    return s;
  }
  *out_device = d;
  return HXB_OK;
}

void hxb_hal_device_release(hxb_hal_device_t* d) {
  if (!d) return;
  if (use_device(d) == HXB_OK) {
    if (d->queue) cudaStreamSynchronize(d->queue);
    if (d->scratch) cudaFree(d->scratch);
    if (d->queue) cudaStreamDestroy(d->queue);
  }
  delete d;
}

void* hxb_hal_device_queue_stream(hxb_hal_device_t* d) { return d ? (void*)d->queue : nullptr; }

hxb_status_t hxb_hal_buffer_allocate(hxb_hal_device_t* d, uint64_t bytes,
                                     hxb_hal_buffer_t** out) {
  if (!d || !out || bytes == 0) return fail(HXB_STATUS_INVALID_ARGUMENT, "buffer_allocate: bad args");
  *out = nullptr;
  hxb_status_t s = use_device(d);
  if (s != HXB_OK) return s;
  hxb_hal_buffer_t* b = new (std::nothrow) hxb_hal_buffer_s();
  if (!b) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "buffer_allocate: out of host memory");
  b->device = d;
  b->bytes = bytes;
  if ((s = cuda_status(cudaMalloc(&b->ptr, bytes), "cudaMalloc(buffer)")) != HXB_OK) {
    delete b;
    return s;
  }
  *out = b;
  return HXB_OK;
}

void* hxb_hal_buffer_device_pointer(hxb_hal_buffer_t* b) { return b ? b->ptr : nullptr; }
uint64_t hxb_hal_buffer_byte_length(hxb_hal_buffer_t* b) { return b ? b->bytes : 0; }

hxb_status_t hxb_hal_buffer_write(hxb_hal_buffer_t* b, uint64_t offset, const void* host,
                                  uint64_t bytes) {
  if (!b || (!host && bytes) || offset > b->bytes || bytes > b->bytes - offset)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "buffer_write: range outside the buffer");
  hxb_status_t s = use_device(b->device);
  if (s != HXB_OK || bytes == 0) return s;
  s = cuda_status(cudaMemcpyAsync(static_cast<uint8_t*>(b->ptr) + offset, host, bytes,
                                  cudaMemcpyHostToDevice, b->device->queue),
                  "buffer_write");
  if (s != HXB_OK) return s;
  return cuda_status(cudaStreamSynchronize(b->device->queue), "buffer_write");
}

hxb_status_t hxb_hal_buffer_read(hxb_hal_buffer_t* b, uint64_t offset, void* host,
                                 uint64_t bytes) {
  if (!b || (!host && bytes) || offset > b->bytes || bytes > b->bytes - offset)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "buffer_read: range outside the buffer");
  hxb_status_t s = use_device(b->device);
  if (s != HXB_OK || bytes == 0) return s;
  s = cuda_status(cudaMemcpyAsync(host, static_cast<const uint8_t*>(b->ptr) + offset, bytes,
                                  cudaMemcpyDeviceToHost, b->device->queue),
                  "buffer_read");
  if (s != HXB_OK) return s;
  return cuda_status(cudaStreamSynchronize(b->device->queue), "buffer_read");
}

void hxb_hal_buffer_release(hxb_hal_buffer_t* b) {
  if (!b) return;
  if (use_device(b->device) == HXB_OK) {
    cudaStreamSynchronize(b->device->queue);
    cudaFree(b->ptr);
  }
  delete b;
}

hxb_status_t hxb_hal_semaphore_create(hxb_hal_device_t* d, uint64_t initial,
                                      hxb_hal_semaphore_t** out) {
  if (!d || !out) return fail(HXB_STATUS_INVALID_ARGUMENT, "semaphore_create: null");
  *out = nullptr;
  hxb_status_t s = use_device(d);
  if (s != HXB_OK) return s;
  hxb_hal_semaphore_t* sem = new (std::nothrow) hxb_hal_semaphore_s();
  if (!sem) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "semaphore_create: out of host memory");
  sem->device = d;
  void* h = nullptr;
  if ((s = cuda_status(cudaHostAlloc(&h, sizeof(uint64_t), cudaHostAllocMapped),
                       "cudaHostAlloc(semaphore)")) != HXB_OK) {
    delete sem;
    return s;
  }
  sem->host = static_cast<uint64_t*>(h);
  __atomic_store_n(sem->host, initial, __ATOMIC_RELEASE);
  void* dp = nullptr;
  if ((s = cuda_status(cudaHostGetDevicePointer(&dp, h, 0), "cudaHostGetDevicePointer")) !=
      HXB_OK) {
    cudaFreeHost(h);
    delete sem;
    return s;
  }
  sem->dev = reinterpret_cast<CUdeviceptr>(dp);
  *out = sem;
  return HXB_OK;
}

hxb_status_t hxb_hal_semaphore_query(hxb_hal_semaphore_t* sem, uint64_t* out_value) {
  if (!sem || !out_value) return fail(HXB_STATUS_INVALID_ARGUMENT, "semaphore_query: null");
  *out_value = load_acquire(sem->host);
  return HXB_OK;
}

hxb_status_t hxb_hal_semaphore_signal(hxb_hal_semaphore_t* sem, uint64_t value) {
  if (!sem) return fail(HXB_STATUS_INVALID_ARGUMENT, "semaphore_signal: null");
  if (value < load_acquire(sem->host))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "semaphore_signal: %llu is below the current value",
                (unsigned long long)value);
  __atomic_store_n(sem->host, value, __ATOMIC_RELEASE);
  return HXB_OK;
}

hxb_status_t hxb_hal_semaphore_wait(hxb_hal_semaphore_t* sem, uint64_t value,
                                    uint64_t timeout_ns) {
  if (!sem) return fail(HXB_STATUS_INVALID_ARGUMENT, "semaphore_wait: null");
  const auto t0 = std::chrono::steady_clock::now();
  while (load_acquire(sem->host) < value) {
    const auto dt = std::chrono::duration_cast<std::chrono::nanoseconds>(
        std::chrono::steady_clock::now() - t0);
    if ((uint64_t)dt.count() >= timeout_ns)
      return fail(HXB_STATUS_DEVICE_TIMEOUT, "semaphore_wait: value %llu not reached in %llu ns",
                  (unsigned long long)value, (unsigned long long)timeout_ns);
    std::this_thread::sleep_for(std::chrono::microseconds(2));
  }
  return HXB_OK;
}

void hxb_hal_semaphore_release(hxb_hal_semaphore_t* sem) {
  if (!sem) return;
  if (use_device(sem->device) == HXB_OK) {
    cudaStreamSynchronize(sem->device->queue);
    cudaFreeHost(sem->host);
  }
  delete sem;
}

hxb_status_t hxb_hal_command_buffer_create(hxb_hal_device_t* d, hxb_hal_command_buffer_t** out) {
  if (!d || !out) return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_create: null");
  *out = nullptr;
  hxb_hal_command_buffer_t* cb = new (std::nothrow) hxb_hal_command_buffer_s();
  if (!cb) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "command_buffer_create: out of host memory");
  cb->device = d;
  *out = cb;
  return HXB_OK;
}

hxb_status_t hxb_hal_command_buffer_begin(hxb_hal_command_buffer_t* cb) {
  if (!cb) return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_begin: null");
  if (cb->state == kCbRecording)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_begin: already recording");
  if (use_device(cb->device) == HXB_OK) destroy_graph(cb);
  cb->commands.clear();
  cb->state = kCbRecording;
  return HXB_OK;
}

hxb_status_t hxb_hal_command_buffer_dispatch(hxb_hal_command_buffer_t* cb, uint32_t ordinal,
                                             const uint32_t* constants, uint32_t constant_count,
                                             const hxb_hal_buffer_ref_t* bindings,
                                             uint32_t binding_count) {
  if (!cb || cb->state != kCbRecording)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_dispatch: not recording");
  const hxb_executable_library_t* l = lib();
  if (ordinal >= l->exports.count)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_dispatch: no export %u", ordinal);
  if ((constant_count && !constants) || (binding_count && !bindings) || binding_count > 255)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_dispatch: bad arrays");
  Recorded r;
  r.ordinal = ordinal;
  r.constants.assign(constants, constants + constant_count);
  // exports read up to 9 constants; missing ones read as 0
  if (r.constants.size() < 16) r.constants.resize(16, 0u);
  for (uint32_t i = 0; i < binding_count; ++i) {
    const hxb_hal_buffer_ref_t& b = bindings[i];
    if (!b.buffer || b.buffer->device != cb->device || b.offset > b.buffer->bytes ||
        b.length > b.buffer->bytes - b.offset)
      return fail(HXB_STATUS_INVALID_ARGUMENT,
                  "command_buffer_dispatch: binding %u is not a range of a buffer of this device",
                  i);
    r.ptrs.push_back(static_cast<uint8_t*>(b.buffer->ptr) + b.offset);
    r.lengths.push_back((size_t)b.length);
  }
  cb->commands.push_back(std::move(r));
  return HXB_OK;
}

hxb_status_t hxb_hal_command_buffer_end(hxb_hal_command_buffer_t* cb) {
  if (!cb || cb->state != kCbRecording)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_end: not recording");
  hxb_status_t s = use_device(cb->device);
  if (s != HXB_OK) return s;
  const hxb_executable_library_t* l = lib();
  cudaStream_t cap = nullptr;
  if ((s = cuda_status(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking),
                       "cudaStreamCreate(capture)")) != HXB_OK)
    return s;
  s = cuda_status(cudaStreamBeginCapture(cap, cudaStreamCaptureModeRelaxed),
                  "cudaStreamBeginCapture");
  if (s == HXB_OK) {
    hxb_executable_environment_t env{nullptr, cap, cb->device->scratch,
                                     cb->device->scratch_bytes};
    for (size_t i = 0; i < cb->commands.size() && s == HXB_OK; ++i) {
      const Recorded& r = cb->commands[i];
      hxb_executable_dispatch_state_t ds{};
      ds.workgroup_size_x = ds.workgroup_size_y = 1;
      ds.workgroup_size_z = 1;
      ds.workgroup_count_x = ds.workgroup_count_y = 1;
      ds.workgroup_count_z = 1;
      ds.binding_count = (uint8_t)r.ptrs.size();
      ds.constants = r.constants.data();
      ds.binding_ptrs = r.ptrs.data();
      ds.binding_lengths = r.lengths.data();
      const int rc = l->exports.ptrs[r.ordinal](&env, &ds, nullptr);
      if (rc != 0) s = (hxb_status_t)rc;  // the message is already set
    }
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(cap, &g);
    if (s == HXB_OK) s = cuda_status(e, "cudaStreamEndCapture");
    if (s == HXB_OK) {
      cb->graph = g;
      s = cuda_status(cudaGraphInstantiate(&cb->exec, g, 0), "cudaGraphInstantiate");
    } else if (g) {
      cudaGraphDestroy(g);
    }
  }
  cudaStreamDestroy(cap);
  if (s != HXB_OK) {
    destroy_graph(cb);
    cb->state = kCbInitial;
    return s;
  }
  cb->state = kCbExecutable;
  return HXB_OK;
}

void hxb_hal_command_buffer_release(hxb_hal_command_buffer_t* cb) {
  if (!cb) return;
  if (use_device(cb->device) == HXB_OK) {
    cudaStreamSynchronize(cb->device->queue);
    destroy_graph(cb);
  }
  delete cb;
}

hxb_status_t hxb_hal_device_queue_execute(hxb_hal_device_t* d, hxb_hal_semaphore_t* wait_sem,
                                          uint64_t wait_value, hxb_hal_command_buffer_t* cb,
                                          hxb_hal_semaphore_t* signal_sem,
                                          uint64_t signal_value) {
  if (!d || (cb && (cb->device != d || cb->state != kCbExecutable)) ||
      (wait_sem && wait_sem->device != d) || (signal_sem && signal_sem->device != d))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "queue_execute: command buffer not ended, or objects of another device");
  hxb_status_t s = use_device(d);
  if (s != HXB_OK) return s;
  if (wait_sem && load_acquire(wait_sem->host) < wait_value) {
    if (!d->stream_mem_ops)
      return fail(HXB_STATUS_UNSUPPORTED,
                  "queue_execute: the device has no 64-bit stream memory operations");
    if (wait_value64()(d->queue, wait_sem->dev, wait_value, CU_STREAM_WAIT_VALUE_GEQ) !=
        CUDA_SUCCESS)
      return fail(HXB_STATUS_CUDA_ERROR, "queue_execute: cuStreamWaitValue64 failed");
  }
  if (cb && (s = cuda_status(cudaGraphLaunch(cb->exec, d->queue), "cudaGraphLaunch")) != HXB_OK)
    return s;
  if (signal_sem) {
    if (d->stream_mem_ops) {
      if (write_value64()(d->queue, signal_sem->dev, signal_value, CU_STREAM_WRITE_VALUE_DEFAULT) !=
          CUDA_SUCCESS)
        return fail(HXB_STATUS_CUDA_ERROR, "queue_execute: cuStreamWriteValue64 failed");
    } else {
      // no stream memory operations: complete the queue work, then signal
      if ((s = cuda_status(cudaStreamSynchronize(d->queue), "queue_execute")) != HXB_OK) return s;
      __atomic_store_n(signal_sem->host, signal_value, __ATOMIC_RELEASE);
    }
  }
  return HXB_OK;
}

}  // extern "C"
