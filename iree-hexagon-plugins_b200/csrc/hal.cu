// HAL-shaped runtime over the B200 dispatch library (include/hxb200_hal.h,
// part 2): driver, driver registry and factory, device (a CUDA device with
// its own queue stream and scratch arena), buffers, timeline semaphores and
// command buffers.
//
// A command buffer records dispatches of the executable library's exports.
// Recorded dispatches whose bindings are all direct are run once by end()
// under stream capture, so argument errors surface there and the recording
// becomes one CUDA graph. Dispatches that bind binding-table slots are
// captured at their first submission, when the table supplies the addresses,
// and re-captured into the same executable graph (cudaGraphExecUpdate) when a
// later table binds other ones; the reference resolves its tables at
// submission as well (plugins/runtime/hexagon/device.c:977-1012).
//
// Queue submission is a graph launch on the device's stream, preceded by a
// bounded one-thread wait kernel on the wait semaphore and followed by a
// one-thread signal kernel, so submission never blocks the host and no
// device-side wait lasts longer than the device's queue wait bound. The
// reference's queue is synchronous (plugins/runtime/hexagon/device.c:
// 1068-1112).
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "hxb200_hal.h"
#include "runtime_common.h"
#include "sm100.cuh"

namespace hxb {
size_t w8_streamk_workspace_bytes(int ctas);
// Resolves the built-in scratch of hxb_matmul_f16_noalloc for the current
// device (matmul_noalloc.cu), so that no capture has to.
hxb_status_t noalloc_prepare_current_device();
}  // namespace hxb

namespace {

using hxb::cuda_status;
using hxb::fail;

// ------------------------------------------------------------ host memory
// Every host object is allocated through the allocator it was created with.
void* host_alloc(const hxb_allocator_t& a, size_t bytes) {
  if (!a.ctl) return calloc(1, bytes);
  hxb_allocator_alloc_params_t p{bytes};
  void* out = nullptr;
  if (a.ctl(a.self, HXB_ALLOCATOR_COMMAND_CALLOC, &p, &out) != HXB_OK) return nullptr;
  return out;
}

void host_free(const hxb_allocator_t& a, void* p) {
  if (!p) return;
  if (!a.ctl) {
    free(p);
    return;
  }
  a.ctl(a.self, HXB_ALLOCATOR_COMMAND_FREE, nullptr, &p);
}

template <class T>
T* host_new(const hxb_allocator_t& a) {
  void* m = host_alloc(a, sizeof(T));
  return m ? new (m) T() : nullptr;
}

template <class T>
void host_delete(const hxb_allocator_t& a, T* p) {
  if (!p) return;
  p->~T();
  host_free(a, p);
}

std::string to_string(hxb_string_view_t v) {
  return v.data ? std::string(v.data, v.size) : std::string();
}

}  // namespace

struct hxb_hal_driver_s {
  hxb_allocator_t allocator{};
  std::string identifier;
  hxb_hal_driver_options_t options{};
};

struct hxb_hal_device_s {
  hxb_allocator_t allocator{};
  std::string identifier;
  int ordinal = 0;
  cudaStream_t queue = nullptr;
  void* scratch = nullptr;
  uint64_t scratch_bytes = 0;
  uint64_t wait_timeout_ns = HXB_HAL_DEFAULT_QUEUE_WAIT_TIMEOUT_NS;
  int* status_word = nullptr;  // the dispatch library's per-device word
  int* lost_host = nullptr;    // host-mapped: set by a queue wait that ran out
  int* lost_dev = nullptr;     // its device address
};

struct hxb_hal_buffer_s {
  hxb_hal_device_t* device = nullptr;
  void* ptr = nullptr;
  uint64_t bytes = 0;
};

struct hxb_hal_semaphore_s {
  hxb_hal_device_t* device = nullptr;
  uint64_t* host = nullptr;  // host-mapped pinned memory
  uint64_t* dev = nullptr;   // its device address
};

struct hxb_hal_channel_s {
  hxb_hal_device_t* device = nullptr;
  ncclComm_t comm = nullptr;
  int32_t rank = 0;
  int32_t count = 1;
  uint64_t timeout_ns = 0;
};

namespace {

struct Ref {
  hxb_hal_buffer_t* buffer;  // NULL: binding-table slot
  uint32_t slot;
  uint64_t offset;
  uint64_t length;
};

constexpr uint32_t kCollective = 0xFFFFFFFFu;  // Recorded::ordinal of a collective

struct Recorded {
  uint32_t ordinal;  // export ordinal, or kCollective
  std::vector<uint32_t> constants;
  std::vector<Ref> refs;
  // collectives: refs = {send, recv}
  hxb_hal_channel_t* channel = nullptr;
  int op = 0;
  int dtype = 0;
  uint64_t count = 0;
};

enum CbState { kCbInitial, kCbRecording, kCbExecutable };

}  // namespace

struct hxb_hal_command_buffer_s {
  hxb_hal_device_t* device = nullptr;
  uint32_t binding_capacity = 0;
  CbState state = kCbInitial;
  bool indirect = false;  // some binding names a table slot
  std::vector<Recorded> commands;
  std::vector<void*> last_resolved;  // the addresses the graph was captured with
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

namespace {

// ------------------------------------------------------------------ NCCL
// Loaded at run time so that the library needs NCCL only when a channel is
// made: the libnccl.so.2 already in the process (PyTorch's, say) or the
// system's.
struct Nccl {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*comm_finalize)(ncclComm_t);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*comm_abort)(ncclComm_t);
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t);
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                             ncclComm_t, cudaStream_t);
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                                 ncclComm_t, cudaStream_t);
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t);
  const char* (*error_string)(ncclResult_t);
};

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    bool all = true;
    auto sym = [&](auto& fn, const char* name) {
      *reinterpret_cast<void**>(&fn) = dlsym(h, name);
      all = all && fn != nullptr;
    };
    sym(n.get_unique_id, "ncclGetUniqueId");
    sym(n.comm_init_rank_config, "ncclCommInitRankConfig");
    sym(n.comm_get_async_error, "ncclCommGetAsyncError");
    sym(n.comm_finalize, "ncclCommFinalize");
    sym(n.comm_destroy, "ncclCommDestroy");
    sym(n.comm_abort, "ncclCommAbort");
    sym(n.all_gather, "ncclAllGather");
    sym(n.all_reduce, "ncclAllReduce");
    sym(n.reduce_scatter, "ncclReduceScatter");
    sym(n.broadcast, "ncclBroadcast");
    sym(n.error_string, "ncclGetErrorString");
    n.ok = all;
  });
  return n;
}

// Polls a non-blocking communicator until its pending operation completes,
// for at most timeout_ns.
hxb_status_t nccl_settle(ncclComm_t comm, ncclResult_t r, uint64_t timeout_ns, const char* what) {
  const Nccl& n = nccl();
  const auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress) {
    if ((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
            std::chrono::steady_clock::now() - t0)
            .count() > timeout_ns)
      return fail(HXB_STATUS_DEVICE_TIMEOUT, "%s: not complete after %llu ns", what,
                  (unsigned long long)timeout_ns);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    if (n.comm_get_async_error(comm, &r) != ncclSuccess) break;
  }
  if (r != ncclSuccess)
    return fail(HXB_STATUS_CUDA_ERROR, "%s: %s", what, n.error_string(r));
  return HXB_OK;
}

// ------------------------------------------------------- queue wait/signal
// One thread polls the host-mapped semaphore word until it reaches `value`,
// sleeping ~2 us between reads, for at most `limit_ns`. When the bound runs
// out it ORs the timeout bit into the dispatch library's status word and
// marks the device lost (host-mapped, so the host sees it without a sync).
__global__ void queue_wait_kernel(const volatile unsigned long long* sem, unsigned long long value,
                                  unsigned long long limit_ns, int* status, volatile int* lost) {
  if (*lost) return;  // the device is lost already: do not wait again
  const unsigned long long t0 = hxb::globaltimer_ns();
  while (*sem < value) {
    if (hxb::globaltimer_ns() - t0 > limit_ns) {
      atomicOr(status, hxb::kStatusTimeout);
      *lost = 1;
      __threadfence_system();
      return;
    }
    __nanosleep(2000);
  }
}

// Publishes `value` after every earlier operation of the queue, unless a wait
// of this device ran out (then the value is never reached, and the waiters
// on it time out in their turn).
__global__ void queue_signal_kernel(volatile unsigned long long* sem, unsigned long long value,
                                    const volatile int* lost) {
  if (*lost) return;
  __threadfence_system();
  if (*sem < value) *sem = value;
  __threadfence_system();
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
  cb->last_resolved.clear();
}

const hxb_executable_library_t* lib() {
  return reinterpret_cast<const hxb_executable_library_t*>(
      hxb_executable_library_query(HXB_EXECUTABLE_LIBRARY_VERSION_LATEST, nullptr));
}

// Device addresses and lengths of every recorded binding, with table slots
// resolved through `table` (NULL when the command buffer has no slots).
hxb_status_t resolve(const hxb_hal_command_buffer_t* cb,
                     const hxb_hal_buffer_binding_table_t* table, std::vector<void*>* ptrs,
                     std::vector<size_t>* lengths) {
  ptrs->clear();
  lengths->clear();
  for (size_t c = 0; c < cb->commands.size(); ++c) {
    for (size_t i = 0; i < cb->commands[c].refs.size(); ++i) {
      const Ref& r = cb->commands[c].refs[i];
      uint8_t* base = nullptr;
      uint64_t avail = 0;
      if (r.buffer) {
        base = static_cast<uint8_t*>(r.buffer->ptr);
        avail = r.buffer->bytes;
      } else {
        if (!table || r.slot >= table->count || !table->bindings)
          return fail(HXB_STATUS_INVALID_ARGUMENT,
                      "dispatch %zu binding %zu names table slot %u, but the binding table "
                      "has %u entries",
                      c, i, r.slot, table ? table->count : 0u);
        const hxb_hal_buffer_binding_t& b = table->bindings[r.slot];
        if (!b.buffer || b.buffer->device != cb->device || b.offset > b.buffer->bytes ||
            b.length > b.buffer->bytes - b.offset)
          return fail(HXB_STATUS_INVALID_ARGUMENT,
                      "binding table slot %u is not a range of a buffer of this device", r.slot);
        base = static_cast<uint8_t*>(b.buffer->ptr) + b.offset;
        avail = b.length;
      }
      if (r.offset > avail || r.length > avail - r.offset)
        return fail(HXB_STATUS_INVALID_ARGUMENT,
                    "dispatch %zu binding %zu: range [%llu, +%llu) exceeds its %llu-byte binding",
                    c, i, (unsigned long long)r.offset, (unsigned long long)r.length,
                    (unsigned long long)avail);
      ptrs->push_back(base + r.offset);
      lengths->push_back((size_t)r.length);
    }
  }
  return HXB_OK;
}

ncclDataType_t nccl_type(int dtype) {
  return dtype == HXB_DTYPE_F16 ? ncclFloat16 : dtype == HXB_DTYPE_F32 ? ncclFloat32 : ncclInt8;
}

// Issues one recorded collective on `stream` (a capturing stream: NCCL's
// kernels become nodes of the command buffer's graph).
hxb_status_t run_collective(const Recorded& r, void* const* p, cudaStream_t stream) {
  const Nccl& n = nccl();
  hxb_hal_channel_t* ch = r.channel;
  const ncclDataType_t t = nccl_type(r.dtype);
  ncclResult_t res = ncclSuccess;
  switch (r.op) {
    case HXB_HAL_COLLECTIVE_ALL_GATHER:
      res = n.all_gather(p[0], p[1], r.count, t, ch->comm, stream);
      break;
    case HXB_HAL_COLLECTIVE_ALL_REDUCE_SUM:
      res = n.all_reduce(p[0], p[1], r.count, t, ncclSum, ch->comm, stream);
      break;
    case HXB_HAL_COLLECTIVE_REDUCE_SCATTER_SUM:
      res = n.reduce_scatter(p[0], p[1], r.count, t, ncclSum, ch->comm, stream);
      break;
    default:
      res = n.broadcast(p[0], p[1], r.count, t, 0, ch->comm, stream);
      break;
  }
  return nccl_settle(ch->comm, res, ch->timeout_ns, "collective");
}

// Runs every recorded dispatch function once on a capturing stream and
// returns the graph (argument errors of any dispatch come back here).
hxb_status_t capture(hxb_hal_command_buffer_t* cb, const std::vector<void*>& ptrs,
                     const std::vector<size_t>& lengths, cudaGraph_t* out) {
  *out = nullptr;
  const hxb_executable_library_t* l = lib();
  cudaStream_t cap = nullptr;
  hxb_status_t s = cuda_status(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking),
                               "cudaStreamCreate(capture)");
  if (s != HXB_OK) return s;
  s = cuda_status(cudaStreamBeginCapture(cap, cudaStreamCaptureModeRelaxed),
                  "cudaStreamBeginCapture");
  if (s == HXB_OK) {
    hxb_executable_environment_t env{nullptr, cap, cb->device->scratch,
                                     cb->device->scratch_bytes};
    size_t next = 0;
    for (size_t i = 0; i < cb->commands.size() && s == HXB_OK; ++i) {
      const Recorded& r = cb->commands[i];
      if (r.ordinal == kCollective) {
        s = run_collective(r, ptrs.data() + next, cap);
        next += r.refs.size();
        continue;
      }
      hxb_executable_dispatch_state_t ds{};
      ds.workgroup_size_x = ds.workgroup_size_y = 1;
      ds.workgroup_size_z = 1;
      ds.workgroup_count_x = ds.workgroup_count_y = 1;
      ds.workgroup_count_z = 1;
      ds.binding_count = (uint8_t)r.refs.size();
      ds.constants = r.constants.data();
      ds.binding_ptrs = ptrs.data() + next;
      ds.binding_lengths = lengths.data() + next;
      next += r.refs.size();
      const int rc = l->exports.ptrs[r.ordinal](&env, &ds, nullptr);
      if (rc != 0) s = (hxb_status_t)rc;  // the message is already set
    }
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(cap, &g);
    if (s == HXB_OK) s = cuda_status(e, "cudaStreamEndCapture");
    if (s == HXB_OK)
      *out = g;
    else if (g)
      cudaGraphDestroy(g);
  }
  cudaStreamDestroy(cap);
  // a failed capture leaves its error as the thread's last error; it is
  // reported through `s` and must not surface at a later, unrelated launch
  if (s != HXB_OK) cudaGetLastError();
  return s;
}

// Makes cb->exec run the dispatches with the given addresses: the first
// time by instantiating, later by updating the executable graph in place
// (same dispatches, so the same topology), re-instantiating if the update
// is refused.
hxb_status_t install(hxb_hal_command_buffer_t* cb, const std::vector<void*>& ptrs,
                     const std::vector<size_t>& lengths) {
  cudaGraph_t g = nullptr;
  hxb_status_t s = capture(cb, ptrs, lengths, &g);
  if (s != HXB_OK) return s;
  if (cb->exec) {
    cudaGraphExecUpdateResultInfo info;
    if (cudaGraphExecUpdate(cb->exec, g, &info) == cudaSuccess) {
      if (cb->graph) cudaGraphDestroy(cb->graph);
      cb->graph = g;
      cb->last_resolved = ptrs;
      return HXB_OK;
    }
    cudaGetLastError();
    cudaGraphExecDestroy(cb->exec);
    cb->exec = nullptr;
  }
  if (cb->graph) cudaGraphDestroy(cb->graph);
  cb->graph = g;
  s = cuda_status(cudaGraphInstantiate(&cb->exec, g, 0), "cudaGraphInstantiate");
  if (s != HXB_OK) {
    destroy_graph(cb);
    return s;
  }
  cb->last_resolved = ptrs;
  return HXB_OK;
}

// ------------------------------------------------------- the b200 factory
const hxb_hal_driver_info_t kB200DriverInfo = {
    {"b200", 4}, {"NVIDIA B200 (sm_100a) CUDA driver", 33}};

hxb_status_t env_u64(const char* name, uint64_t lo, uint64_t hi, uint64_t* out, bool* set) {
  *set = false;
  const char* v = getenv(name);
  if (!v || !*v) return HXB_OK;
  char* end = nullptr;
  const unsigned long long x = strtoull(v, &end, 10);
  if (*end != '\0' || v[0] == '-' || x < lo || x > hi)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "%s='%s' is not a decimal in [%llu, %llu]", name, v,
                (unsigned long long)lo, (unsigned long long)hi);
  *out = x;
  *set = true;
  return HXB_OK;
}

hxb_status_t b200_enumerate(void*, size_t* count, const hxb_hal_driver_info_t** infos) {
  *count = 1;
  *infos = &kB200DriverInfo;
  return HXB_OK;
}

hxb_status_t b200_try_create(void*, hxb_string_view_t name, hxb_allocator_t alloc,
                             hxb_hal_driver_t** out) {
  if (to_string(name) != "b200")
    return fail(HXB_STATUS_UNAVAILABLE, "no driver '%s' is provided by this factory",
                to_string(name).c_str());
  hxb_hal_driver_options_t o;
  hxb_hal_driver_options_initialize(&o);
  bool set = false;
  uint64_t v = 0;
  hxb_status_t s = env_u64("HXB_HAL_SCRATCH_BYTES", 4096, 1ull << 40, &v, &set);
  if (s != HXB_OK) return s;
  if (set) o.default_device_options.scratch_bytes = v;
  s = env_u64("HXB_HAL_QUEUE_WAIT_TIMEOUT_MS", 1,
              HXB_HAL_MAX_QUEUE_WAIT_TIMEOUT_NS / 1000000ull, &v, &set);
  if (s != HXB_OK) return s;
  if (set) o.default_device_options.queue_wait_timeout_ns = v * 1000000ull;
  return hxb_hal_driver_create(name, &o, alloc, out);
}

}  // namespace

struct hxb_hal_driver_registry_s {
  hxb_allocator_t allocator{};
  std::vector<const hxb_hal_driver_factory_t*> factories;
};

extern "C" {

void hxb_hal_device_options_initialize(hxb_hal_device_options_t* o) {
  if (!o) return;
  o->scratch_bytes = 0;
  o->queue_wait_timeout_ns = HXB_HAL_DEFAULT_QUEUE_WAIT_TIMEOUT_NS;
}

void hxb_hal_driver_options_initialize(hxb_hal_driver_options_t* o) {
  if (!o) return;
  hxb_hal_device_options_initialize(&o->default_device_options);
}

hxb_status_t hxb_hal_driver_create(hxb_string_view_t identifier,
                                   const hxb_hal_driver_options_t* options,
                                   hxb_allocator_t host_allocator, hxb_hal_driver_t** out_driver) {
  if (!out_driver) return fail(HXB_STATUS_INVALID_ARGUMENT, "driver_create: null out_driver");
  *out_driver = nullptr;
  hxb_hal_driver_t* d = host_new<hxb_hal_driver_s>(host_allocator);
  if (!d) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "driver_create: out of host memory");
  d->allocator = host_allocator;
  d->identifier = identifier.size ? to_string(identifier) : "b200";
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

hxb_status_t hxb_hal_driver_query_available_devices(hxb_hal_driver_t* driver,
                                                    hxb_hal_device_info_t* infos,
                                                    int32_t capacity, int32_t* out_count) {
  if (!driver || !out_count || capacity < 0 || (capacity > 0 && !infos))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "query_available_devices: bad arguments");
  int32_t n = 0;
  hxb_status_t s = hxb_hal_driver_query_device_count(driver, &n);
  if (s != HXB_OK) return s;
  for (int32_t i = 0; i < n && i < capacity; ++i) {
    hxb_hal_device_info_t& info = infos[i];
    memset(&info, 0, sizeof(info));
    info.device_id = (uint64_t)i;
    snprintf(info.path, sizeof(info.path), "cuda:%d", i);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, i) == cudaSuccess)
      snprintf(info.name, sizeof(info.name), "%s", prop.name);
    else
      cudaGetLastError();
  }
  *out_count = n;
  return HXB_OK;
}

hxb_status_t hxb_hal_driver_create_device_by_id(
    hxb_hal_driver_t* driver, uint64_t device_id,
    const hxb_hal_device_create_params_t* create_params, hxb_allocator_t host_allocator,
    hxb_hal_device_t** out_device) {
  if (!driver) return fail(HXB_STATUS_INVALID_ARGUMENT, "create_device_by_id: null driver");
  if (device_id > 0x7fffffffull)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "create_device_by_id: id %llu out of range",
                (unsigned long long)device_id);
  hxb_string_view_t id{driver->identifier.data(), driver->identifier.size()};
  return hxb_hal_device_create(id, (hxb_hal_domain_id_t)device_id,
                               &driver->options.default_device_options, create_params,
                               host_allocator, out_device);
}

void hxb_hal_driver_release(hxb_hal_driver_t* driver) {
  if (driver) host_delete(hxb_allocator_t(driver->allocator), driver);
}

hxb_status_t hxb_hal_device_create(hxb_string_view_t identifier, hxb_hal_domain_id_t domain_id,
                                   const hxb_hal_device_options_t* options,
                                   const hxb_hal_device_create_params_t* create_params,
                                   hxb_allocator_t host_allocator,
                                   hxb_hal_device_t** out_device) {
  if (!out_device) return fail(HXB_STATUS_INVALID_ARGUMENT, "device_create: null out_device");
  *out_device = nullptr;
  if (create_params && create_params->flags != 0)
    return fail(HXB_STATUS_UNSUPPORTED, "device_create: create_params flags 0x%llx unsupported",
                (unsigned long long)create_params->flags);
  hxb_hal_device_options_t o;
  hxb_hal_device_options_initialize(&o);
  if (options) o = *options;
  if (o.queue_wait_timeout_ns == 0) o.queue_wait_timeout_ns = HXB_HAL_DEFAULT_QUEUE_WAIT_TIMEOUT_NS;
  if (o.queue_wait_timeout_ns > HXB_HAL_MAX_QUEUE_WAIT_TIMEOUT_NS)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "device_create: queue wait bound %llu ns exceeds the %llu ns maximum",
                (unsigned long long)o.queue_wait_timeout_ns,
                (unsigned long long)HXB_HAL_MAX_QUEUE_WAIT_TIMEOUT_NS);
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || domain_id < 0 || domain_id >= n) {
    cudaGetLastError();
    return fail(HXB_STATUS_INVALID_ARGUMENT, "device_create: no CUDA device %d (%d present)",
                (int)domain_id, n);
  }
  hxb_hal_device_t* d = host_new<hxb_hal_device_s>(host_allocator);
  if (!d) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "device_create: out of host memory");
  d->allocator = host_allocator;
  d->identifier = identifier.size ? to_string(identifier) : "b200";
  d->ordinal = domain_id;
  d->wait_timeout_ns = o.queue_wait_timeout_ns;
  hxb_status_t s = use_device(d);
  hxb::DeviceInfo* info = nullptr;
  // resolve the per-device state of the dispatch library now, outside any
  // stream capture: the status word and the no-allocation scratch
  if (s == HXB_OK) s = hxb::current_device(&info);
  if (s == HXB_OK) s = hxb::noalloc_prepare_current_device();
  if (s == HXB_OK) {
    d->status_word = info->status_word;
    s = cuda_status(cudaStreamCreateWithFlags(&d->queue, cudaStreamNonBlocking),
                    "cudaStreamCreate");
  }
  if (s == HXB_OK) {
    d->scratch_bytes =
        o.scratch_bytes ? o.scratch_bytes : hxb::w8_streamk_workspace_bytes(info->num_sms);
    s = cuda_status(cudaMalloc(&d->scratch, d->scratch_bytes), "cudaMalloc(scratch)");
  }
  if (s == HXB_OK) s = cuda_status(cudaMemset(d->scratch, 0, d->scratch_bytes), "cudaMemset");
  if (s == HXB_OK) {
    void* h = nullptr;
    s = cuda_status(cudaHostAlloc(&h, sizeof(int), cudaHostAllocMapped), "cudaHostAlloc(lost)");
    if (s == HXB_OK) {
      d->lost_host = static_cast<int*>(h);
      __atomic_store_n(d->lost_host, 0, __ATOMIC_RELEASE);
      void* dp = nullptr;
      s = cuda_status(cudaHostGetDevicePointer(&dp, h, 0), "cudaHostGetDevicePointer(lost)");
      d->lost_dev = static_cast<int*>(dp);
    }
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
    // bounded: every wait the queue holds ends within wait_timeout_ns
    if (d->queue) cudaStreamSynchronize(d->queue);
    if (d->scratch) cudaFree(d->scratch);
    if (d->queue) cudaStreamDestroy(d->queue);
    if (d->lost_host) cudaFreeHost(d->lost_host);
  }
  host_delete(hxb_allocator_t(d->allocator), d);
}

void* hxb_hal_device_queue_stream(hxb_hal_device_t* d) { return d ? (void*)d->queue : nullptr; }

int hxb_hal_device_is_lost(hxb_hal_device_t* d) {
  return d && d->lost_host ? __atomic_load_n(d->lost_host, __ATOMIC_ACQUIRE) : 0;
}

// ------------------------------------------------------------ registry
hxb_status_t hxb_hal_driver_registry_create(hxb_allocator_t host_allocator,
                                            hxb_hal_driver_registry_t** out) {
  if (!out) return fail(HXB_STATUS_INVALID_ARGUMENT, "registry_create: null out");
  *out = nullptr;
  hxb_hal_driver_registry_t* r = host_new<hxb_hal_driver_registry_s>(host_allocator);
  if (!r) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "registry_create: out of host memory");
  r->allocator = host_allocator;
  *out = r;
  return HXB_OK;
}

void hxb_hal_driver_registry_release(hxb_hal_driver_registry_t* r) {
  if (r) host_delete(hxb_allocator_t(r->allocator), r);
}

hxb_status_t hxb_hal_driver_registry_register_factory(hxb_hal_driver_registry_t* r,
                                                      const hxb_hal_driver_factory_t* f) {
  if (!r || !f || !f->enumerate || !f->try_create)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "register_factory: null registry or factory");
  for (const hxb_hal_driver_factory_t* g : r->factories)
    if (g == f) return fail(HXB_STATUS_ALREADY_EXISTS, "register_factory: already registered");
  r->factories.push_back(f);
  return HXB_OK;
}

hxb_status_t hxb_hal_driver_registry_enumerate(hxb_hal_driver_registry_t* r,
                                               hxb_hal_driver_info_t* infos, int32_t capacity,
                                               int32_t* out_count) {
  if (!r || !out_count || capacity < 0 || (capacity > 0 && !infos))
    return fail(HXB_STATUS_INVALID_ARGUMENT, "registry_enumerate: bad arguments");
  int32_t n = 0;
  for (const hxb_hal_driver_factory_t* f : r->factories) {
    size_t count = 0;
    const hxb_hal_driver_info_t* list = nullptr;
    hxb_status_t s = f->enumerate(f->self, &count, &list);
    if (s != HXB_OK) return s;
    for (size_t i = 0; i < count; ++i, ++n)
      if (n < capacity) infos[n] = list[i];
  }
  *out_count = n;
  return HXB_OK;
}

hxb_status_t hxb_hal_driver_registry_try_create(hxb_hal_driver_registry_t* r,
                                                hxb_string_view_t name,
                                                hxb_allocator_t host_allocator,
                                                hxb_hal_driver_t** out) {
  if (!r || !out) return fail(HXB_STATUS_INVALID_ARGUMENT, "registry_try_create: null");
  *out = nullptr;
  for (const hxb_hal_driver_factory_t* f : r->factories) {
    size_t count = 0;
    const hxb_hal_driver_info_t* list = nullptr;
    hxb_status_t s = f->enumerate(f->self, &count, &list);
    if (s != HXB_OK) return s;
    for (size_t i = 0; i < count; ++i)
      if (to_string(list[i].driver_name) == to_string(name))
        return f->try_create(f->self, name, host_allocator, out);
  }
  return fail(HXB_STATUS_UNAVAILABLE, "no registered factory provides driver '%s'",
              to_string(name).c_str());
}

hxb_status_t hxb_hal_driver_module_register(hxb_hal_driver_registry_t* registry) {
  static const hxb_hal_driver_factory_t factory = {nullptr, b200_enumerate, b200_try_create};
  return hxb_hal_driver_registry_register_factory(registry, &factory);
}

// ------------------------------------------------------------- buffers
hxb_status_t hxb_hal_buffer_allocate(hxb_hal_device_t* d, uint64_t bytes,
                                     hxb_hal_buffer_t** out) {
  if (!d || !out || bytes == 0) return fail(HXB_STATUS_INVALID_ARGUMENT, "buffer_allocate: bad args");
  *out = nullptr;
  hxb_status_t s = use_device(d);
  if (s != HXB_OK) return s;
  hxb_hal_buffer_t* b = host_new<hxb_hal_buffer_s>(d->allocator);
  if (!b) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "buffer_allocate: out of host memory");
  b->device = d;
  b->bytes = bytes;
  if ((s = cuda_status(cudaMalloc(&b->ptr, bytes), "cudaMalloc(buffer)")) != HXB_OK) {
    host_delete(d->allocator, b);
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
  hxb_hal_device_t* d = b->device;
  if (use_device(d) == HXB_OK) {
    cudaStreamSynchronize(d->queue);
    cudaFree(b->ptr);
  }
  host_delete(d->allocator, b);
}

// ---------------------------------------------------------- semaphores
hxb_status_t hxb_hal_semaphore_create(hxb_hal_device_t* d, uint64_t initial,
                                      hxb_hal_semaphore_t** out) {
  if (!d || !out) return fail(HXB_STATUS_INVALID_ARGUMENT, "semaphore_create: null");
  *out = nullptr;
  hxb_status_t s = use_device(d);
  if (s != HXB_OK) return s;
  hxb_hal_semaphore_t* sem = host_new<hxb_hal_semaphore_s>(d->allocator);
  if (!sem) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "semaphore_create: out of host memory");
  sem->device = d;
  void* h = nullptr;
  if ((s = cuda_status(cudaHostAlloc(&h, sizeof(uint64_t), cudaHostAllocMapped),
                       "cudaHostAlloc(semaphore)")) != HXB_OK) {
    host_delete(d->allocator, sem);
    return s;
  }
  sem->host = static_cast<uint64_t*>(h);
  __atomic_store_n(sem->host, initial, __ATOMIC_RELEASE);
  void* dp = nullptr;
  if ((s = cuda_status(cudaHostGetDevicePointer(&dp, h, 0), "cudaHostGetDevicePointer")) !=
      HXB_OK) {
    cudaFreeHost(h);
    host_delete(d->allocator, sem);
    return s;
  }
  sem->dev = static_cast<uint64_t*>(dp);
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
  hxb_hal_device_t* d = sem->device;
  if (use_device(d) == HXB_OK) {
    cudaStreamSynchronize(d->queue);
    cudaFreeHost(sem->host);
  }
  host_delete(d->allocator, sem);
}

// ------------------------------------------------------ command buffers
hxb_status_t hxb_hal_command_buffer_create(hxb_hal_device_t* d, uint32_t binding_capacity,
                                           hxb_hal_command_buffer_t** out) {
  if (!d || !out) return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_create: null");
  *out = nullptr;
  hxb_hal_command_buffer_t* cb = host_new<hxb_hal_command_buffer_s>(d->allocator);
  if (!cb) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "command_buffer_create: out of host memory");
  cb->device = d;
  cb->binding_capacity = binding_capacity;
  *out = cb;
  return HXB_OK;
}

hxb_status_t hxb_hal_command_buffer_begin(hxb_hal_command_buffer_t* cb) {
  if (!cb) return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_begin: null");
  if (cb->state == kCbRecording)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_begin: already recording");
  if (use_device(cb->device) == HXB_OK) destroy_graph(cb);
  cb->commands.clear();
  cb->indirect = false;
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
  // exports read up to 11 constants; missing ones read as 0
  if (r.constants.size() < 16) r.constants.resize(16, 0u);
  for (uint32_t i = 0; i < binding_count; ++i) {
    const hxb_hal_buffer_ref_t& b = bindings[i];
    if (b.buffer) {
      if (b.buffer->device != cb->device || b.offset > b.buffer->bytes ||
          b.length > b.buffer->bytes - b.offset)
        return fail(HXB_STATUS_INVALID_ARGUMENT,
                    "command_buffer_dispatch: binding %u is not a range of a buffer of this "
                    "device",
                    i);
    } else if (b.buffer_slot >= cb->binding_capacity) {
      return fail(HXB_STATUS_INVALID_ARGUMENT,
                  "command_buffer_dispatch: binding %u names table slot %u, but the command "
                  "buffer's binding capacity is %u",
                  i, b.buffer_slot, cb->binding_capacity);
    } else {
      cb->indirect = true;
    }
    r.refs.push_back(Ref{b.buffer, b.buffer_slot, b.offset, b.length});
  }
  cb->commands.push_back(std::move(r));
  return HXB_OK;
}

hxb_status_t hxb_hal_command_buffer_end(hxb_hal_command_buffer_t* cb) {
  if (!cb || cb->state != kCbRecording)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_end: not recording");
  hxb_status_t s = use_device(cb->device);
  if (s != HXB_OK) return s;
  if (!cb->indirect) {
    std::vector<void*> ptrs;
    std::vector<size_t> lengths;
    s = resolve(cb, nullptr, &ptrs, &lengths);
    if (s == HXB_OK) s = install(cb, ptrs, lengths);
    if (s != HXB_OK) {
      destroy_graph(cb);
      cb->state = kCbInitial;
      return s;
    }
  }
  cb->state = kCbExecutable;
  return HXB_OK;
}

void hxb_hal_command_buffer_release(hxb_hal_command_buffer_t* cb) {
  if (!cb) return;
  hxb_hal_device_t* d = cb->device;
  if (use_device(d) == HXB_OK) {
    cudaStreamSynchronize(d->queue);  // bounded, see hxb_hal_device_release
    destroy_graph(cb);
  }
  host_delete(d->allocator, cb);
}

hxb_status_t hxb_hal_device_queue_execute(hxb_hal_device_t* d, hxb_hal_semaphore_t* wait_sem,
                                          uint64_t wait_value, hxb_hal_command_buffer_t* cb,
                                          const hxb_hal_buffer_binding_table_t* table,
                                          hxb_hal_semaphore_t* signal_sem,
                                          uint64_t signal_value) {
  if (!d || (cb && (cb->device != d || cb->state != kCbExecutable)) ||
      (wait_sem && wait_sem->device != d) || (signal_sem && signal_sem->device != d))
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "queue_execute: command buffer not ended, or objects of another device");
  if (hxb_hal_device_is_lost(d))
    return fail(HXB_STATUS_DEVICE_TIMEOUT,
                "queue_execute: device lost (an earlier queue wait ran out after %llu ns)",
                (unsigned long long)d->wait_timeout_ns);
  hxb_status_t s = use_device(d);
  if (s != HXB_OK) return s;
  if (cb && cb->indirect) {
    // table slots: (re)capture when the addresses differ from the last ones
    std::vector<void*> ptrs;
    std::vector<size_t> lengths;
    if ((s = resolve(cb, table, &ptrs, &lengths)) != HXB_OK) return s;
    if (!cb->exec || ptrs != cb->last_resolved) {
      // the update applies to later launches only; earlier ones keep theirs
      if ((s = install(cb, ptrs, lengths)) != HXB_OK) return s;
    }
  }
  if (wait_sem && load_acquire(wait_sem->host) < wait_value) {
    queue_wait_kernel<<<1, 1, 0, d->queue>>>(
        reinterpret_cast<const volatile unsigned long long*>(wait_sem->dev),
        (unsigned long long)wait_value, (unsigned long long)d->wait_timeout_ns, d->status_word,
        d->lost_dev);
    if ((s = cuda_status(cudaGetLastError(), "queue_execute: wait launch")) != HXB_OK) return s;
  }
  if (cb && (s = cuda_status(cudaGraphLaunch(cb->exec, d->queue), "cudaGraphLaunch")) != HXB_OK)
    return s;
  if (signal_sem) {
    queue_signal_kernel<<<1, 1, 0, d->queue>>>(
        reinterpret_cast<volatile unsigned long long*>(signal_sem->dev),
        (unsigned long long)signal_value, d->lost_dev);
    if ((s = cuda_status(cudaGetLastError(), "queue_execute: signal launch")) != HXB_OK) return s;
  }
  return HXB_OK;
}

// ------------------------------------------------------------- channels
hxb_status_t hxb_hal_channel_id_create(uint8_t* out_id) {
  if (!out_id) return fail(HXB_STATUS_INVALID_ARGUMENT, "channel_id_create: null id");
  const Nccl& n = nccl();
  if (!n.ok) return fail(HXB_STATUS_UNAVAILABLE, "channel_id_create: libnccl.so.2 not found");
  ncclUniqueId id;
  const ncclResult_t r = n.get_unique_id(&id);
  if (r != ncclSuccess)
    return fail(HXB_STATUS_CUDA_ERROR, "ncclGetUniqueId: %s", n.error_string(r));
  static_assert(sizeof(id) == HXB_HAL_CHANNEL_ID_BYTES, "NCCL unique id size");
  memcpy(out_id, &id, sizeof(id));
  return HXB_OK;
}

hxb_status_t hxb_hal_channel_create(hxb_hal_device_t* d, const uint8_t* id, int32_t rank,
                                    int32_t count, uint64_t timeout_ns,
                                    hxb_hal_channel_t** out) {
  if (!d || !id || !out || count < 1 || rank < 0 || rank >= count || timeout_ns == 0)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "channel_create: bad arguments");
  *out = nullptr;
  const Nccl& n = nccl();
  if (!n.ok) return fail(HXB_STATUS_UNAVAILABLE, "channel_create: libnccl.so.2 not found");
  hxb_status_t s = use_device(d);
  if (s != HXB_OK) return s;
  hxb_hal_channel_t* ch = host_new<hxb_hal_channel_s>(d->allocator);
  if (!ch) return fail(HXB_STATUS_RESOURCE_EXHAUSTED, "channel_create: out of host memory");
  ch->device = d;
  ch->rank = rank;
  ch->count = count;
  ch->timeout_ns = timeout_ns;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  // non-blocking initialisation, so a rank that never joins ends in a
  // timeout instead of a hang
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = n.comm_init_rank_config(&ch->comm, count, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    host_delete(d->allocator, ch);
    return fail(HXB_STATUS_CUDA_ERROR, "ncclCommInitRankConfig: %s", n.error_string(r));
  }
  s = nccl_settle(ch->comm, r, timeout_ns, "channel_create");
  if (s != HXB_OK) {
    n.comm_abort(ch->comm);
    host_delete(d->allocator, ch);
    return s;
  }
  *out = ch;
  return HXB_OK;
}

int32_t hxb_hal_channel_rank(hxb_hal_channel_t* ch) { return ch ? ch->rank : -1; }
int32_t hxb_hal_channel_count(hxb_hal_channel_t* ch) { return ch ? ch->count : 0; }

void hxb_hal_channel_release(hxb_hal_channel_t* ch) {
  if (!ch) return;
  hxb_hal_device_t* d = ch->device;
  const Nccl& n = nccl();
  if (use_device(d) == HXB_OK) {
    cudaStreamSynchronize(d->queue);  // bounded, see hxb_hal_device_release
    ncclResult_t r = n.comm_finalize(ch->comm);
    if (nccl_settle(ch->comm, r, ch->timeout_ns, "channel_release") == HXB_OK)
      n.comm_destroy(ch->comm);
    else
      n.comm_abort(ch->comm);
  }
  host_delete(d->allocator, ch);
}

hxb_status_t hxb_hal_command_buffer_collective(hxb_hal_command_buffer_t* cb,
                                               hxb_hal_channel_t* ch,
                                               hxb_hal_collective_op_t op,
                                               hxb_dtype_t element_type,
                                               hxb_hal_buffer_ref_t send,
                                               hxb_hal_buffer_ref_t recv,
                                               uint64_t element_count) {
  if (!cb || cb->state != kCbRecording)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_collective: not recording");
  if (!ch || ch->device != cb->device)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "command_buffer_collective: the channel belongs to another device");
  if (op < HXB_HAL_COLLECTIVE_ALL_GATHER || op > HXB_HAL_COLLECTIVE_BROADCAST ||
      (element_type != HXB_DTYPE_F16 && element_type != HXB_DTYPE_F32 &&
       element_type != HXB_DTYPE_I8) ||
      element_count == 0)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "command_buffer_collective: bad op, type or count");
  const uint64_t esz = element_type == HXB_DTYPE_F32 ? 4 : element_type == HXB_DTYPE_F16 ? 2 : 1;
  const uint64_t n = element_count * esz, g = n * (uint64_t)ch->count;
  const uint64_t send_need = op == HXB_HAL_COLLECTIVE_REDUCE_SCATTER_SUM ? g : n;
  const uint64_t recv_need = op == HXB_HAL_COLLECTIVE_ALL_GATHER ? g : n;
  if (send.length < send_need || recv.length < recv_need)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "command_buffer_collective: send needs %llu bytes and recv %llu, got %llu / %llu",
                (unsigned long long)send_need, (unsigned long long)recv_need,
                (unsigned long long)send.length, (unsigned long long)recv.length);
  Recorded r;
  r.ordinal = kCollective;
  r.channel = ch;
  r.op = op;
  r.dtype = element_type;
  r.count = element_count;
  for (const hxb_hal_buffer_ref_t* b : {&send, &recv}) {
    if (b->buffer) {
      if (b->buffer->device != cb->device || b->offset > b->buffer->bytes ||
          b->length > b->buffer->bytes - b->offset)
        return fail(HXB_STATUS_INVALID_ARGUMENT,
                    "command_buffer_collective: a binding is not a range of a buffer of this "
                    "device");
    } else if (b->buffer_slot >= cb->binding_capacity) {
      return fail(HXB_STATUS_INVALID_ARGUMENT,
                  "command_buffer_collective: table slot %u beyond the binding capacity %u",
                  b->buffer_slot, cb->binding_capacity);
    } else {
      cb->indirect = true;
    }
    r.refs.push_back(Ref{b->buffer, b->buffer_slot, b->offset, b->length});
  }
  cb->commands.push_back(std::move(r));
  return HXB_OK;
}

}  // extern "C"
