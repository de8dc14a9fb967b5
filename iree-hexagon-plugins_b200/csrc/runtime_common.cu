#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "runtime_common.h"
#include "sm100.cuh"

// One status word per device (a file-scope device variable exists once on
// every device that loads this library). Kernels OR error bits into it, e.g.
// when a wait timed out; hxb_device_status() reads and optionally clears it.
static __device__ int g_hxb_status_word;

namespace hxb {

static thread_local char t_last_error[512];

const char* last_error() { return t_last_error; }

hxb_status_t fail(hxb_status_t code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

hxb_status_t cuda_status(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return HXB_OK;
  return fail(HXB_STATUS_CUDA_ERROR, "%s: %s (%s)", where,
              cudaGetErrorString(e), cudaGetErrorName(e));
}

static constexpr int kMaxDevices = 64;
static DeviceInfo g_devices[kMaxDevices];
static bool g_device_ready[kMaxDevices];
static std::mutex g_device_mu;

hxb_status_t current_device(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return fail(HXB_STATUS_INVALID_ARGUMENT, "device ordinal %d out of range", dev);
  if (g_device_ready[dev]) {
    *out = &g_devices[dev];
    return HXB_OK;
  }
  std::lock_guard<std::mutex> lock(g_device_mu);
  if (!g_device_ready[dev]) {
    DeviceInfo d{};
    d.ordinal = dev;
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, dev)) != cudaSuccess)
      return cuda_status(e, "cudaGetDeviceProperties");
    if (prop.major != 10)
      return fail(HXB_STATUS_UNSUPPORTED,
                  "device %d is sm_%d%d; this library is built for sm_100a only",
                  dev, prop.major, prop.minor);
    d.num_sms = prop.multiProcessorCount;
    d.max_smem_optin = (int)prop.sharedMemPerBlockOptin;
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, g_hxb_status_word)) != cudaSuccess)
      return cuda_status(e, "cudaGetSymbolAddress(status word)");
    d.status_word = static_cast<int*>(p);
    g_devices[dev] = d;
    g_device_ready[dev] = true;
  }
  *out = &g_devices[dev];
  return HXB_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t,
                                  void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                         cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

hxb_status_t encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype,
                               int rank, const void* base,
                               const uint64_t* dims, const uint64_t* strides,
                               const uint32_t* box,
                               CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn)
    return fail(HXB_STATUS_CUDA_ERROR,
                "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t gdim[5], gstride[4];
  cuuint32_t bdim[5], estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstride[i] = strides[i];
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), gdim,
                  gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(HXB_STATUS_INVALID_ARGUMENT,
                "cuTensorMapEncodeTiled failed (CUresult %d): rank %d dims "
                "[%llu,%llu] box [%u,%u]",
                (int)r, rank, (unsigned long long)dims[0],
                (unsigned long long)dims[1], box[0], box[1]);
  return HXB_OK;
}

}  // namespace hxb

extern "C" const char* hxb_last_error_message(void) { return hxb::last_error(); }

extern "C" hxb_status_t hxb_device_status(int clear, int* out_bits) {
  hxb::DeviceInfo* d = nullptr;
  hxb_status_t s = hxb::current_device(&d);
  if (s != HXB_OK) return s;
  int bits = 0;
  cudaError_t e = cudaMemcpy(&bits, d->status_word, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return hxb::cuda_status(e, "read status word");
  if (clear && bits) {
    const int zero = 0;
    e = cudaMemcpy(d->status_word, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return hxb::cuda_status(e, "clear status word");
  }
  if (out_bits) *out_bits = bits;
  return HXB_OK;
}

extern "C" int hxb_abi_version(void) { return HXB_ABI_VERSION; }

// ---------------------------------------------------------------- CUDA IPC
// Peer buffers for the all-gather epilogue: a rank maps the other ranks'
// output buffers into ITS OWN device's context (the current device), with
// peer access enabled, so kernels running on that device can store into them
// over NVLink. Plain IPC mappings; no NVLink multicast objects.

extern "C" hxb_status_t hxb_ipc_get_handle(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset)
    return hxb::fail(HXB_STATUS_INVALID_ARGUMENT, "ipc_get_handle: null argument");
  // the handle names the whole allocation; report where ptr sits inside it
  typedef CUresult (*RangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
  static RangeFn range = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<RangeFn>(p);
  }();
  if (!range) return hxb::fail(HXB_STATUS_CUDA_ERROR, "ipc_get_handle: cuMemGetAddressRange missing");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return hxb::fail(HXB_STATUS_INVALID_ARGUMENT, "ipc_get_handle: not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return hxb::cuda_status(e, "cudaIpcGetMemHandle");
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return HXB_OK;
}

extern "C" hxb_status_t hxb_ipc_open(const void* handle, int64_t offset, void** ptr) {
  if (!handle || !ptr || offset < 0)
    return hxb::fail(HXB_STATUS_INVALID_ARGUMENT, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return hxb::cuda_status(e, "cudaIpcOpenMemHandle");
  // make sure the current device may access the owner's memory
  int cur = 0;
  cudaPointerAttributes attr;
  if (cudaGetDevice(&cur) == cudaSuccess && cudaPointerGetAttributes(&attr, base) == cudaSuccess &&
      attr.device != cur) {
    int can = 0;
    cudaDeviceCanAccessPeer(&can, cur, attr.device);
    if (!can) {
      cudaIpcCloseMemHandle(base);
      return hxb::fail(HXB_STATUS_UNSUPPORTED, "ipc_open: device %d cannot access device %d",
                       cur, attr.device);
    }
    e = cudaDeviceEnablePeerAccess(attr.device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
      cudaGetLastError();
    } else if (e != cudaSuccess) {
      cudaIpcCloseMemHandle(base);
      return hxb::cuda_status(e, "cudaDeviceEnablePeerAccess");
    }
  }
  *ptr = static_cast<uint8_t*>(base) + offset;
  return HXB_OK;
}

extern "C" hxb_status_t hxb_ipc_close(void* ptr, int64_t offset) {
  if (!ptr || offset < 0) return hxb::fail(HXB_STATUS_INVALID_ARGUMENT, "ipc_close: bad argument");
  return hxb::cuda_status(cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset),
                          "cudaIpcCloseMemHandle");
}

// ------------------------------------------------------- peer barrier
// One thread per peer: it stores `epoch` into the peer's flag array at this
// rank's slot (release, system scope: everything this rank's stream did
// before -- the fused epilogue's peer stores included -- is visible to a peer
// that acquires the flag), then waits, bounded, until the peer's arrival for
// this epoch lands in this rank's own flag array.
namespace {
constexpr int kMaxPeers = 8;
struct PeerFlags {
  unsigned int* p[kMaxPeers];  // each rank's flag array, this rank's own included
};

__global__ void peer_barrier_kernel(PeerFlags flags, int world, int rank, unsigned int epoch,
                                    unsigned long long limit_ns, int* status) {
  hxb::pdl_wait();
  const int t = threadIdx.x;
  if (t >= world || t == rank) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flags.p[t] + rank), "r"(epoch)
               : "memory");
  const unsigned int* mine = flags.p[rank] + t;
  const unsigned long long t0 = hxb::globaltimer_ns();
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if ((int)(v - epoch) >= 0) break;
    if (hxb::globaltimer_ns() - t0 > limit_ns) {
      atomicOr(status, hxb::kStatusTimeout);
      break;
    }
    __nanosleep(100);
  }
}
}  // namespace

extern "C" hxb_status_t hxb_peer_barrier(void* const* flags, int world, int rank,
                                         uint32_t epoch, void* stream) {
  if (!flags || world < 1 || world > kMaxPeers || rank < 0 || rank >= world || epoch == 0)
    return hxb::fail(HXB_STATUS_INVALID_ARGUMENT,
                     "peer_barrier: 1..%d ranks, a rank among them and an epoch > 0", kMaxPeers);
  PeerFlags f{};
  for (int i = 0; i < world; ++i) {
    if (!flags[i] || (reinterpret_cast<uintptr_t>(flags[i]) & 3u))
      return hxb::fail(HXB_STATUS_INVALID_ARGUMENT, "peer_barrier: flag array %d", i);
    f.p[i] = static_cast<unsigned int*>(flags[i]);
  }
  if (world == 1) return HXB_OK;
  hxb::DeviceInfo* dev = nullptr;
  hxb_status_t s = hxb::current_device(&dev);
  if (s != HXB_OK) return s;
  return hxb::launch_pdl(peer_barrier_kernel, dim3(1), dim3(32), 0,
                         static_cast<cudaStream_t>(stream), "peer barrier launch", f, world, rank,
                         (unsigned int)epoch, hxb::kWaitLimitNs, dev->status_word);
}
