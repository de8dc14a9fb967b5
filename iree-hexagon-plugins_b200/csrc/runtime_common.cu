#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "runtime_common.h"

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
