// hxb_matmul_f16_noalloc: the f16 matmul dispatch for callers that cannot
// allocate device memory.
//
// hxb_matmul_f16 needs device scratch when an operand's row pitch is not a
// multiple of 16 bytes: the operand is re-pitched into that scratch before the
// tcgen05 kernel reads it through TMA. Its caller passes the scratch in. Some
// callers have no way to get it: a compiled dispatch function runs with only
// the buffers its runtime bound to it and no allocator (the executable-library
// dispatch contract gives it bindings and push constants, nothing more), and
// code running while a stream is being captured must not call cudaMalloc. This
// entry point serves them from a scratch array that is part of the library
// image instead.
//
// The scratch is a file-scope __device__ array of HXB_NOALLOC_SCRATCH_BYTES
// (32 MiB, declared in hxb200.h); larger re-pitches are rejected. Every
// GPU on which the library is loaded holds it until the process exits. All
// calls on a device share it and it keeps the last call's contents, so calls
// whose execution overlaps on the GPU (different streams, or the same array
// reached from two threads) race on it; serialise them on one stream. Nothing
// in the scratch has to start at zero: the re-pitch copy writes every byte the
// kernel then reads (the tensor maps keep the operands' true extents, so the
// pad columns are never read).
//
// Set-up: the first call on a device (with that device current) resolves the
// device address of the array with cudaGetSymbolAddress and caches it with
// the id of the CUDA context it belongs to; a call that finds a different
// context current (the device was reset with cudaDeviceReset and its primary
// context re-created) resolves it again. In host code the array's name is
// only a host-side stand-in, never a device address, so the kernel is always
// given the resolved pointer. Make that first call on each device before any
// stream capture begins; a HAL device (hxb_hal_device_create) makes it when
// it is created. The stream must belong to the current device: the scratch
// is chosen by the current device, and a stream of another device is
// rejected.
#include <mutex>

#include "runtime_common.h"

namespace {

constexpr size_t kNoAllocScratchBytes = HXB_NOALLOC_SCRATCH_BYTES;  // 32 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
struct ScratchSlot {
  void* addr;
  unsigned long long ctx_id;  // context the address was resolved in
  bool ready;
};
ScratchSlot g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

template <class Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion(name, &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

// Id of the calling thread's current CUDA context, 0 if none is current.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of this device's scratch array, resolved once per device
// and context.
hxb_status_t scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return hxb::cuda_status(e, "matmul_f16_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return hxb::fail(HXB_STATUS_INVALID_ARGUMENT,
                     "matmul_f16_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& slot = g_scratch[dev];
  const unsigned long long ctx = slot.ready ? current_context_id() : 0;
  if (!slot.ready || ctx != slot.ctx_id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // also makes the context current
    if (e != cudaSuccess)
      return hxb::cuda_status(e, "matmul_f16_noalloc: cudaGetSymbolAddress(scratch)");
    slot.addr = p;
    slot.ctx_id = current_context_id();
    slot.ready = true;
  }
  *out = slot.addr;
  return HXB_OK;
}

}  // namespace

namespace hxb {
hxb_status_t noalloc_prepare_current_device() {
  void* p = nullptr;
  return scratch_for_current_device(&p);
}
}  // namespace hxb

namespace hxb {
// Defined in gemm.cu: the f16 dispatch behind hxb_matmul_f16.
hxb_status_t gemm_f16_impl(const void* A, int64_t lda, const void* B,
                           int64_t ldb, int transpose_b, const void* C_init,
                           void* C, int64_t ldc, hxb_dtype_t c_dtype, int64_t M,
                           int64_t N, int64_t K, void* workspace,
                           size_t workspace_bytes, cudaStream_t stream);
}  // namespace hxb

extern "C" hxb_status_t hxb_matmul_f16_noalloc(const void* A, int64_t lda, const void* B,
                                               int64_t ldb, int transpose_b,
                                               const void* C_init, void* C, int64_t ldc,
                                               hxb_dtype_t c_dtype, int64_t M, int64_t N,
                                               int64_t K, void* stream) {
  // Shape errors are reported by the shared dispatch path; the scratch size
  // is only meaningful for positive extents.
  if (M >= 1 && N >= 1 && K >= 1 && lda >= 1 && ldb >= 1) {
    const size_t need =
        hxb_matmul_f16_workspace_bytes(A, lda, B, ldb, transpose_b, M, N, K);
    if (need > kNoAllocScratchBytes)
      return hxb::fail(HXB_STATUS_INVALID_ARGUMENT,
                       "matmul_f16_noalloc: re-pitching these operands needs %zu bytes of "
                       "scratch but the built-in scratch holds %zu bytes; use "
                       "hxb_matmul_f16 with a workspace, or pass operands whose row "
                       "pitch is a multiple of 16 bytes (they need no scratch)",
                       need, kNoAllocScratchBytes);
  }
  // The stream's device is checked when the stream is not being captured (a
  // query of a capturing stream would invalidate the capture; a stream being
  // captured by this thread was made current-device work by its caller).
  int cur = 0, sdev = 0;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &cap) == cudaSuccess &&
      cap == cudaStreamCaptureStatusNone && cudaGetDevice(&cur) == cudaSuccess &&
      cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev) == cudaSuccess &&
      sdev != cur)
    return hxb::fail(HXB_STATUS_INVALID_ARGUMENT,
                     "matmul_f16_noalloc: the stream belongs to device %d, but device %d is "
                     "current (the built-in scratch is the current device's)",
                     sdev, cur);
  cudaGetLastError();
  void* scratch = nullptr;
  hxb_status_t s = scratch_for_current_device(&scratch);
  if (s != HXB_OK) return s;
  return hxb::gemm_f16_impl(A, lda, B, ldb, transpose_b, C_init, C, ldc, c_dtype, M, N,
                            K, scratch, kNoAllocScratchBytes,
                            static_cast<cudaStream_t>(stream));
}
