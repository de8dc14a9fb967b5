// Host-side helpers shared by the dispatch launchers: status codes, the
// per-device facts the launchers need (SM count, device status word) and
// TMA descriptor encoding through the driver entry point (no -lcuda link).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "hxb200.h"

namespace hxb {

// Maps a CUDA runtime error to the C-ABI status and remembers its text for
// hxb_last_error_message().
hxb_status_t cuda_status(cudaError_t e, const char* where);
hxb_status_t fail(hxb_status_t code, const char* fmt, ...);

// Launches `kernel` with programmatic stream serialization: it may start while
// the previous kernel of `stream` runs, and must order its dependent accesses
// with pdl_wait() (sm100.cuh).
template <typename... KArgs, typename... Args>
hxb_status_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                        cudaStream_t stream, const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...), what);
}

struct DeviceInfo {
  int ordinal;
  int num_sms;
  int max_smem_optin;
  int* status_word;  // device address of this device's status word
};

// Cached per device; first call on a device resolves the status word's
// address (no allocation).
hxb_status_t current_device(DeviceInfo** out);

// Encodes a 2-D or 3-D tiled tensor map. dims/strides are innermost first;
// strides are in bytes and exclude the innermost (unit) stride.
hxb_status_t encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype,
                               int rank, const void* base,
                               const uint64_t* dims, const uint64_t* strides,
                               const uint32_t* box,
                               CUtensorMapSwizzle swizzle);

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

}  // namespace hxb
