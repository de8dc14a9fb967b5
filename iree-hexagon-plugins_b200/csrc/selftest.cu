// hxb_selftest_wait_timeout: runs, on purpose and on a short limit, the
// failure path every pipelined kernel of this library takes when one of its
// bounded waits runs out.
//
// The kernel has the roles of the GEMM and attention kernels -- a producer
// thread with a bulk copy in flight, a single-thread MMA issuer holding TMEM,
// and an epilogue warp -- and every role waits on an mbarrier that nothing
// ever arrives at, through the same mbar_wait_for the product kernels use
// (sm100.cuh). The first wait to run out raises the CTA's abort flag and ORs
// HXB_DEVICE_STATUS_TIMEOUT into the device status word; the other roles see
// the flag and stop; the producer then waits (bounded) for its own copy to
// land, and the TMEM owner frees its columns before the CTA exits. The host
// reads the status word with hxb_device_status() and the per-role outcome
// from `result`. No GPU fault is involved: the barrier is valid, the copy is
// in bounds, and every wait ends.
#include "runtime_common.h"
#include "sm100.cuh"

namespace hxb {
namespace {

constexpr uint32_t kCopyBytes = 4096;
constexpr uint32_t kTmemCols = 32;

// result[0]: waits that reported success (0 expected)
// result[1]: the CTA's abort flag after the roles stopped (1 expected)
// result[2]: 1 if the producer's bulk copy landed intact
// result[3]: 1 once TMEM was freed
__global__ void __launch_bounds__(96, 1)
    wait_timeout_kernel(const uint4* __restrict__ src, int* status,
                        unsigned long long limit_ns, int* result) {
  __shared__ __align__(128) uint8_t buf[kCopyBytes];
  __shared__ uint64_t loaded, never;
  __shared__ uint32_t tmem_holder;
  __shared__ int abort_word;
  __shared__ int successes;
  volatile int* abort_flag = &abort_word;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const FailState fs{abort_flag, status};

  if (threadIdx.x == 0) {
    mbar_init(&loaded, 1);
    mbar_init(&never, 1);
    *abort_flag = 0;
    successes = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_holder;

  if (warp == 0) {
    // producer: a real copy in flight, then a wait that never completes
    if (lane == 0) {
      mbar_arrive_expect_tx(&loaded, kCopyBytes);
      bulk_load_1d(buf, src, kCopyBytes, &loaded);
      if (mbar_wait_for(&never, 0, fs, limit_ns)) atomicAdd(&successes, 1);
      // failure path: never leave with a copy still landing in shared memory
      const unsigned long long t0 = globaltimer_ns();
      while (!mbar_try_wait(&loaded, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    }
  } else if (warp == 1) {
    // MMA issuer role: holds the TMEM allocation while it waits
    if (lane == 0 && mbar_wait_for(&never, 0, fs, limit_ns)) atomicAdd(&successes, 1);
  } else {
    // epilogue role: the whole warp waits and agrees before going on
    const bool ready = mbar_wait_for(&never, 0, fs, limit_ns);
    if (__all_sync(0xffffffffu, ready) && lane == 0) atomicAdd(&successes, 1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint4* got = reinterpret_cast<const uint4*>(buf);
    int intact = 1;
    for (uint32_t i = 0; i < kCopyBytes / 16; ++i) {
      const uint4 a = got[i], b = src[i];
      intact &= (a.x == b.x) & (a.y == b.y) & (a.z == b.z) & (a.w == b.w);
    }
    result[0] = successes;
    result[1] = *abort_flag;
    result[2] = intact;
    result[3] = 1;
  }
}

}  // namespace
}  // namespace hxb

extern "C" hxb_status_t hxb_selftest_wait_timeout(uint64_t limit_ns, const void* src,
                                                  int32_t* result, void* stream) {
  if (limit_ns == 0 || limit_ns > 1000000000ull)
    return hxb::fail(HXB_STATUS_INVALID_ARGUMENT,
                     "selftest_wait_timeout: limit %llu ns outside (0, 1 s]",
                     (unsigned long long)limit_ns);
  if (!src || !result || !hxb::aligned16(src))
    return hxb::fail(HXB_STATUS_INVALID_ARGUMENT,
                     "selftest_wait_timeout: src (16-byte aligned, 4096 bytes) and result "
                     "(4 int32) are required");
  hxb::DeviceInfo* dev = nullptr;
  hxb_status_t s = hxb::current_device(&dev);
  if (s != HXB_OK) return s;
  hxb::wait_timeout_kernel<<<1, 96, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), dev->status_word, (unsigned long long)limit_ns,
      reinterpret_cast<int*>(result));
  return hxb::cuda_status(cudaGetLastError(), "selftest_wait_timeout launch");
}
