// sm_100a building blocks shared by the dispatch kernels: mbarriers with
// bounded waits, TMA tile loads (no multicast, ever), tcgen05 MMA / TMEM
// management and the shared-memory matrix descriptors the tensor core reads.
//
// These replace the Hexagon HMX primitives the reference lowers to
// (plugins/runtime/hexagon/dsp/ukernel/hmx/api.h:22-67): there is no pack
// step because TMA writes tiles straight into the 128B-swizzled layout that
// tcgen05.mma consumes, and the accumulator lives in TMEM in f32 instead of
// the HMX f16 read-out.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace hxb {

// Every spin-wait in every kernel gives up after this long, records an error
// in the caller-visible status word and lets the CTA wind down instead of
// hanging the GPU. Legitimate waits inside one launch are microseconds.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// Status bits written into the device status word on a failed wait.
constexpr int kStatusTimeout = 1;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------- programmatic dependent launch
// A kernel launched with launch_pdl (programmatic stream serialization) may be
// scheduled while the kernel before it in the stream still runs. It must call
// pdl_wait() before it reads anything that kernel (or any earlier one) writes,
// or writes anything they read; pdl_wait() returns once they have completed
// and their memory is visible. pdl_trigger() lets the next such kernel be
// scheduled as soon as every CTA of this grid has called it or exited; it
// does not let that kernel pass its own pdl_wait() before this grid ends.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Makes generic-proxy shared-memory writes visible to the async proxy (TMA
// and the tensor core read shared memory through it).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Per-CTA failure state: the first wait that times out raises `abort` in
// shared memory (so every role of the CTA stops waiting) and ORs
// kStatusTimeout into the launch's global status word.
struct FailState {
  volatile int* abort;  // shared memory
  int* status;          // global memory, may be null
};

__device__ __forceinline__ void raise_failure(const FailState& fs) {
  *fs.abort = 1;
  if (fs.status) atomicOr(fs.status, kStatusTimeout);
}

// Waits for the phase of `bar` with parity `parity` to complete. Returns false
// (after raising the failure state) when the wait exceeds `limit_ns` or when
// another role of this CTA already gave up.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity,
                                              const FailState& fs,
                                              unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*fs.abort) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      raise_failure(fs);
      return false;
    }
  }
}

// mbar_wait_for with the library-wide limit kWaitLimitNs (every kernel's
// waits go through this).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          const FailState& fs) {
  return mbar_wait_for(bar, parity, fs, kWaitLimitNs);
}

// mbar_wait for a barrier that other CTAs of the cluster arrive on
// (mbar_arrive_cluster): the completed phase is acquired at cluster scope.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  const FailState& fs) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*fs.abort) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_failure(fs);
      return false;
    }
  }
}

// Named barrier among `count` threads (a multiple of 32) of this CTA.
__device__ __forceinline__ void named_barrier_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ------------------------------------------------------------- clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster (release / acquire).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Arrives once on an mbarrier of any CTA of the cluster (address from
// map_to_rank), releasing this thread's prior accesses at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_addr)
               : "memory");
}

// --------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// 2-D tiled bulk tensor load into this CTA's shared memory; completion is
// signalled as transaction bytes on `bar`. x is the innermost coordinate.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map,
                                            uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Asks the TMA unit to bring a 2-D box of `map` into L2 (no shared-memory
// destination, no completion signal). x is the innermost coordinate. L2 is
// the device's point of coherence, so a prefetch issued before
// griddepcontrol.wait cannot make a later load see data older than the
// previous kernel's writes: those writes update the L2 line.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map),
               "r"(x), "r"(y)
               : "memory");
}

// CTA-pair forms (cta_group::2, no multicast): each CTA of the pair loads its
// own half of the operands into its own shared memory, and the completion is
// counted on `bar_addr`, an mbarrier that may live in the peer CTA (the pair's
// leader, whose thread issues the pair's MMAs).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_addr, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_addr), "r"(x), "r"(y)
      : "memory");
}
// --------------------------------------------------------------- tcgen05
// 2-D TMA store of a shared-memory box to global memory (bulk group of the
// issuing thread). x * element size must be a multiple of 16 bytes and both
// coordinates non-negative; the part of the box past the tensor is dropped.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   map),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until this thread's committed bulk stores have finished reading
// shared memory (the source may be overwritten).
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Waits until this thread's committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// 1-D bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// from global memory into this CTA's shared memory; completion is signalled as
// transaction bytes on `bar`.
__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes,
                                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Orders this thread's earlier generic-proxy accesses to global memory (an
// acquire of data another CTA published) before its later async-proxy ones
// (bulk copies of that data).
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols)
      : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}

// TMEM allocation shared by a CTA pair: one warp with the same warp index in
// each CTA of the pair issues it; both CTAs get the same column range.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols)
      : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (f16 or bf16 inputs,
// f32 accumulator). Issued by a single thread.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t adesc,
                                            uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16. A is read from TMEM: lane m
// holds row m, each 32-bit column two consecutive K elements (lower K index in
// the low half). Issued by a single thread.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem,
                                            uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread
// has completed (and its shared-memory operands may be overwritten).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}

// Pair MMA (issued by the leader CTA's thread): M = 256 rows, the leader's
// TMEM holds rows 0-127 and the peer's rows 128-255; A and B are read from
// the same shared-memory offsets in both CTAs (A split along M, B along N).
__device__ __forceinline__ void umma_f16_ss_pair(uint32_t d_tmem, uint64_t adesc,
                                                 uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on the mbarrier at `bar_addr` (this CTA's or the peer's, from
// map_to_rank) when every pair MMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_addr) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          bar_addr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Each thread of the warp reads 32 consecutive f32 columns of its own TMEM
// lane (lane = warp's quarter * 32 + lane id).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr,
                                                   uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Each thread writes 32 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr,
                                                   const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, "
      "%31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
      "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
      "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 2^x on the special-function unit (PTX ex2.approx, flush-to-zero).
// Per-warpgroup register reallocation: every warp of a warpgroup executes the
// same setmaxnreg. The counts after all increases must fit in the registers the
// block was launched with (threads x registers per thread at launch), or the
// increasing warps wait for good; callers check the launch count on the host.
template <int N>
__device__ __forceinline__ void reg_dealloc() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "setmaxnreg count");
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void reg_alloc() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "setmaxnreg count");
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------- packed f32 pairs (sm_100)
// Two f32 values in one 64-bit register pair, operated on by the f32x2
// instructions (one issue slot for both lanes).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}


__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr,
                                                   uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
}

// Each thread writes 16 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// Shared-memory matrix descriptor (tcgen05 "version 1" format):
//   [0,14)  start address >> 4
//   [16,30) leading-dimension byte offset >> 4
//   [32,46) stride-dimension byte offset >> 4
//   [46,48) version = 1
//   [61,64) layout: 0 none, 2 = 128-byte swizzle
// For a K-major 128B-swizzled operand the rows are 128 bytes of K and SBO is
// the distance between 8-row groups; for an MN-major one the 128-byte rows run
// along M/N, LBO steps between 64-element MN chunks and SBO between 8-row K
// groups.
constexpr uint32_t kLayoutSwizzle128 = 2;

__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo,
                                                   uint32_t sbo,
                                                   uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with f16 A/B and an f32 accumulator.
// a_mn / b_mn select MN-major (transposed) operands.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, int a_mn,
                                                      int b_mn) {
  return (1u << 4)                              // D format f32
         | (0u << 7) | (0u << 10)               // A, B format f16
         | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16)  // majors
         | ((uint32_t)(N >> 3) << 17)           // N / 8
         | ((uint32_t)(M >> 4) << 24);          // M / 16
}

// --------------------------------------------------------------- numerics
__device__ __forceinline__ uint32_t pack_half2(float x, float y) {
  __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}


}  // namespace hxb
