// kq_common.cuh -- device helpers shared by the kq kernels (sm_100a).
//
// PTX wrappers for mbarriers, non-tensor bulk copies (cp.async.bulk, the TMA engine's 1-D form),
// L2 cache policies and programmatic dependent launch (griddepcontrol). Every wait on a barrier is
// bounded: after KQ_WAIT_LIMIT polls it records an error in the model's device error word and the
// caller unwinds, so a lost copy can never hang the GPU.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace kq {

// Device error word bits (read by the host after every synchronised call).
enum : int {
  KQ_DEV_ERR_WAIT_FULL = 1,     // a consumer gave up waiting for a weight stage
  KQ_DEV_ERR_WAIT_EMPTY = 2,    // the producer gave up waiting for a free stage
  KQ_DEV_ERR_DRAIN = 4,         // copies still in flight at exit after a failure
  KQ_DEV_ERR_BAD_TOKEN = 8,     // a token id outside [0, vocab) reached a kernel
  KQ_DEV_ERR_BAD_POS = 16,      // a position outside [0, ctx) reached a kernel
  KQ_DEV_ERR_GRID = 32,         // a software grid-barrier wait gave up
};

// Polls of mbarrier.try_wait before giving up. Each poll may suspend the thread for a
// hardware-chosen time; 1 << 26 polls is seconds, orders of magnitude above any real wait.
constexpr uint32_t KQ_WAIT_LIMIT = 1u << 26;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Arrive once; true when this arrival completed the barrier's current phase (it was the last).
__device__ __forceinline__ bool mbar_arrive_completes(uint64_t* bar, uint32_t cnt = 1) {
  uint64_t st;
  uint32_t ok;
  asm volatile("mbarrier.arrive.shared::cta.b64 %0, [%1], %2;" : "=l"(st) : "r"(smem_u32(bar)), "r"(cnt) : "memory");
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(smem_u32(bar)), "l"(st) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Non-blocking probe: true if the phase with this parity has completed. Unlike try_wait it never
// suspends the thread, so it suits loops that do other work between probes.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait; false (and the error bit set) if the phase never completed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int bit) {
  for (uint32_t it = 0; it < KQ_WAIT_LIMIT; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicOr(err, bit);
  return false;
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol) : "memory");
}

// Programmatic dependent launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(smem_u32(p)));
  return v;
}
__device__ __forceinline__ uint32_t lds32(const void* p) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ float h2f_bits(uint32_t h16) { return __half2float(__ushort_as_half((unsigned short)h16)); }

// Named barrier over `nthreads` (a multiple of 32) threads.
__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------------------ tracing
// Compile-time opt-in (-DKQ_TRACE): per-CTA %globaltimer stamps at phase boundaries of the decode
// kernels, written to a device buffer the host reads with kq_trace_read (kq_api.cu). Off by
// default; the product build contains no trace code.
constexpr int KQ_TRACE_LAUNCHES = 256, KQ_TRACE_CTAS = 1024, KQ_TRACE_POINTS = 12;
#ifdef KQ_TRACE
__device__ unsigned long long g_kq_trace[KQ_TRACE_LAUNCHES][KQ_TRACE_CTAS][KQ_TRACE_POINTS];
__device__ __forceinline__ void kq_trace(int launch, int point) {
  if (launch < 0 || launch >= KQ_TRACE_LAUNCHES) return;
  const int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  if (cta >= KQ_TRACE_CTAS) return;
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  g_kq_trace[launch][cta][point] = t;
}
#define KQ_TRACE_AT(launch, point) kq_trace((launch), (point))
#else
#define KQ_TRACE_AT(launch, point) ((void)0)
#endif

}  // namespace kq
