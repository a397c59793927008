// PTX building blocks for sm_100a: shared-memory mbarriers, 1-D bulk copies (TMA engine without
// a tensor map), bounded waits and the library's device-side error word.
//
// Every wait here is bounded: after about a second of SM clock it gives up, records the reason
// in the error word and returns false, and the caller winds down instead of spinning forever.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fa {

// Limits of the launch argument tables (kernel parameters, up to 32 KB on sm_70 and later).
constexpr int kMaxEnds = 64;         // Mask::Groups ends per span
constexpr int kMaxBatchRows = 256;   // independent rows per attend launch

// About one second at the B200's 1.9 GHz SM clock.
constexpr long long kWaitCycles = 2000000000LL;

// Bits of the device error word every kernel receives (a per-device word the host reads and
// clears in fa_device_status).
constexpr unsigned kErrTimeout = 1u;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy and the other threads.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase of `bar` with parity `parity` to complete; after kWaitCycles it sets
// kErrTimeout in *err and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > kWaitCycles) {
      atomicOr(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from global to
// this CTA's shared memory; completes `bytes` transactions on `bar`.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// The same with an L2 eviction-priority policy (a createpolicy result).
__device__ __forceinline__ void bulk_g2s_hint(void* smem_dst, const void* gmem_src,
                                              uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// An L2 policy that evicts streamed data first (each K/V byte is read once per launch).
// Programmatic dependent launch: a kernel launched with programmatic stream serialization may
// start while the kernel before it in the stream still runs; pdl_wait() blocks the calling
// thread until that kernel has completed and its memory is visible (at once when there is no
// such kernel). pdl_trigger() lets the next kernel of the stream start early (a no-op when it
// was launched without the attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// Named barrier over `threads` threads (a multiple of 32) with id `id` (1..15).
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Named barrier that also ORs `pred` over the participating threads: every thread gets the same
// answer, so a decision taken on it (leaving a loop that holds further barriers) is uniform.
__device__ __forceinline__ bool named_sync_or(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(pred)), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

// Every thread of every CTA of the cluster arrives (release) and waits (acquire); hardware
// barrier, so every thread of the cluster must reach it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// A float of CTA `rank`'s shared memory at the address of `local` in this CTA's.
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// blockIdx.x read as a volatile special register: never merged with an earlier read, so a value
// derived from it is recomputed where it is needed instead of being held in a register.
__device__ __forceinline__ uint32_t ctaid_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%ctaid.x;" : "=r"(r));
  return r;
}

// max(a, b, c) in one instruction (sm_100a's three-input max).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float bf16_lo(uint32_t packed) {
  return __uint_as_float(packed << 16);
}
__device__ __forceinline__ float bf16_hi(uint32_t packed) {
  return __uint_as_float(packed & 0xFFFF0000u);
}

}  // namespace fa
