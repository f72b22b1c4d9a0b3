// stage.cuh -- shared-memory staging with the bulk-copy (TMA) engine and mbarriers, sm_90+.
//
// One elected lane arms an mbarrier with the byte count it expects, the warp issues 1-D bulk
// copies (cp.async.bulk, no multicast) that complete on that mbarrier, and consumers wait on
// the barrier's phase. Every wait is bounded: after kMaxWaitRounds suspended try_wait rounds
// (~10 ms each) the waiter records kFaultWaitTimeout in g_mb200_fault and carries on with
// whatever is in shared memory, so a kernel can never hang on a copy that does not arrive.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mb200 {

constexpr int kFaultWaitTimeout = 1;
constexpr int kMaxWaitRounds = 256;       // x ~10 ms suspend hint -> ~2.5 s worst case
constexpr uint32_t kWaitHintNs = 10000000;

// Sticky device-side fault word. Each translation unit that includes this header owns its own
// copy (no relocatable device code); its host side reads and clears it through read_fault().
static __device__ int g_mb200_fault;

// Host side: copy this translation unit's fault word into *out and clear it (synchronous).
static inline cudaError_t read_fault_word(int* out) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_mb200_fault, sizeof(int));
  if (e != cudaSuccess) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_mb200_fault, &zero, sizeof(int));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make the initialised barriers visible to the async (bulk copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Arrive once and add `bytes` to the transaction count the current phase waits for.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before later async-proxy
// (bulk copy) writes to the same buffer.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Global -> shared bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned),
// completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Wait until the barrier phase with the given parity has completed; bounded (see above).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  for (int round = 0; round < kMaxWaitRounds; ++round) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity), "r"(kWaitHintNs)
        : "memory");
    if (done) return true;
  }
  atomicOr(&g_mb200_fault, kFaultWaitTimeout);
  return false;
}

}  // namespace mb200
