// tmem.cuh -- Tensor Memory (TMEM) as per-thread scratch on sm_100a.
//
// Each SM has 512 columns x 128 lanes of 32-bit TMEM. A CTA allocates a power-of-two number of
// columns (>= 32) once, from one warp; warp w may then read and write lanes [32 (w % 4), +32) of
// every allocated column, i.e. each of its threads owns one lane ("row") of the allocation. The
// accesses used here are the 32x32b shapes: thread i of the warp moves N consecutive columns of
// lane 32 (w % 4) + i to or from N registers. Loads and stores are asynchronous: tcgen05.wait::ld
// makes earlier loads' registers valid, tcgen05.wait::st completes earlier stores. The destination
// registers of a load must not be read before its wait: code placed between the two must leave
// them alone, and under register pressure the compiler may move or spill them (reading them
// early), so waits follow loads closely.
//
// Kernels using this keep co-resident CTAs x columns <= 512, so an allocation never waits, and
// free their columns (from the allocating warp) before the CTA exits.
#pragma once

#include <stdint.h>

namespace mb200 {

// Warp-wide: allocate ncols columns; the TMEM address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(d), "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// Warp-wide (the allocating warp): free the allocation.
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Order TMEM accesses before / after a thread barrier.
__device__ __forceinline__ void tmem_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Address of column `col` of this warp's lane quarter.
__device__ __forceinline__ uint32_t tmem_lane_addr(uint32_t base, int warp, int col) {
  return base + (static_cast<uint32_t>((warp & 3) * 32) << 16) + static_cast<uint32_t>(col);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld2(uint32_t taddr, float& a, float& b) {
  uint32_t x, y;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(x), "=r"(y) : "r"(taddr) : "memory");
  a = __uint_as_float(x);
  b = __uint_as_float(y);
}

__device__ __forceinline__ void tmem_st2(uint32_t taddr, float a, float b) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr), "r"(__float_as_uint(a)),
               "r"(__float_as_uint(b))
               : "memory");
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, const float* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3]))
               : "memory");
}

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float* v) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}

// K consecutive columns (K a multiple of 4) from / to v[0..K).
template <int K>
__device__ __forceinline__ void tmem_st_n(uint32_t taddr, const float (&v)[K]) {
#pragma unroll
  for (int i = 0; i < K; i += 4) tmem_st4(taddr + i, v + i);
}
template <int K>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, float (&v)[K]) {
#pragma unroll
  for (int i = 0; i < K; i += 4) tmem_ld4(taddr + i, v + i);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}

// Warp-wide: 16 lanes x 16 columns starting at TMEM address taddr (whose lane field selects the
// first of the 16 lanes) into 8 registers per thread, spread across threads (shape 16x256b, .x2).
// Thread t receives, with r = lane (taddr) + t / 4 and c = 2 (t % 4):
//   v[0], v[1] = (r, c), (r, c + 1)          v[2], v[3] = (r + 8, c), (r + 8, c + 1)
//   v[4], v[5] = (r, c + 8), (r, c + 9)      v[6], v[7] = (r + 8, c + 8), (r + 8, c + 9)
// (checked on a B200 by storing lane * 100 + column with 32x32b and reading it back this way).
// The first 8 columns only (shape 16x256b, .x1): v[0..3] as above.
__device__ __forceinline__ void tmem_ld16x256b_x1(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x1.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld16x256b_x2(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace mb200
