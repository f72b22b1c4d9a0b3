// common.cuh -- shared device helpers for the sm_100a selective-scan / conv1d kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "mamba_b200.h"

namespace mb200 {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kChunk = MB200_CHUNK;      // timesteps per chunk (chunk_states granularity)
constexpr int kMaxState = MB200_MAX_DSTATE;

// Staged B/C tile rows in shared memory: kChunk elements per row, stored as two halves. For 4-byte
// elements the second half starts 16 bytes later than contiguous, so the 8 time-segment lanes of
// a channel (each reading 16-byte pieces 32 bytes apart) fall in distinct banks.
template <typename T>
struct TileRow {
  static constexpr int kShift = sizeof(T) == 4 ? 4 : 0;  // elements
  static constexpr int kStride = kChunk + 8;             // elements per staged row (16-byte multiple)
  __host__ __device__ static constexpr int pos(int t) { return t < kChunk / 2 ? t : t + kShift; }
};

// ---- element conversions ------------------------------------------------------------------

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// ---- vectorised row access ----------------------------------------------------------------
// K consecutive elements starting at p. The widest access (16, 8, 4 bytes) that divides
// K * sizeof(T) is used; callers guarantee p is aligned to it.

template <int BYTES>
struct VecOf;
template <>
struct VecOf<16> { using type = uint4; };
template <>
struct VecOf<8> { using type = uint2; };
template <>
struct VecOf<4> { using type = uint32_t; };
template <>
struct VecOf<2> { using type = uint16_t; };

template <typename T, int K>
struct RowVec {
  static constexpr int kBytes = K * (int)sizeof(T);
  static constexpr int kVB = kBytes % 16 == 0 ? 16 : kBytes % 8 == 0 ? 8 : kBytes % 4 == 0 ? 4 : (int)sizeof(T);
  static constexpr int kEPV = kVB / (int)sizeof(T);
  static constexpr int kNV = K / kEPV;
  using V = typename VecOf<kVB>::type;
};

// Streaming load (read once: evict-first in L1/L2).
template <typename T, int K>
__device__ __forceinline__ void load_stream(const T* p, float (&x)[K]) {
  using R = RowVec<T, K>;
#pragma unroll
  for (int v = 0; v < R::kNV; ++v) {
    typename R::V raw = __ldcs(reinterpret_cast<const typename R::V*>(p) + v);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int j = 0; j < R::kEPV; ++j) x[v * R::kEPV + j] = to_f32<T>(e[j]);
  }
}

// Cached load (data shared by several threads / CTAs, e.g. B and C).
template <typename T, int K>
__device__ __forceinline__ void load_cached(const T* p, float (&x)[K]) {
  using R = RowVec<T, K>;
#pragma unroll
  for (int v = 0; v < R::kNV; ++v) {
    typename R::V raw = __ldg(reinterpret_cast<const typename R::V*>(p) + v);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int j = 0; j < R::kEPV; ++j) x[v * R::kEPV + j] = to_f32<T>(e[j]);
  }
}

// K consecutive elements from shared memory (16/8/4-byte vector reads).
template <typename T, int K>
__device__ __forceinline__ void load_cached_smem(const T* p, float (&x)[K]) {
  using R = RowVec<T, K>;
#pragma unroll
  for (int v = 0; v < R::kNV; ++v) {
    typename R::V raw = reinterpret_cast<const typename R::V*>(p)[v];
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int j = 0; j < R::kEPV; ++j) x[v * R::kEPV + j] = to_f32<T>(e[j]);
  }
}

template <typename T, int K>
__device__ __forceinline__ void store_stream(T* p, const float (&x)[K]) {
  using R = RowVec<T, K>;
#pragma unroll
  for (int v = 0; v < R::kNV; ++v) {
    typename R::V raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int j = 0; j < R::kEPV; ++j) e[j] = from_f32<T>(x[v * R::kEPV + j]);
    __stcs(reinterpret_cast<typename R::V*>(p) + v, raw);
  }
}

// K items of a row at [t0, t0 + K): vectorised when `vec` and fully in range, else per element
// with `fill` beyond seqlen.
template <typename T, int K>
__device__ __forceinline__ void load_items(const T* row, int64_t t0, int64_t L, bool vec, float fill,
                                           float (&x)[K]) {
  if (vec && t0 + K <= L) {
    load_stream<T, K>(row + t0, x);
  } else {
#pragma unroll
    for (int i = 0; i < K; ++i) x[i] = (t0 + i < L) ? to_f32<T>(row[t0 + i]) : fill;
  }
}

template <typename T, int K>
__device__ __forceinline__ void store_items(T* row, int64_t t0, int64_t L, bool vec, const float (&x)[K]) {
  if (vec && t0 + K <= L) {
    store_stream<T, K>(row + t0, x);
  } else {
#pragma unroll
    for (int i = 0; i < K; ++i)
      if (t0 + i < L) row[t0 + i] = from_f32<T>(x[i]);
  }
}

// Strided (B / C) items: element (t) at p[t * stride].
template <typename T, int K>
__device__ __forceinline__ void load_bc_items(const T* p, int64_t stride, int64_t t0, int64_t L, bool vec,
                                              float (&x)[K]) {
  if (vec && t0 + K <= L) {
    load_cached<T, K>(p + t0, x);
  } else {
#pragma unroll
    for (int i = 0; i < K; ++i) x[i] = (t0 + i < L) ? to_f32<T>(__ldg(p + (t0 + i) * stride)) : 0.f;
  }
}

// Hint: bring the 128-byte line holding p into L2 (no register result).
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// ---- math ---------------------------------------------------------------------------------

// 2^x on the SFU (MUFU.EX2). Inputs below -126 give 0 (flush), +inf gives +inf, NaN gives NaN.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// torch.nn.functional.softplus with its default threshold 20 (mamba-cpu selective_scan.cpp:45:
// x for x > 20, else log(1 + e^x)), evaluated as max(x, 0) + log1p(y) with y = e^-|x| <= 1 and
//   log1p(y) = 2 atanh(s) = 2 (s + s^3/3 + s^5/5 + ...),   s = y / (2 + y) <= 1/3,
// whose series, cut after s^13, is accurate to ~1e-8 relative over the whole range of y, so the
// result keeps the relative accuracy of e^-|x| (a few 1e-7) without a library log1p.
__device__ __forceinline__ float softplus_f(float x) {
  const float y = __expf(-fabsf(x));
  const float s = __fdividef(y, 2.f + y);
  const float s2 = s * s;
  float p = fmaf(s2, 1.f / 13.f, 1.f / 11.f);
  p = fmaf(s2, p, 1.f / 9.f);
  p = fmaf(s2, p, 1.f / 7.f);
  p = fmaf(s2, p, 1.f / 5.f);
  p = fmaf(s2, p, 1.f / 3.f);
  p = fmaf(s2, p, 1.f);
  const float r = fmaxf(x, 0.f) + 2.f * s * p;
  return x <= 20.f ? r : x;  // NaN takes the first branch and stays NaN
}

// softplus_f(x) and its derivative sigmoid(x) from one exponential: with y = e^-|x|,
// sigmoid(x) = (x >= 0 ? 1 : y) / (1 + y).
__device__ __forceinline__ float softplus_dsig(float x, float& sig) {
  const float y = __expf(-fabsf(x));
  sig = __fdividef(x >= 0.f ? 1.f : y, 1.f + y);
  const float s = __fdividef(y, 2.f + y);
  const float s2 = s * s;
  float p = fmaf(s2, 1.f / 13.f, 1.f / 11.f);
  p = fmaf(s2, p, 1.f / 9.f);
  p = fmaf(s2, p, 1.f / 7.f);
  p = fmaf(s2, p, 1.f / 5.f);
  p = fmaf(s2, p, 1.f / 3.f);
  p = fmaf(s2, p, 1.f);
  const float r = fmaxf(x, 0.f) + 2.f * s * p;
  return x <= 20.f ? r : x;
}

// 1 / (1 + e^-x); +-inf inputs give 0 / 1 (the fast division returns 0 for denominators past
// 2^126, the correctly rounded value to within its error bound).
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// x * sigmoid(x) (SiLU); -inf gives NaN as -inf * 0 does.
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.f + __expf(-x)); }

// ---- dtype dispatch helpers -----------------------------------------------------------------

inline int dtype_size(int code) {
  return code == MB200_F32 ? 4 : (code == MB200_BF16 || code == MB200_F16) ? 2 : 0;
}

__host__ __device__ inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Kernel launch counter (per host thread) reported by mb200_last_launch_count().
void note_launches(int n);
void reset_launches();

}  // namespace mb200
