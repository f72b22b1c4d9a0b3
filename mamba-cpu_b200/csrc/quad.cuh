// quad.cuh -- four consecutive timesteps of a row as one unit of global-memory traffic.
//
// The scan kernels move (batch, dim, seqlen) rows in groups of four elements: one 16-byte access
// for fp32, one 8-byte access for bf16 / fp16. Loads are split in two halves so that a prefetch
// can be issued long before its data is needed: ld_* returns the raw bits (no use of the result,
// hence no wait), to_float4 converts them when the consumer runs.
#pragma once

#include "common.cuh"

namespace mb200 {

template <typename T>
struct Quad {
  using V = typename VecOf<4 * sizeof(T)>::type;  // uint4 (fp32) or uint2 (16-bit types)
  V v;
};

// Four elements at p (aligned to 4 * sizeof(T)), streaming (evict-first) load.
template <typename T>
__device__ __forceinline__ Quad<T> ld_quad_stream(const T* p) {
  Quad<T> q;
  q.v = __ldcs(reinterpret_cast<const typename Quad<T>::V*>(p));
  return q;
}

// Four elements at p (aligned), read-only cached load (data shared by several CTAs).
template <typename T>
__device__ __forceinline__ Quad<T> ld_quad_cached(const T* p) {
  Quad<T> q;
  q.v = __ldg(reinterpret_cast<const typename Quad<T>::V*>(p));
  return q;
}

// Elements p[(t + e) * stride] for e < 4, zero where t + e >= L.
template <typename T>
__device__ __forceinline__ Quad<T> ld_quad_masked(const T* p, int64_t t, int64_t L, int64_t stride) {
  T e[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) e[i] = (t + i < L) ? p[(t + i) * stride] : from_f32<T>(0.f);
  Quad<T> q;
  memcpy(&q.v, e, sizeof(e));
  return q;
}

template <typename T>
__device__ __forceinline__ Quad<T> zero_quad() {
  Quad<T> q;
  memset(&q.v, 0, sizeof(q.v));
  return q;
}

template <typename T>
__device__ __forceinline__ float4 to_float4(const Quad<T>& q) {
  const T* e = reinterpret_cast<const T*>(&q.v);
  return make_float4(to_f32<T>(e[0]), to_f32<T>(e[1]), to_f32<T>(e[2]), to_f32<T>(e[3]));
}

// Four elements to p (aligned), streaming store.
template <typename T>
__device__ __forceinline__ void st_quad_stream(T* p, float4 v) {
  T e[4] = {from_f32<T>(v.x), from_f32<T>(v.y), from_f32<T>(v.z), from_f32<T>(v.w)};
  typename Quad<T>::V raw;
  memcpy(&raw, e, sizeof(e));
  __stcs(reinterpret_cast<typename Quad<T>::V*>(p), raw);
}

// p[t + e] = v[e] for the e < 4 with t + e < L.
template <typename T>
__device__ __forceinline__ void st_quad_masked(T* p, int64_t t, int64_t L, float4 v) {
  const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (t + i < L) p[t + i] = from_f32<T>(x[i]);
}

__device__ __forceinline__ float2 lo2(float4 v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(float4 v) { return make_float2(v.z, v.w); }

}  // namespace mb200
