// conv1d.cu -- causal depthwise conv1d with optional SiLU on sm_100a.
//
// out[b, d, t] = act(bias[d] + sum_k w[d, k] * xf[b, d, t + k]), xf = [initial_states | x] (or
// W-1 zeros in front of x), as mamba-cpu's causal_conv1d_fn computes with F.conv1d
// (src/mamba_cpu/ops/causal_conv1d.py:37-47). The op is HBM-bound (one read of x, one write of
// out): each thread produces 32 bytes' worth of consecutive outputs of one row (8 fp32 or 16
// 16-bit items) from two 16-byte loads of its inputs plus a W-1 element halo served by L1.
#include "conv1d.cuh"

namespace mb200 {

namespace {

template <typename T, int W>
__global__ void __launch_bounds__(kConvThreads) conv_fwd_kernel(const ConvArgs a) {
  constexpr int J = conv_items<T>();
  constexpr int P = W - 1;
  // One CTA per (channel, span of the row); it walks the batch's rows of that channel, so a CTA
  // streams batch x 32 bytes per thread instead of exiting after one round trip.
  const int64_t d = blockIdx.x / a.blocks_per_row;
  const int64_t tb = blockIdx.x % a.blocks_per_row;
  const int64_t t0 = (tb * kConvThreads + threadIdx.x) * J;
  const int64_t L = a.L;
  if (t0 >= L && !(L == 0 && t0 == 0)) return;
  float w[W];
#pragma unroll
  for (int k = 0; k < W; ++k) w[k] = a.w[d * W + k];
  const float bias = a.bias ? a.bias[d] : 0.f;
  for (int64_t b = 0; b < a.batch; ++b) {
    const int64_t row = b * a.dim + d;
    const T* xrow = static_cast<const T*>(a.x) + row * L;
    const T* irow = a.init ? static_cast<const T*>(a.init) + row * P : nullptr;

    float xv[J + P];
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int64_t s = t0 - P + j;
      xv[j] = s >= 0 ? to_f32<T>(xrow[s]) : (irow ? to_f32<T>(irow[P + s]) : 0.f);
    }
    {
      float m[J];
      load_items<T, J>(xrow, t0, L, a.vec != 0, 0.f, m);
#pragma unroll
      for (int i = 0; i < J; ++i) xv[P + i] = m[i];
    }
    float o[J];
#pragma unroll
    for (int i = 0; i < J; ++i) {
      float acc = bias;
#pragma unroll
      for (int k = 0; k < W; ++k) acc = fmaf(w[k], xv[i + k], acc);
      o[i] = a.silu ? acc * sigmoid_f(acc) : acc;
    }
    store_items<T, J>(static_cast<T*>(a.out) + row * L, t0, L, a.vec != 0, o);

    // The thread holding the last timestep (or thread 0 of an empty row) writes the final states:
    // the last W-1 entries of [initial_states | x] (causal_conv1d.py:48-53).
    if (a.final_states != nullptr && P > 0 && t0 <= (L > 0 ? L - 1 : 0) && (L == 0 || L - 1 < t0 + J)) {
      T* frow = static_cast<T*>(a.final_states) + row * P;
#pragma unroll
      for (int j = 0; j < P; ++j) {
        const int64_t s = L - P + j;
        float v = s >= 0 ? to_f32<T>(xrow[s]) : (irow ? to_f32<T>(irow[P + s]) : 0.f);
        frow[j] = from_f32<T>(v);
      }
    }
  }  // batch rows
}

// Backward: g[t] = dout[t] * act'(pre[t]);  dx[s] = sum_k w[k] g[s + P - k];
// dinit[j] = sum_k w[k] g[j - k] (j < P);  dw[k] = sum_{b,t} g[t] xf[t + k];  dbias = sum g.
// Per-CTA partials of dw / dbias go to `part` and are summed per channel by conv_bwd_reduce.
template <typename T, int W>
__global__ void __launch_bounds__(kConvThreads) conv_bwd_kernel(const ConvArgs a, const T* dout, T* dx,
                                                                T* dinit, float* part) {
  constexpr int J = conv_items<T>();
  constexpr int P = W - 1;
  __shared__ float red[kConvThreads / 32][W + 1];
  const int64_t row = blockIdx.x / a.blocks_per_row;
  const int64_t tb = blockIdx.x % a.blocks_per_row;
  const int64_t t0 = (tb * kConvThreads + threadIdx.x) * J;
  const int64_t L = a.L;
  const int64_t d = row % a.dim;
  const T* xrow = static_cast<const T*>(a.x) + row * L;
  const T* irow = a.init ? static_cast<const T*>(a.init) + row * P : nullptr;
  const T* grow = dout + row * L;

  float w[W];
#pragma unroll
  for (int k = 0; k < W; ++k) w[k] = a.w[d * W + k];
  const float bias = a.bias ? a.bias[d] : 0.f;

  float pw[W + 1];
#pragma unroll
  for (int k = 0; k <= W; ++k) pw[k] = 0.f;

  if (t0 < L) {
    // xv[m] = xf at x-index t0 - P + m, m in [0, J + 2P)
    float xv[J + 2 * P];
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int64_t s = t0 - P + j;
      xv[j] = s >= 0 ? to_f32<T>(xrow[s]) : (irow ? to_f32<T>(irow[P + s]) : 0.f);
    }
    {
      float m[J];
      load_items<T, J>(xrow, t0, L, a.vec != 0, 0.f, m);
#pragma unroll
      for (int i = 0; i < J; ++i) xv[P + i] = m[i];
    }
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int64_t s = t0 + J + j;
      xv[P + J + j] = s < L ? to_f32<T>(xrow[s]) : 0.f;
    }
    // gg[m] = g at t0 + m, m in [0, J + P)
    float gg[J + P];
    {
      float dm[J];
      load_items<T, J>(grow, t0, L, a.vec != 0, 0.f, dm);
#pragma unroll
      for (int m = 0; m < J + P; ++m) {
        const int64_t t = t0 + m;
        const float go = m < J ? dm[m] : (t < L ? to_f32<T>(grow[t]) : 0.f);
        float pre = bias;
#pragma unroll
        for (int k = 0; k < W; ++k) pre = fmaf(w[k], xv[m + k], pre);
        float gd = go;
        if (a.silu) {
          const float sg = sigmoid_f(pre);
          gd = go * sg * (1.f + pre * (1.f - sg));
        }
        gg[m] = t < L ? gd : 0.f;
      }
    }
    float o[J];
#pragma unroll
    for (int i = 0; i < J; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < W; ++k) acc = fmaf(w[k], gg[i + P - k], acc);
      o[i] = acc;
      if (t0 + i < L) {
#pragma unroll
        for (int k = 0; k < W; ++k) pw[k] = fmaf(gg[i], xv[i + k], pw[k]);
        pw[W] += gg[i];
      }
    }
    store_items<T, J>(dx + row * L, t0, L, a.vec != 0, o);
    if (dinit != nullptr && t0 == 0) {
#pragma unroll
      for (int j = 0; j < P; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < W; ++k)
          if (j - k >= 0 && j - k < J + P) acc = fmaf(w[k], gg[j - k], acc);
        dinit[row * P + j] = from_f32<T>(acc);
      }
    }
  } else if (dinit != nullptr && t0 == 0) {
    // empty row: no output depends on the initial states
#pragma unroll
    for (int j = 0; j < P; ++j) dinit[row * P + j] = from_f32<T>(0.f);
  }

  // CTA sum of the dw / dbias partials
#pragma unroll
  for (int k = 0; k <= W; ++k) {
    float v = pw[k];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][k] = v;
  }
  __syncthreads();
  if (threadIdx.x <= W) {
    float v = 0.f;
#pragma unroll
    for (int wi = 0; wi < kConvThreads / 32; ++wi) v += red[wi][threadIdx.x];
    part[blockIdx.x * (W + 1) + threadIdx.x] = v;
  }
}

// ---- forward through a shared-memory pipeline (aligned rows, batch >= 8) -----------------------
// The register-load kernel above keeps ~64 bytes per thread in flight, which leaves HBM under-used.
// Here a CTA owns one (channel, span) and walks the batch's rows of that channel through a
// kConvStages-deep pipeline of cp.async copies into shared memory: the copies of the next rows are
// in flight while a row is computed. Per stage: x = [kJ items before the span | span]; items before
// t = 0 are the initial states (or zeros).
constexpr int kConvStages = 3;
constexpr int64_t kConvStagedMinBatch = 8;

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(
                   smem_dst))),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T>
struct ConvStage {  // element counts
  static constexpr int kJ = conv_items<T>();         // items per thread (32 bytes)
  static constexpr int kSpan = kConvThreads * kJ;   // items per CTA and row
};

template <typename T, int W>
__global__ void __launch_bounds__(kConvThreads) conv_fwd_staged_kernel(const ConvArgs a) {
  using St = ConvStage<T>;
  constexpr int J = St::kJ;
  constexpr int P = W - 1;
  constexpr int kXF = J + St::kSpan;  // elements per stage; kXF * sizeof(T) is a multiple of 16
  static_assert(P <= J, "the halo holds the W - 1 items before the span");
  extern __shared__ __align__(16) unsigned char conv_smem[];
  T* sbuf = reinterpret_cast<T*>(conv_smem);
  const int tid = threadIdx.x;
  const int64_t d = blockIdx.x / a.blocks_per_row;
  const int64_t tb = blockIdx.x % a.blocks_per_row;
  const int64_t s0 = tb * St::kSpan;
  const int64_t t0 = s0 + (int64_t)tid * J;
  const int64_t L = a.L;
  const T* x = static_cast<const T*>(a.x);
  const T* init = static_cast<const T*>(a.init);
  const T zero = from_f32<T>(0.f);
  float w[W];
#pragma unroll
  for (int k = 0; k < W; ++k) w[k] = a.w[d * W + k];
  const float bias = a.bias ? a.bias[d] : 0.f;

  auto issue = [&](int64_t b, int st) {
    T* xs = sbuf + (size_t)st * kXF;
    const int64_t row = b * a.dim + d;
    const T* xrow = x + row * L;
    if (t0 + J <= L) {
      cp_async16(xs + J + tid * J, xrow + t0);
      cp_async16(xs + J + tid * J + J / 2, xrow + t0 + J / 2);
    } else {
#pragma unroll
      for (int i = 0; i < J; ++i) xs[J + tid * J + i] = t0 + i < L ? xrow[t0 + i] : zero;
    }
    if (tid == 0) {
      if (s0 >= J) {
        cp_async16(xs, xrow + s0 - J);
        cp_async16(xs + J / 2, xrow + s0 - J / 2);
      } else {
        const T* irow = init ? init + row * P : nullptr;
#pragma unroll
        for (int i = 0; i < J; ++i) {
          const int sidx = i - J;
          xs[i] = (irow != nullptr && sidx >= -P) ? irow[P + sidx] : zero;
        }
      }
    }
  };

#pragma unroll
  for (int sidx = 0; sidx < kConvStages - 1; ++sidx) {
    if (sidx < a.batch) issue(sidx, sidx);
    cp_async_commit();
  }
  for (int64_t b = 0; b < a.batch; ++b) {
    const int64_t nb = b + kConvStages - 1;
    if (nb < a.batch) issue(nb, (int)(nb % kConvStages));
    cp_async_commit();
    cp_async_wait<kConvStages - 1>();
    __syncthreads();
    const T* xs = sbuf + (size_t)(b % kConvStages) * kXF;
    const int64_t row = b * a.dim + d;
    if (t0 < L || (L == 0 && t0 == 0)) {
      float xv[J + P];
#pragma unroll
      for (int m = 0; m < J + P; ++m) xv[m] = to_f32<T>(xs[J + tid * J - P + m]);
      float o[J];
#pragma unroll
      for (int i = 0; i < J; ++i) {
        float acc = bias;
#pragma unroll
        for (int k = 0; k < W; ++k) acc = fmaf(w[k], xv[i + k], acc);
        o[i] = a.silu ? acc * sigmoid_f(acc) : acc;
      }
      store_items<T, J>(static_cast<T*>(a.out) + row * L, t0, L, true, o);
      // final states: the last W-1 entries of [initial_states | x], by the thread holding the
      // last timestep (or thread 0 of an empty row)
      if (a.final_states != nullptr && P > 0 && t0 <= (L > 0 ? L - 1 : 0) && (L == 0 || L - 1 < t0 + J)) {
        const T* xrow = x + row * L;
        const T* irow = init ? init + row * P : nullptr;
        T* frow = static_cast<T*>(a.final_states) + row * P;
#pragma unroll
        for (int j = 0; j < P; ++j) {
          const int64_t sidx = L - P + j;
          frow[j] = sidx >= 0 ? xrow[sidx] : (irow ? irow[P + sidx] : zero);
        }
      }
    }
    __syncthreads();
  }
}

// ---- streaming backward (16-byte aligned rows) --------------------------------------------------
// One thread per 16 consecutive outputs of a row (four 16-byte vectors of fp32, two of 16-bit
// types) of x and dout plus one halo vector on each side: every load of a thread is issued before
// the first use, so each SM keeps 50-100 KB of loads in flight (HBM latency x bandwidth per SM is
// about 40-70 KB). The CTAs of a channel cover the batch rows of that channel, so the dw / dbias
// partials are one per CTA, already summed over the batch.
// 128-thread CTAs capped at 64 registers a thread: 8 CTAs (32 warps) per SM keep more loads in
// flight than 256-thread CTAs at 70 registers (3 CTAs, 24 warps): config-4 layer shape bf16
// 154.6 -> 138.2 µs, config-5 shape (L 4096) 101.4 -> 91.1 µs.
constexpr int kStreamThreads = 128;
constexpr int kStreamItems = 16;  // outputs per thread

template <typename T>
struct StreamShape {
  static constexpr int kV = 16 / (int)sizeof(T);      // elements per 16-byte vector
  static constexpr int kU = kStreamItems / kV;        // vectors per thread
};

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float* out) {
  const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(p));
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int j = 0; j < StreamShape<T>::kV; ++j) out[j] = to_f32<T>(e[j]);
}

template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float* v) {
  uint4 raw;
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int j = 0; j < StreamShape<T>::kV; ++j) e[j] = from_f32<T>(v[j]);
  __stcs(reinterpret_cast<uint4*>(p), raw);
}

// x (or xf = [init | x] before t = 0) at t0 - kH*V .. t0 + (U + kA) * V into xv; kH / kA halo
// vectors before / after the thread's own U vectors (t0 a multiple of 16 items, so a halo vector
// before t = 0 lies entirely in the initial states and one after L entirely past the row end).
template <typename T, int kH, int kA>
__device__ __forceinline__ void load_span(const T* xrow, const T* irow, int P, int64_t t0, int64_t L,
                                          float (&xv)[(kH + StreamShape<T>::kU + kA) * StreamShape<T>::kV]) {
  constexpr int V = StreamShape<T>::kV, U = StreamShape<T>::kU;
#pragma unroll
  for (int j = 0; j < U + kA; ++j) {  // own vectors and the halo after: in flight together
    const int64_t s = t0 + j * V;
    if (s < L) {
      load_vec<T>(xrow + s, &xv[(kH + j) * V]);
    } else {
#pragma unroll
      for (int e = 0; e < V; ++e) xv[(kH + j) * V + e] = 0.f;
    }
  }
#pragma unroll
  for (int j = 0; j < kH; ++j) {
    const int64_t s = t0 - (kH - j) * V;
    if (s >= 0) {
      load_vec<T>(xrow + s, &xv[j * V]);
    } else {
#pragma unroll
      for (int e = 0; e < V; ++e) {
        const int64_t idx = s + e;  // negative: initial state P + idx, zeros before it
        xv[j * V + e] = (irow != nullptr && idx >= -P) ? to_f32<T>(irow[P + idx]) : 0.f;
      }
    }
  }
}

// Backward, one CTA per (channel, group of kStreamThreads pieces of its batch rows): per thread
// g = dout * act'(pre) over its 16 outputs and the P after them, dx from g, and the thread's share
// of dw / dbias; the CTA's sum is written to part (summed per channel by conv_bwd_reduce).
template <typename T, int W>
__global__ void __launch_bounds__(kStreamThreads, 8) conv_bwd_stream_kernel(const ConvArgs a, const T* dout, T* dx,
                                                                         T* dinit, float* part, int64_t cpr,
                                                                         int64_t cpc) {
  constexpr int V = StreamShape<T>::kV, U = StreamShape<T>::kU;
  constexpr int P = W - 1;
  constexpr int kH = (P + V - 1) / V;
  constexpr int kA = (P + V - 1) / V;
  constexpr int J = kStreamItems;
  __shared__ float red[kStreamThreads / 32][W + 1];
  const int64_t d = blockIdx.x / cpc;
  const int64_t task = (blockIdx.x % cpc) * kStreamThreads + threadIdx.x;
  const int64_t b = task / cpr;
  const int64_t t0 = (task % cpr) * J;
  const int64_t L = a.L;
  float w[W];
#pragma unroll
  for (int k = 0; k < W; ++k) w[k] = a.w[d * W + k];
  const float bias = a.bias ? a.bias[d] : 0.f;
  float pw[W + 1];
#pragma unroll
  for (int k = 0; k <= W; ++k) pw[k] = 0.f;
  if (b < a.batch) {
    const int64_t row = b * a.dim + d;
    const T* xrow = static_cast<const T*>(a.x) + row * L;
    const T* irow = a.init ? static_cast<const T*>(a.init) + row * P : nullptr;
    const T* grow = dout + row * L;
    float xv[(kH + U + kA) * V];
    float gv[(U + kA) * V];
#pragma unroll
    for (int j = 0; j < U + kA; ++j) {
      const int64_t s = t0 + j * V;
      if (s < L) {
        load_vec<T>(grow + s, &gv[j * V]);
      } else {
#pragma unroll
        for (int e = 0; e < V; ++e) gv[j * V + e] = 0.f;
      }
    }
    load_span<T, kH, kA>(xrow, irow, P, t0, L, xv);
    // gg[m] = g at t0 + m, m in [0, J + P): dout * act'(pre), 0 past the row end
    float gg[J + P];
#pragma unroll
    for (int m = 0; m < J + P; ++m) {
      float pre = bias;
#pragma unroll
      for (int k = 0; k < W; ++k) pre = fmaf(w[k], xv[kH * V + m - P + k], pre);
      float gd = gv[m];
      if (a.silu) {
        const float sg = sigmoid_f(pre);
        gd *= sg * (1.f + pre * (1.f - sg));
      }
      gg[m] = t0 + m < L ? gd : 0.f;
    }
    float o[J];
#pragma unroll
    for (int i = 0; i < J; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < W; ++k) acc = fmaf(w[k], gg[i + P - k], acc);
      o[i] = acc;
#pragma unroll
      for (int k = 0; k < W; ++k) pw[k] = fmaf(gg[i], xv[kH * V + i - P + k], pw[k]);
      pw[W] += gg[i];  // gg is 0 past the row end
    }
    T* dxrow = dx + row * L;
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (t0 + j * V < L) store_vec<T>(dxrow + t0 + j * V, &o[j * V]);
    if (dinit != nullptr && t0 == 0) {
#pragma unroll
      for (int j = 0; j < P; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < W; ++k)
          if (j - k >= 0) acc = fmaf(w[k], gg[j - k], acc);
        dinit[row * P + j] = from_f32<T>(acc);
      }
    }
  }
  // CTA sum of the dw / dbias partials
#pragma unroll
  for (int k = 0; k <= W; ++k) {
    float v = pw[k];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][k] = v;
  }
  __syncthreads();
  if (threadIdx.x <= W) {
    float v = 0.f;
#pragma unroll
    for (int wi = 0; wi < kStreamThreads / 32; ++wi) v += red[wi][threadIdx.x];
    part[blockIdx.x * (W + 1) + threadIdx.x] = v;
  }
}

// dw[d, k] = sum over (batch group, CTA of the row) of the partials; one thread per (d, k). The
// register-load kernel writes one partial per (batch row, span) (groups = batch), the staged one
// one per (channel, span) already summed over the batch (groups = 1).
__global__ void conv_bwd_reduce(const float* part, float* dw, float* dbias, int64_t batch, int64_t dim,
                                int64_t bpr, int W) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= dim * (W + 1)) return;
  const int64_t d = i / (W + 1);
  const int k = (int)(i % (W + 1));
  float acc = 0.f;
  for (int64_t b = 0; b < batch; ++b) {
    const float* p = part + ((b * dim + d) * bpr) * (W + 1);
    for (int64_t t = 0; t < bpr; ++t) acc += p[t * (W + 1) + k];
  }
  if (k < W)
    dw[d * W + k] = acc;
  else if (dbias != nullptr)
    dbias[d] = acc;
}

template <typename T, int W>
cudaError_t fwd_w(const ConvArgs& a, cudaStream_t stream) {
  const int64_t blocks = a.dim * a.blocks_per_row;  // each CTA walks the batch
  if (a.vec != 0 && a.batch >= kConvStagedMinBatch) {  // as the backward: aligned rows, batch >= 8
    const size_t smem = kConvStages * (size_t)(ConvStage<T>::kJ + ConvStage<T>::kSpan) * sizeof(T);
    conv_fwd_staged_kernel<T, W><<<(unsigned)blocks, kConvThreads, smem, stream>>>(a);
  } else {
    conv_fwd_kernel<T, W><<<(unsigned)blocks, kConvThreads, 0, stream>>>(a);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t fwd_t(const ConvArgs& a, cudaStream_t stream) {
  switch (a.width) {
    case 1: return fwd_w<T, 1>(a, stream);
    case 2: return fwd_w<T, 2>(a, stream);
    case 3: return fwd_w<T, 3>(a, stream);
    case 4: return fwd_w<T, 4>(a, stream);
    case 5: return fwd_w<T, 5>(a, stream);
    case 6: return fwd_w<T, 6>(a, stream);
    case 7: return fwd_w<T, 7>(a, stream);
    default: return fwd_w<T, 8>(a, stream);
  }
}

// Pieces of kStreamItems outputs per row, and CTAs per channel of the streaming backward.
int64_t stream_cpr(const ConvArgs& a) { return (a.L + kStreamItems - 1) / kStreamItems; }
int64_t stream_cpc(const ConvArgs& a) { return (a.batch * stream_cpr(a) + kStreamThreads - 1) / kStreamThreads; }
bool use_stream(const ConvArgs& a) { return a.vec != 0 && a.L > 0; }

template <typename T, int W>
cudaError_t bwd_w(const ConvArgs& a, const void* dout, void* dx, float* dweight, float* dbias, void* dinit,
                  float* part, cudaStream_t stream) {
  // Aligned rows (16-byte row starts, rows a multiple of 16 bytes): the streaming kernel, whose
  // CTAs cover the batch rows of one channel (partials summed over the batch). Anything else: the
  // register-load kernel (one partial per batch row and span).
  int64_t groups = a.batch, per = a.blocks_per_row;
  if (use_stream(a) && aligned16(dout) && aligned16(dx)) {
    const int64_t cpr = stream_cpr(a), cpc = stream_cpc(a);
    conv_bwd_stream_kernel<T, W><<<(unsigned)(a.dim * cpc), kStreamThreads, 0, stream>>>(
        a, static_cast<const T*>(dout), static_cast<T*>(dx), static_cast<T*>(dinit), part, cpr, cpc);
    groups = 1;
    per = cpc;
  } else {
    const int64_t blocks = a.batch * a.dim * a.blocks_per_row;
    conv_bwd_kernel<T, W><<<(unsigned)blocks, kConvThreads, 0, stream>>>(
        a, static_cast<const T*>(dout), static_cast<T*>(dx), static_cast<T*>(dinit), part);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t n = a.dim * (W + 1);
  conv_bwd_reduce<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(part, dweight, dbias, groups, a.dim, per, W);
  return cudaGetLastError();
}

template <typename T>
cudaError_t bwd_t(const ConvArgs& a, const void* dout, void* dx, float* dweight, float* dbias, void* dinit,
                  float* part, cudaStream_t stream) {
  switch (a.width) {
    case 1: return bwd_w<T, 1>(a, dout, dx, dweight, dbias, dinit, part, stream);
    case 2: return bwd_w<T, 2>(a, dout, dx, dweight, dbias, dinit, part, stream);
    case 3: return bwd_w<T, 3>(a, dout, dx, dweight, dbias, dinit, part, stream);
    case 4: return bwd_w<T, 4>(a, dout, dx, dweight, dbias, dinit, part, stream);
    case 5: return bwd_w<T, 5>(a, dout, dx, dweight, dbias, dinit, part, stream);
    case 6: return bwd_w<T, 6>(a, dout, dx, dweight, dbias, dinit, part, stream);
    case 7: return bwd_w<T, 7>(a, dout, dx, dweight, dbias, dinit, part, stream);
    default: return bwd_w<T, 8>(a, dout, dx, dweight, dbias, dinit, part, stream);
  }
}

}  // namespace

int64_t conv_bwd_partials(const ConvArgs& a) {
  const int64_t reg = a.batch * a.dim * a.blocks_per_row;  // register-load kernel
  const int64_t str = a.dim * stream_cpc(a);               // streaming kernel
  return reg > str ? reg : str;
}

cudaError_t launch_conv_fwd(const ConvArgs& a, int dtype, cudaStream_t stream) {
  if (a.batch == 0 || a.dim == 0) return cudaSuccess;
  if (dtype == MB200_F32) return fwd_t<float>(a, stream);
  if (dtype == MB200_BF16) return fwd_t<__nv_bfloat16>(a, stream);
  return fwd_t<__half>(a, stream);
}

cudaError_t launch_conv_bwd(const ConvArgs& a, int dtype, const void* dout, void* dx, float* dweight,
                            float* dbias, void* dinit, float* part, cudaStream_t stream) {
  if (a.dim == 0) return cudaSuccess;
  if (a.batch == 0) {
    // no rows: dweight / dbias are zero
    cudaError_t e = cudaMemsetAsync(dweight, 0, sizeof(float) * a.dim * a.width, stream);
    if (e == cudaSuccess && dbias) e = cudaMemsetAsync(dbias, 0, sizeof(float) * a.dim, stream);
    return e;
  }
  if (dtype == MB200_F32) return bwd_t<float>(a, dout, dx, dweight, dbias, dinit, part, stream);
  if (dtype == MB200_BF16) return bwd_t<__nv_bfloat16>(a, dout, dx, dweight, dbias, dinit, part, stream);
  return bwd_t<__half>(a, dout, dx, dweight, dbias, dinit, part, stream);
}

}  // namespace mb200
