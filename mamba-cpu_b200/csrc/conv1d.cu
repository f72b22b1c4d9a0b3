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

// dw[d, k] = sum over (batch, CTA of the row) of the partials; one thread per (d, k).
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
  conv_fwd_kernel<T, W><<<(unsigned)blocks, kConvThreads, 0, stream>>>(a);
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

template <typename T, int W>
cudaError_t bwd_w(const ConvArgs& a, const void* dout, void* dx, float* dweight, float* dbias, void* dinit,
                  float* part, cudaStream_t stream) {
  const int64_t blocks = a.batch * a.dim * a.blocks_per_row;
  conv_bwd_kernel<T, W><<<(unsigned)blocks, kConvThreads, 0, stream>>>(
      a, static_cast<const T*>(dout), static_cast<T*>(dx), static_cast<T*>(dinit), part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t n = a.dim * (W + 1);
  conv_bwd_reduce<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(part, dweight, dbias, a.batch, a.dim,
                                                                   a.blocks_per_row, W);
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

int64_t conv_bwd_partials(const ConvArgs& a) { return a.batch * a.dim * a.blocks_per_row; }

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
