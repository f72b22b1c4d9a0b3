// decode.cu -- one-token decode kernels on sm_100a.
//
// selective_state_update (mamba-cpu src/mamba_cpu/ops/selective_state_update.py:5-57):
//   dt = softplus(dt + dt_bias); state = state * exp(dt * A) + dt * x * B; out = <state, C> + D x,
//   out *= silu(z). dstate <= 16 (Mamba-1): one thread per (batch, channel), the dstate entries of
//   its state row in registers. Wider states (Mamba-2's 64 / 128 per head channel): one warp per
//   (batch, channel), lane l owning entries l, l + 32, ..., so the state row, A row and B / C rows
//   move as coalesced 128-byte lines; <state, C> is summed over the warp by shuffles. B / C rows
//   are shared by the channels of a group and read through L1.
// causal_conv1d_update (src/mamba_cpu/ops/causal_conv1d.py:56-85): the conv state window is
//   shifted by seqlen new inputs in place and every new input yields one output.
#include "decode.cuh"

namespace mb200 {

namespace {

template <typename TI, typename TW, typename TS>
__global__ void state_update_kernel(const mb200_state_update_params p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.batch * p.dim) return;
  const int64_t b = i / p.dim, d = i % p.dim;
  const int64_t g = d / (p.dim / p.ngroups);
  const int N = (int)p.dstate;
  TS* st = static_cast<TS*>(p.state) + i * N;
  const TW* Bp = static_cast<const TW*>(p.B) + (b * p.ngroups + g) * N;
  const TW* Cp = static_cast<const TW*>(p.C) + (b * p.ngroups + g) * N;
  const float x = to_f32<TI>(static_cast<const TI*>(p.x)[i]);
  float dt = to_f32<TI>(static_cast<const TI*>(p.dt)[i]) + (p.dt_bias ? p.dt_bias[d] : 0.f);
  if (p.dt_softplus) dt = softplus_f(dt);
  const float dtx = dt * x;
  float y = 0.f;
#pragma unroll
  for (int n = 0; n < kMaxState; ++n) {
    if (n < N) {
      const float a = ex2(dt * p.A[d * N + n] * kLog2e);
      const float s = fmaf(to_f32<TS>(st[n]), a, dtx * to_f32<TW>(__ldg(Bp + n)));
      st[n] = from_f32<TS>(s);
      y = fmaf(s, to_f32<TW>(__ldg(Cp + n)), y);
    }
  }
  if (p.D) y = fmaf(x, p.D[d], y);
  if (p.z) {
    const float z = to_f32<TI>(static_cast<const TI*>(p.z)[i]);
    y *= z * sigmoid_f(z);
  }
  static_cast<TI*>(p.out)[i] = from_f32<TI>(y);
}

constexpr int kWideWarps = 8;  // rows (warps) per CTA of the wide-state kernel

template <typename TI, typename TW, typename TS>
__global__ void __launch_bounds__(32 * kWideWarps) state_update_wide_kernel(const mb200_state_update_params p) {
  const int lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * kWideWarps + (threadIdx.x >> 5);
  if (i >= p.batch * p.dim) return;  // warp-uniform
  const int64_t b = i / p.dim, d = i % p.dim;
  const int64_t g = d / (p.dim / p.ngroups);
  const int N = (int)p.dstate;
  TS* st = static_cast<TS*>(p.state) + i * N;
  const TW* Bp = static_cast<const TW*>(p.B) + (b * p.ngroups + g) * N;
  const TW* Cp = static_cast<const TW*>(p.C) + (b * p.ngroups + g) * N;
  const float* Ap = p.A + d * N;
  const float x = to_f32<TI>(static_cast<const TI*>(p.x)[i]);
  float dt = to_f32<TI>(static_cast<const TI*>(p.dt)[i]) + (p.dt_bias ? p.dt_bias[d] : 0.f);
  if (p.dt_softplus) dt = softplus_f(dt);
  const float dtx = dt * x;
  const float dtl = dt * kLog2e;
  float y = 0.f;
  for (int n = lane; n < N; n += 32) {
    const float a = ex2(dtl * Ap[n]);
    const float s = fmaf(to_f32<TS>(st[n]), a, dtx * to_f32<TW>(__ldg(Bp + n)));
    st[n] = from_f32<TS>(s);
    y = fmaf(s, to_f32<TW>(__ldg(Cp + n)), y);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) y += __shfl_xor_sync(0xffffffffu, y, off);
  if (lane == 0) {
    if (p.D) y = fmaf(x, p.D[d], y);
    if (p.z) {
      const float z = to_f32<TI>(static_cast<const TI*>(p.z)[i]);
      y *= z * sigmoid_f(z);
    }
    static_cast<TI*>(p.out)[i] = from_f32<TI>(y);
  }
}

template <typename T>
__global__ void conv_update_kernel(const mb200_conv1d_update_params p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.batch * p.dim) return;
  const int64_t d = i % p.dim;
  const int64_t S = p.state_len, L = p.seqlen, W = p.width;
  T* st = static_cast<T*>(p.conv_state) + i * S;
  const T* xr = static_cast<const T*>(p.x) + i * L;
  T* orow = static_cast<T*>(p.out) + i * L;
  const float bias = p.bias ? p.bias[d] : 0.f;
  const float* w = p.weight + d * W;
  // window[j] = [state | x][j]; output t uses window[S + t - (W - 1) + k]
  for (int64_t t = 0; t < L; ++t) {
    float acc = bias;
    for (int64_t k = 0; k < W; ++k) {
      const int64_t j = S + t - (W - 1) + k;
      const float v = j < S ? to_f32<T>(st[j]) : to_f32<T>(xr[j - S]);
      acc = fmaf(w[k], v, acc);
    }
    orow[t] = from_f32<T>(p.activation ? acc * sigmoid_f(acc) : acc);
  }
  // new state = last S entries of [state | x]
  for (int64_t j = 0; j < S; ++j) {
    const int64_t src = j + L;
    const T v = src < S ? st[src] : xr[src - S];
    st[j] = v;
  }
}

template <typename TI, typename TW>
cudaError_t su_state(const mb200_state_update_params& p, cudaStream_t stream) {
  const int64_t n = p.batch * p.dim;
  if (p.dstate > kMaxState) {
    const unsigned wblocks = (unsigned)((n + kWideWarps - 1) / kWideWarps);
    if (p.state_dtype == MB200_F32)
      state_update_wide_kernel<TI, TW, float><<<wblocks, 32 * kWideWarps, 0, stream>>>(p);
    else
      state_update_wide_kernel<TI, TW, TI><<<wblocks, 32 * kWideWarps, 0, stream>>>(p);
    return cudaGetLastError();
  }
  const unsigned blocks = (unsigned)((n + 127) / 128);
  if (p.state_dtype == MB200_F32)
    state_update_kernel<TI, TW, float><<<blocks, 128, 0, stream>>>(p);
  else
    state_update_kernel<TI, TW, TI><<<blocks, 128, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_state_update(const mb200_state_update_params& p, cudaStream_t stream) {
  if (p.batch == 0 || p.dim == 0) return cudaSuccess;
  if (p.io_dtype == MB200_F32) return su_state<float, float>(p, stream);
  if (p.io_dtype == MB200_BF16)
    return p.bc_dtype == MB200_BF16 ? su_state<__nv_bfloat16, __nv_bfloat16>(p, stream)
                                    : su_state<__nv_bfloat16, float>(p, stream);
  return p.bc_dtype == MB200_F16 ? su_state<__half, __half>(p, stream) : su_state<__half, float>(p, stream);
}

cudaError_t launch_conv_update(const mb200_conv1d_update_params& p, cudaStream_t stream) {
  if (p.batch == 0 || p.dim == 0) return cudaSuccess;
  const int64_t n = p.batch * p.dim;
  const unsigned blocks = (unsigned)((n + 127) / 128);
  if (p.x_dtype == MB200_F32)
    conv_update_kernel<float><<<blocks, 128, 0, stream>>>(p);
  else if (p.x_dtype == MB200_BF16)
    conv_update_kernel<__nv_bfloat16><<<blocks, 128, 0, stream>>>(p);
  else
    conv_update_kernel<__half><<<blocks, 128, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace mb200
