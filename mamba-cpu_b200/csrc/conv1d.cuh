// conv1d.cuh -- causal depthwise conv1d (+ SiLU) launchers.
#pragma once

#include "common.cuh"

namespace mb200 {

constexpr int kConvMaxWidth = 8;
constexpr int kConvThreads = 128;  // threads per CTA
// Consecutive outputs per thread: 32 bytes of each input row per thread (8 fp32, 16 bf16 / fp16
// items), so that every thread keeps two 16-byte loads per row in flight.
constexpr int kConvRowBytes = 32;
template <typename T>
constexpr int conv_items() { return kConvRowBytes / (int)sizeof(T); }

struct ConvArgs {
  const void* x;
  const float* w;
  const float* bias;
  const void* init;
  void* out;
  void* final_states;
  int64_t batch, dim, L, width;
  int silu;
  int vec;  // x / out rows allow 16-byte vector access
  int64_t blocks_per_row;
};

// Number of per-CTA partial rows (each width + 1 floats) the backward writes for dweight/dbias.
int64_t conv_bwd_partials(const ConvArgs& a);

cudaError_t launch_conv_fwd(const ConvArgs& a, int dtype, cudaStream_t stream);
cudaError_t launch_conv_bwd(const ConvArgs& a, int dtype, const void* dout, void* dx, float* dweight,
                            float* dbias, void* dinit, float* part, cudaStream_t stream);

}  // namespace mb200
