// segscan.cuh -- the time-parallel pieces shared by the forward and backward scans.
//
// A chunk of kChunk timesteps is split over the S lanes of a channel (segments of K = kChunk/S
// steps). Per state n each lane summarises its segment as the affine map h -> Al * h + Bl and the
// lanes combine those maps with a Kogge-Stone shuffle scan (width S, earlier segments first).
//
// Accuracy: Al is exp(A * sum(dt)) evaluated ONCE per segment (with the accurate expf) rather than
// the product of the K per-step fast-exp2 factors, and the state handed to the next segment /
// chunk is derived from the scanned segment maps. Long-range decay therefore passes through about
// L/K accurately rounded exponentials instead of L fast ones. This matters for channels with a
// long memory (|A dt| << 1): there every factor is close to 1, where the SFU's exp2 has an error
// of a few ulp with a consistent sign, and thousands of them would compound.
#pragma once

#include "common.cuh"

namespace mb200 {

constexpr unsigned kFullMask = 0xffffffffu;

// exp(A * sdt) for a segment whose dt sum is sdt. A segment whose steps all have dt == 0 (padding
// past seqlen) is the identity even when A is infinite.
__device__ __forceinline__ float seg_decay(float A, float sdt) { return sdt == 0.f ? 1.f : expf(A * sdt); }

// Inclusive scan (earlier segments first) of (A, B): afterwards lane s holds the composition of
// segments 0..s. Composition of an earlier map (Ap, Bp) with a later (A, B): (A Ap, A Bp + B).
template <int S>
__device__ __forceinline__ void scan_up(int s, float& A, float& B) {
#pragma unroll
  for (int off = 1; off < S; off <<= 1) {
    const float Ap = __shfl_up_sync(kFullMask, A, off, S);
    const float Bp = __shfl_up_sync(kFullMask, B, off, S);
    if (s >= off) {
      B = fmaf(A, Bp, B);
      A *= Ap;
    }
  }
}

// Reverse inclusive scan (later segments first): afterwards lane s holds the composition of
// segments s..S-1 applied from the end, i.e. the map gh_in(chunk end) -> gh_out(segment s start).
template <int S>
__device__ __forceinline__ void scan_down(int s, float& A, float& B) {
#pragma unroll
  for (int off = 1; off < S; off <<= 1) {
    const float An = __shfl_down_sync(kFullMask, A, off, S);
    const float Bn = __shfl_down_sync(kFullMask, B, off, S);
    if (s + off < S) {
      B = fmaf(A, Bn, B);
      A *= An;
    }
  }
}

// scan_up / scan_down of two independent states at once (their shuffles and FMAs interleave).
template <int S>
__device__ __forceinline__ void scan_up2(int s, float (&A)[2], float (&B)[2]) {
#pragma unroll
  for (int off = 1; off < S; off <<= 1) {
    float Ap[2], Bp[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      Ap[j] = __shfl_up_sync(kFullMask, A[j], off, S);
      Bp[j] = __shfl_up_sync(kFullMask, B[j], off, S);
    }
    if (s >= off) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        B[j] = fmaf(A[j], Bp[j], B[j]);
        A[j] *= Ap[j];
      }
    }
  }
}

template <int S>
__device__ __forceinline__ void scan_down2(int s, float (&A)[2], float (&B)[2]) {
#pragma unroll
  for (int off = 1; off < S; off <<= 1) {
    float An[2], Bn[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      An[j] = __shfl_down_sync(kFullMask, A[j], off, S);
      Bn[j] = __shfl_down_sync(kFullMask, B[j], off, S);
    }
    if (s + off < S) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        B[j] = fmaf(A[j], Bn[j], B[j]);
        A[j] *= An[j];
      }
    }
  }
}

}  // namespace mb200
