// scan_fwd.cu -- forward selective scan on sm_100a.
//
// Computes, for every row (batch b, channel d) and timestep t (mamba-cpu
// csrc/selective_scan.cpp:120-145 states the same recurrence as a sequential CPU loop):
//   dt_t = softplus(delta_t + bias_d)            (or delta_t + bias_d without softplus)
//   h_t  = exp(dt_t * A_d) * h_{t-1} + dt_t * u_t * B_t      (dstate lanes of h, h_{-1} = 0)
//   y_t  = <h_t, C_t> + D_d * u_t ;  out_t = y_t * silu(z_t)  (the gate only when z is given)
//
// Work decomposition (time-parallel within a warp):
//   * a warp owns CW = 32 / S channels; the S lanes of a channel split each 64-step chunk into S
//     segments of K = 64 / S consecutive timesteps;
//   * for each state n the lane forms the affine map of its K steps, h -> Al * h + Bl, the S
//     segments are combined with a log2(S)-step shuffle scan of these maps (segscan.cuh), and the
//     lane then re-applies its K steps from the exact start state. exp(dt * A) is evaluated once
//     per (t, n) and kept in registers between the two uses;
//   * the chunk-end state (from the scanned segment maps) is carried in registers to the next
//     chunk and optionally written to chunk_states, which the backward uses as restart points.
// Data movement: the B/C tile of a chunk (dstate rows x 64 steps, shared by every channel of the
// CTA) is staged in shared memory by the bulk-copy engine one chunk ahead (double buffer,
// mbarrier completion); each lane's own u / delta / z items are prefetched one chunk ahead into
// registers with 16-byte streaming loads. Full chunks run unmasked; a partial last chunk, or
// rows that are not 16-byte aligned, take the masked direct-load path.
#include "scan.cuh"
#include "segscan.cuh"
#include "stage.cuh"

namespace mb200 {

namespace {

constexpr unsigned kFull = 0xffffffffu;

template <typename TI, typename TW, int S>
struct FwdCtx {
  const TW* Bbase;
  const TW* Cbase;
  int64_t sBn, sBl, sCn, sCl;
  int64_t L;
  int N;
  int s;
  bool vec_bc;
};

// B (or C) items of state n for this lane's K steps, from the staged tile or from global memory.
template <typename TW, int K, bool STAGED, bool MASKED>
__device__ __forceinline__ void bc_items(const TW* tile_row, const TW* grow, int64_t stride, int64_t t0, int64_t L,
                                         bool vec, float (&x)[K]) {
  if constexpr (STAGED) {
    load_cached_smem<TW, K>(tile_row, x);
  } else if constexpr (MASKED) {
    load_bc_items<TW, K>(grow, stride, t0, L, false, x);
  } else {
    load_bc_items<TW, K>(grow, stride, t0, L, vec, x);
  }
}

template <typename TI, typename TW, int S, bool HAS_Z, bool WRITE_OUT, bool STAGED, bool MASKED>
__device__ __forceinline__ void fwd_chunk(const FwdCtx<TI, TW, S>& x, int k, const float (&u)[kChunk / S],
                                          const float (&dl)[kChunk / S], const float (&zz)[kChunk / S],
                                          const TW* sB, const TW* sC, const float* Av, float Dv, float bias,
                                          bool softplus, float* hc, float* st_out, float (&y)[kChunk / S]) {
  constexpr int K = kChunk / S;
  const int64_t t0 = (int64_t)k * kChunk + x.s * K;
  float dt[K], dtu[K];
  float sdt = 0.f;
#pragma unroll
  for (int i = 0; i < K; ++i) {
    float v = dl[i] + bias;
    v = softplus ? softplus_f(v) : v;
    if (MASKED) v = (t0 + i < x.L) ? v : 0.f;
    dt[i] = v;
    dtu[i] = v * u[i];
    y[i] = Dv * u[i];
    sdt += v;
  }
#pragma unroll
  for (int n = 0; n < kMaxState; ++n) {
    if (n < x.N) {
      float Bn[K], Cn[K], av[K], bv[K];
      constexpr int kRS = TileRow<TW>::kStride;
      const int tpos = TileRow<TW>::pos(x.s * K);
      bc_items<TW, K, STAGED, MASKED>(sB + n * kRS + tpos, x.Bbase + n * x.sBn, x.sBl, t0, x.L, x.vec_bc, Bn);
      if (WRITE_OUT)
        bc_items<TW, K, STAGED, MASKED>(sC + n * kRS + tpos, x.Cbase + n * x.sCn, x.sCl, t0, x.L, x.vec_bc, Cn);
      const float An = Av[n];
      const float A2n = An * kLog2e;
#pragma unroll
      for (int i = 0; i < K; ++i) {
        av[i] = ex2(dt[i] * A2n);
        bv[i] = dtu[i] * Bn[i];
      }
      if (MASKED) {  // steps past seqlen are the identity map (a = 1, b = 0)
#pragma unroll
        for (int i = 0; i < K; ++i)
          if (t0 + i >= x.L) {
            av[i] = 1.f;
            bv[i] = 0.f;
          }
      }
      float Al = seg_decay(An, sdt), Bl = bv[0];
#pragma unroll
      for (int i = 1; i < K; ++i) Bl = fmaf(av[i], Bl, bv[i]);
      float h;
      if constexpr (S > 1) {
        scan_up<S>(x.s, Al, Bl);
        float Ae = __shfl_up_sync(kFull, Al, 1, S);
        float Be = __shfl_up_sync(kFull, Bl, 1, S);
        if (x.s == 0) {
          Ae = 1.f;
          Be = 0.f;
        }
        h = fmaf(Ae, hc[n], Be);
      } else {
        h = hc[n];
      }
      __syncwarp();  // every lane of the channel has read hc[n] before the last lane updates it
#pragma unroll
      for (int i = 0; i < K; ++i) {
        h = fmaf(av[i], h, bv[i]);
        if (WRITE_OUT) y[i] = fmaf(h, Cn[i], y[i]);
      }
      // next chunk's start state: the scanned map of the whole chunk applied to this one's. The
      // last segment lane holds it; it becomes visible to the channel's other lanes after the
      // warp / block synchronisation that ends the chunk.
      if (x.s == S - 1) {
        const float hn = fmaf(Al, hc[n], Bl);
        hc[n] = hn;
        if (st_out != nullptr) st_out[n] = hn;
      }
    }
  }
  if (WRITE_OUT && HAS_Z) {
#pragma unroll
    for (int i = 0; i < K; ++i) y[i] *= zz[i] * sigmoid_f(zz[i]);
  }
}

template <typename TI, typename TW, int S, bool HAS_Z, bool WRITE_OUT>
__global__ void __launch_bounds__(kFwdWarps * 32, 3) scan_fwd_kernel(const ScanArgs a) {
  constexpr int K = kChunk / S;
  constexpr int CW = 32 / S;
  constexpr int CPC = kFwdWarps * CW;  // channels per CTA
  extern __shared__ __align__(128) unsigned char smem_raw[];
  constexpr int kRS = TileRow<TW>::kStride;
  TW* sB = reinterpret_cast<TW*>(smem_raw);  // [2][kMaxState][kRS]
  TW* sC = sB + 2 * kMaxState * kRS;         // [2][kMaxState][kRS]
  float* sA = reinterpret_cast<float*>(sC + 2 * kMaxState * kRS);  // [CPC][kMaxState]: A rows
  float* sH = sA + CPC * kMaxState;                                  // [CPC][kMaxState]: carried state
  uint64_t* bar = reinterpret_cast<uint64_t*>(sH + CPC * kMaxState);

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int c = lane / S;
  const int s = lane % S;
  const int64_t tile = blockIdx.x % a.tiles;
  const int64_t slice = blockIdx.x / a.tiles;
  const int64_t b = slice / a.ngroups;
  const int64_t g = slice % a.ngroups;
  const int64_t cig = tile * CPC + warp * CW + c;  // channel index inside the group
  const bool valid = cig < a.dpg;
  const int64_t d = g * a.dpg + (valid ? cig : 0);  // masked lanes read a real row, store nothing
  const int64_t row = b * a.dim + d;
  const int64_t L = a.L;
  const int N = (int)a.N;

  FwdCtx<TI, TW, S> x;
  x.Bbase = static_cast<const TW*>(a.B) + b * a.sBb + g * a.sBg;
  x.Cbase = static_cast<const TW*>(a.C) + b * a.sCb + g * a.sCg;
  x.sBn = a.sBn;
  x.sBl = a.sBl;
  x.sCn = a.sCn;
  x.sCl = a.sCl;
  x.L = L;
  x.N = N;
  x.s = s;
  x.vec_bc = a.vec_bc != 0;

  const TI* urow = static_cast<const TI*>(a.u) + row * L;
  const TI* drow = static_cast<const TI*>(a.delta) + row * L;
  const TI* zrow = HAS_Z ? static_cast<const TI*>(a.z) + row * L : nullptr;
  TI* orow = WRITE_OUT ? static_cast<TI*>(a.out) + row * L : nullptr;

  const int cl = warp * CW + c;  // this channel's slot in the CTA
  float* Av = sA + cl * kMaxState;
  float* hc = sH + cl * kMaxState;
  if (s == 0) {
    for (int n = 0; n < N; ++n) {
      Av[n] = a.A[d * N + n];
      hc[n] = 0.f;
    }
  }
  const float Dv = a.D ? a.D[d] : 0.f;
  const float bias = a.delta_bias ? a.delta_bias[d] : 0.f;
  const bool vec_io = a.vec_io != 0;
  const bool softplus = a.softplus != 0;
  const bool staged = a.vec_bc != 0;

  // Full chunks of 16-byte aligned rows with a stageable B/C tile run unmasked from shared memory;
  // everything else (partial last chunk, unaligned rows, strided B/C) takes the masked path.
  const int nfull = (vec_io && staged) ? (int)(L / kChunk) : 0;

  if (staged && threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_fence_init();
  }
  __syncthreads();

  auto issue_bc = [&](int k, int buf) {
    // Each row in two halves (the second shifted by TileRow::kShift elements).
    constexpr uint32_t half_bytes = kChunk / 2 * sizeof(TW);
    const int rows = WRITE_OUT ? 2 * N : N;
    if (lane == 0) mbar_arrive_expect_tx(&bar[buf], rows * 2 * half_bytes);
    __syncwarp();
    fence_proxy_async();
    for (int j = lane; j < 2 * rows; j += 32) {
      const int r = j >> 1, hf = j & 1;
      const bool isC = r >= N;
      const int n = isC ? r - N : r;
      const TW* src = (isC ? x.Cbase + n * x.sCn : x.Bbase + n * x.sBn) + (int64_t)k * kChunk + hf * (kChunk / 2);
      TW* dst = (isC ? sC : sB) + (buf * kMaxState + n) * kRS + TileRow<TW>::pos(hf * (kChunk / 2));
      bulk_g2s(dst, src, half_bytes, &bar[buf]);
    }
  };

  float nu[K], nd[K], nz[K];
  if (nfull > 0) {
    load_stream<TI, K>(urow + s * K, nu);
    load_stream<TI, K>(drow + s * K, nd);
    if constexpr (HAS_Z && WRITE_OUT) load_stream<TI, K>(zrow + s * K, nz);
    if (warp == 0) issue_bc(0, 0);
  }
  for (int k = 0; k < nfull; ++k) {
    const int buf = k & 1;
    float u[K], dl[K], zz[K];
#pragma unroll
    for (int i = 0; i < K; ++i) {
      u[i] = nu[i];
      dl[i] = nd[i];
      if constexpr (HAS_Z) zz[i] = nz[i];
    }
    if (k + 1 < nfull) {
      const int64_t t1 = (int64_t)(k + 1) * kChunk + s * K;
      load_stream<TI, K>(urow + t1, nu);
      load_stream<TI, K>(drow + t1, nd);
      if constexpr (HAS_Z && WRITE_OUT) load_stream<TI, K>(zrow + t1, nz);
      if (warp == 0) issue_bc(k + 1, buf ^ 1);
    }
    float y[K];
    mbar_wait(&bar[buf], (k >> 1) & 1);
    float* st = (a.chunk_states != nullptr && valid) ? a.chunk_states + (row * a.nchunks + k) * N : nullptr;
    fwd_chunk<TI, TW, S, HAS_Z, WRITE_OUT, true, false>(x, k, u, dl, zz, sB + buf * kMaxState * kRS,
                                                        sC + buf * kMaxState * kRS, Av, Dv, bias, softplus, hc, st,
                                                        y);
    const int64_t t0 = (int64_t)k * kChunk + s * K;
    if (WRITE_OUT && valid) store_stream<TI, K>(orow + t0, y);
    __syncthreads();  // every lane is done with this B/C buffer before it is refilled
  }
  // Remaining chunks (a partial last chunk, or all chunks of an unaligned row): masked path.
  for (int k = nfull; k < a.nchunks; ++k) {
    const int64_t t0 = (int64_t)k * kChunk + s * K;
    float u[K], dl[K], zz[K], y[K];
    load_items<TI, K>(urow, t0, L, false, 0.f, u);
    load_items<TI, K>(drow, t0, L, false, 0.f, dl);
    if constexpr (HAS_Z && WRITE_OUT) load_items<TI, K>(zrow, t0, L, false, 0.f, zz);
    float* st = (a.chunk_states != nullptr && valid) ? a.chunk_states + (row * a.nchunks + k) * N : nullptr;
    fwd_chunk<TI, TW, S, HAS_Z, WRITE_OUT, false, true>(x, k, u, dl, zz, nullptr, nullptr, Av, Dv, bias, softplus,
                                                        hc, st, y);
    if (WRITE_OUT && valid) store_items<TI, K>(orow, t0, L, false, y);
    __syncwarp();
  }
  __syncwarp();
  if (a.last_state != nullptr && valid && s == 0) {
    float* st = a.last_state + row * N;
    for (int n = 0; n < N; ++n) st[n] = hc[n];
  }
}

template <typename TW, int S>
constexpr size_t fwd_smem_bytes() {
  return 2 * 2 * kMaxState * TileRow<TW>::kStride * sizeof(TW) + 2 * kFwdWarps * (32 / S) * kMaxState * sizeof(float) +
         2 * sizeof(uint64_t);
}

template <typename TI, typename TW, int S, bool HAS_Z, bool WRITE_OUT>
cudaError_t launch_one(const ScanArgs& a, dim3 grid, cudaStream_t stream) {
  auto kern = scan_fwd_kernel<TI, TW, S, HAS_Z, WRITE_OUT>;
  constexpr size_t smem = fwd_smem_bytes<TW, S>();
  static bool attr_set = false;  // per instantiation; setting it twice is harmless
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  kern<<<grid, kFwdWarps * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

template <typename TI, typename TW, int S>
cudaError_t launch_typed(ScanArgs a, bool write_out, cudaStream_t stream) {
  constexpr int CPC = kFwdWarps * (32 / S);
  a.tiles = (int)((a.dpg + CPC - 1) / CPC);
  const dim3 grid((unsigned)(a.tiles * a.batch * a.ngroups));
  if (!write_out) return launch_one<TI, TW, S, false, false>(a, grid, stream);
  if (a.z != nullptr) return launch_one<TI, TW, S, true, true>(a, grid, stream);
  return launch_one<TI, TW, S, false, true>(a, grid, stream);
}

template <typename TI, typename TW>
cudaError_t launch_seg(const ScanArgs& a, bool write_out, cudaStream_t stream) {
  if (fwd_segments(a.batch * a.dim) == 8) return launch_typed<TI, TW, 8>(a, write_out, stream);
  return launch_typed<TI, TW, 16>(a, write_out, stream);
}

}  // namespace

int fwd_segments(int64_t rows) {
  // Enough resident warps to keep every SM sub-partition busy: 148 SMs x 4 x ~4 warps.
  return rows >= 4096 ? 8 : 16;
}

cudaError_t read_fault_fwd(int* out) { return read_fault_word(out); }

cudaError_t launch_scan_fwd(const ScanArgs& a, int io_dtype, int bc_dtype, bool write_out,
                            cudaStream_t stream) {
  if (a.batch == 0 || a.dim == 0) return cudaSuccess;
  if (io_dtype == MB200_F32) return launch_seg<float, float>(a, write_out, stream);
  if (io_dtype == MB200_BF16) {
    if (bc_dtype == MB200_BF16) return launch_seg<__nv_bfloat16, __nv_bfloat16>(a, write_out, stream);
    return launch_seg<__nv_bfloat16, float>(a, write_out, stream);
  }
  if (bc_dtype == MB200_F16) return launch_seg<__half, __half>(a, write_out, stream);
  return launch_seg<__half, float>(a, write_out, stream);
}

}  // namespace mb200
