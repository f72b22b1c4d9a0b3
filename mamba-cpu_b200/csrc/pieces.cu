// pieces.cu -- summaries of sequence pieces for the scans (rows split over CTAs).
//
// When a call's rows give too few CTAs to fill the GPU, the forward and backward kernels cut each
// row into `pieces` runs of whole 64-step chunks (ScanArgs::pieces / piece_chunks). The recurrence
// is affine in its initial value -- forward h_end = P h_start + e, backward (the adjoint, run from
// the end) g_start = P g_end + G -- so every piece can start from the value its neighbours leave
// once their summaries (P, e) / (P, G) from a zero start are known. This kernel computes them:
//   * forward: pieces 0 .. pieces - 2, h_t = a_t h_{t-1} + dt_t u_t B_t from h = 0;
//   * backward: pieces 1 .. pieces - 1, g_{t-1} = a_t (g_t + dy_t C_t) from g = 0, dy_t = dout_t *
//     silu(z_t) (dout_t without z);
// with a_t = exp(dt_t A), dt_t = softplus(delta_t + bias) (or delta_t + bias).
//
// Work decomposition: one CTA per (piece, batch-group slice, 8 channels); the piece's chunks are
// cut into 16 consecutive runs, 4 per warp (lane = run-in-warp * 8 + channel), and each lane walks
// its run in the recurrence's direction with all states of its channel at once (dt and the inputs
// are computed once per step). Per chunk a warp stages the B (forward) or C (backward) tiles of its
// 4 runs' current chunks in shared memory with 16-byte loads all in flight, and each lane
// prefetches its next four steps of the row inputs while it computes the current ones. A lane
// starts every chunk from zero and composes it into its run with the chunk's exact decay
// expf(A sum dt) -- the same per-chunk decay the scan kernels apply to carried values, so the
// summaries agree with them to rounding. The 16 runs are then composed in chunk order through
// shared memory. Composition is associative (earlier run e, later run l):
//   forward  (P_e P_l, P_l e_e + e_l)       backward  (P_e P_l, P_e G_l + G_e).
#include "quad.cuh"
#include "scan.cuh"
#include "segscan.cuh"

namespace mb200 {

namespace {

constexpr int kSumCh = 8;                          // channels per CTA (and per warp)
constexpr int kSumRunsWarp = 32 / kSumCh;          // runs per warp
constexpr int kSumWarps = 4;
constexpr int kSumThreads = kSumWarps * 32;
constexpr int kSumRuns = kSumWarps * kSumRunsWarp;  // runs per piece

// Shared memory: per warp, the tiles (dstate x 64 steps) of its runs' current chunks, each tile
// padded by 16 bytes so the 4 runs' rows fall in different banks; reused after the walk for the
// runs' summaries (kSumRuns x kSumCh x dstate x {P, S} floats).
template <typename TW>
struct SumShape {
  static constexpr int kTileElems = kMaxState * kChunk + 16 / (int)sizeof(TW);
  static constexpr size_t kTileBytes = (size_t)kSumWarps * kSumRunsWarp * kTileElems * sizeof(TW);
  static constexpr size_t kCombBytes = (size_t)2 * kSumRuns * kSumCh * kMaxState * sizeof(float);
  static constexpr size_t kBytes = kTileBytes > kCombBytes ? kTileBytes : kCombBytes;
};

template <typename T>
__device__ __forceinline__ Quad<T> row_quad(const T* row, int64_t t, int64_t L, bool vec) {
  // four steps t .. t + 3 of a row (zeros past L); vec: dense, aligned and inside the row
  if (vec && t + 4 <= L) return ld_quad_cached(row + t);
  return ld_quad_masked(row, t, L, 1);
}

template <typename TI, typename TW, bool BWD, bool HAS_Z, bool STRIDED>
__global__ void __launch_bounds__(kSumThreads) scan_piece_summary_kernel(const ScanArgs f, const TI* dout,
                                                                         float* outS, float* outP, int rgroups,
                                                                         float* part) {
  using Sh = SumShape<TW>;
  extern __shared__ __align__(16) unsigned char sum_smem[];
  // blockIdx.x = ((piece * slices + slice) * groups + grp) * rgroups + rg: the CTA takes runs
  // [rg * kSumRuns, (rg + 1) * kSumRuns) of the piece's rgroups * kSumRuns runs
  const int64_t slices = f.batch * f.ngroups;
  const int64_t groups = (f.dpg + kSumCh - 1) / kSumCh;
  const int rg = (int)(blockIdx.x % rgroups);
  const int64_t item = blockIdx.x / rgroups;
  const int64_t grp = item % groups;
  const int64_t slice = (item / groups) % slices;
  const int piece = (int)(item / groups / slices) + (BWD ? 1 : 0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ch = lane % kSumCh, rw = lane / kSumCh;  // channel slot, run within the warp
  const int run = warp * kSumRunsWarp + rw;
  const int N = (int)f.N;
  const int64_t L = f.L;
  const int64_t rows = f.batch * f.dim;
  const int64_t b = slice / f.ngroups, g = slice % f.ngroups;
  const int64_t cig = grp * kSumCh + ch;
  const int64_t d = g * f.dpg + (cig < f.dpg ? cig : 0);  // slots past the group's channels repeat one
  const int64_t row = b * f.dim + d;

  // runs of the piece's chunks: run r = [k_lo + r m, k_lo + (r + 1) m) clipped to the piece; this
  // CTA's run i is the piece's run rg * kSumRuns + i
  const int k_lo = piece * f.piece_chunks;
  const int k_hi = min(f.nchunks, k_lo + f.piece_chunks);
  const int m = (k_hi - k_lo + kSumRuns * rgroups - 1) / (kSumRuns * rgroups);
  auto run_lo = [&](int r) { return min(k_hi, k_lo + (rg * kSumRuns + r) * m); };
  auto run_len = [&](int r) { return min(k_hi, run_lo(r) + m) - run_lo(r); };
  const int ca = run_lo(run), len = run_len(run);
  const int wlen = run_len(warp * kSumRunsWarp);  // the warp's longest run (its first)

  const TI* drow = static_cast<const TI*>(f.delta) + (STRIDED ? b * f.sdb + d * f.sdd : row * L);
  // forward: u; backward: dout (dense rows) and z
  const TI* xrow = BWD ? dout + row * L : static_cast<const TI*>(f.u) + (STRIDED ? b * f.sub + d * f.sud : row * L);
  const TI* zrow = HAS_Z ? static_cast<const TI*>(f.z) + (STRIDED ? b * f.szb + d * f.szd : row * L) : nullptr;
  const TW* Mb = BWD ? static_cast<const TW*>(f.C) + b * f.sCb + g * f.sCg
                     : static_cast<const TW*>(f.B) + b * f.sBb + g * f.sBg;
  const int64_t sMn = BWD ? f.sCn : f.sBn, sMl = BWD ? f.sCl : f.sBl;
  const bool vio = f.vec_io != 0, vbc = f.vec_bc != 0;
  const float bias = f.delta_bias ? f.delta_bias[d] : 0.f;
  TW* tiles = reinterpret_cast<TW*>(sum_smem) + (size_t)warp * kSumRunsWarp * Sh::kTileElems;
  const TW* mytile = tiles + (size_t)rw * Sh::kTileElems;

  float Aj[kMaxState], P[kMaxState], S[kMaxState];
#pragma unroll
  for (int n = 0; n < kMaxState; ++n) {
    Aj[n] = n < N ? f.A[d * N + n] : 0.f;
    P[n] = 1.f;
    S[n] = 0.f;
  }

  for (int ci = 0; ci < wlen; ++ci) {
    // -- stage the tiles of the warp's runs' chunk ci (runs shorter than ci + 1 load nothing)
    __syncwarp();
    {
      constexpr int kVec = 16 / (int)sizeof(TW);     // elements per 16-byte piece
      constexpr int kPer = kChunk / kVec;            // pieces per tile row
      for (int j = lane; j < kSumRunsWarp * N * kPer; j += 32) {
        const int r = j / (N * kPer), n = (j / kPer) % N, v = j % kPer;
        const int rr = warp * kSumRunsWarp + r;
        if (ci >= run_len(rr)) continue;
        const int k = BWD ? run_lo(rr) + run_len(rr) - 1 - ci : run_lo(rr) + ci;
        const int64_t t = (int64_t)k * kChunk + v * kVec;
        TW* dst = tiles + (size_t)r * Sh::kTileElems + n * kChunk + v * kVec;
        const TW* src = Mb + n * sMn;
        if (vbc && t + kVec <= L) {
          *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src + t));
        } else {
#pragma unroll
          for (int e = 0; e < kVec; ++e) dst[e] = t + e < L ? src[(t + e) * sMl] : from_f32<TW>(0.f);
        }
      }
    }
    __syncwarp();
    if (ci >= len) continue;
    const int k = BWD ? ca + len - 1 - ci : ca + ci;
    const int64_t c0 = (int64_t)k * kChunk;
    const int nq = (int)((min(L, c0 + kChunk) - c0 + 3) / 4);  // quads of this chunk inside the row
    float loc[kMaxState];
#pragma unroll
    for (int n = 0; n < kMaxState; ++n) loc[n] = 0.f;
    float sdt = 0.f;
    auto quad_t = [&](int qi) { return c0 + 4 * (BWD ? nq - 1 - qi : qi); };
    Quad<TI> qd = row_quad<TI>(drow, quad_t(0), L, vio), qx = row_quad<TI>(xrow, quad_t(0), L, vio), qz{};
    if constexpr (HAS_Z) qz = row_quad<TI>(zrow, quad_t(0), L, vio);
    for (int qi = 0; qi < nq; ++qi) {
      const int64_t t = quad_t(qi);
      const float4 dl = to_float4(qd), xv = to_float4(qx);
      float4 zv = make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (HAS_Z) zv = to_float4(qz);
      if (qi + 1 < nq) {  // the next four steps load while these are computed
        const int64_t tn = quad_t(qi + 1);
        qd = row_quad<TI>(drow, tn, L, vio);
        qx = row_quad<TI>(xrow, tn, L, vio);
        if constexpr (HAS_Z) qz = row_quad<TI>(zrow, tn, L, vio);
      }
      float dt[4] = {dl.x, dl.y, dl.z, dl.w};
      float in[4] = {xv.x, xv.y, xv.z, xv.w};
      const float zz[4] = {zv.x, zv.y, zv.z, zv.w};
      float dtl[4];  // dt * log2(e): a = 2^(dtl A)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool live = t + e < L;
        float v = dt[e] + bias;
        v = f.softplus ? softplus_f(v) : v;
        dt[e] = live ? v : 0.f;  // a step past the row end: a = 1, no input
        dtl[e] = dt[e] * kLog2e;
        sdt += dt[e];
        if constexpr (BWD) {
          if constexpr (HAS_Z) in[e] *= silu_f(zz[e]);
        } else {
          in[e] *= dt[e];  // dt * u
        }
        in[e] = live ? in[e] : 0.f;
      }
      const int tq = (int)(t - c0);
#pragma unroll
      for (int n = 0; n < kMaxState; ++n) {
        if (n >= N) continue;
        const float4 mv = to_float4(*reinterpret_cast<const Quad<TW>*>(mytile + n * kChunk + tq));
        const float mm[4] = {mv.x, mv.y, mv.z, mv.w};
        if constexpr (BWD) {
#pragma unroll
          for (int e = 3; e >= 0; --e) loc[n] = ex2(dtl[e] * Aj[n]) * fmaf(in[e], mm[e], loc[n]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) loc[n] = fmaf(ex2(dtl[e] * Aj[n]), loc[n], in[e] * mm[e]);
        }
      }
    }
    // compose the chunk into the run (same form in both directions: the chunk comes after the
    // chunks already folded, in the recurrence's order)
#pragma unroll
    for (int n = 0; n < kMaxState; ++n) {
      const float exact = seg_decay(Aj[n], sdt);
      S[n] = fmaf(exact, S[n], loc[n]);
      P[n] *= exact;
    }
  }

  // compose the runs in chunk order (run r is earlier than run r + 1) through shared memory
  __syncthreads();  // every warp is done with its tiles
  float* sP = reinterpret_cast<float*>(sum_smem);              // [run][n][channel]
  float* sS = sP + kSumRuns * kMaxState * kSumCh;
#pragma unroll
  for (int n = 0; n < kMaxState; ++n) {
    sP[(run * kMaxState + n) * kSumCh + ch] = P[n];
    sS[(run * kMaxState + n) * kSumCh + ch] = S[n];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < kSumCh * N; idx += kSumThreads) {
    const int c = idx % kSumCh, n = idx / kSumCh;
    float Pe = sP[n * kSumCh + c], Se = sS[n * kSumCh + c];
    for (int r = 1; r < kSumRuns; ++r) {
      const float Pl = sP[(r * kMaxState + n) * kSumCh + c], Sl = sS[(r * kMaxState + n) * kSumCh + c];
      if constexpr (BWD)
        Se = fmaf(Pe, Sl, Se);
      else
        Se = fmaf(Pl, Se, Sl);
      Pe *= Pl;
    }
    if (grp * kSumCh + c < f.dpg) {
      const int64_t at = ((int64_t)piece * rows + b * f.dim + g * f.dpg + grp * kSumCh + c) * N + n;
      if (rgroups == 1) {
        outS[at] = Se;
        outP[at] = Pe;
      } else {  // this run group's part, composed with the others' by piece_combine_kernel
        part[(at * rgroups + rg) * 2] = Pe;
        part[(at * rgroups + rg) * 2 + 1] = Se;
      }
    }
  }
}

// Composes the run groups' parts of each (piece, row, state) in chunk order.
template <bool BWD>
__global__ void piece_combine_kernel(const float* part, int rgroups, int64_t first, int64_t count, float* outS,
                                     float* outP) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const int64_t at = first + i;
  float Pe = part[at * rgroups * 2], Se = part[at * rgroups * 2 + 1];
  for (int r = 1; r < rgroups; ++r) {
    const float Pl = part[(at * rgroups + r) * 2], Sl = part[(at * rgroups + r) * 2 + 1];
    if constexpr (BWD)
      Se = fmaf(Pe, Sl, Se);
    else
      Se = fmaf(Pl, Se, Sl);
    Pe *= Pl;
  }
  outS[at] = Se;
  outP[at] = Pe;
}

template <typename TI, typename TW, bool BWD>
cudaError_t launch_summary_t(const ScanArgs& f, const void* dout, float* outS, float* outP, cudaStream_t stream) {
  const int rgroups = summary_rgroups(f);
  const unsigned blocks =
      (unsigned)((int64_t)(f.pieces - 1) * f.batch * f.ngroups * ((f.dpg + kSumCh - 1) / kSumCh) * rgroups);
  const bool strided = io_rows_strided(f);
  const TI* go = static_cast<const TI*>(dout);
  auto kern = (BWD && f.z != nullptr) ? (strided ? scan_piece_summary_kernel<TI, TW, BWD, true, true>
                                                 : scan_piece_summary_kernel<TI, TW, BWD, true, false>)
                                      : (strided ? scan_piece_summary_kernel<TI, TW, BWD, false, true>
                                                 : scan_piece_summary_kernel<TI, TW, BWD, false, false>);
  constexpr size_t smem = SumShape<TW>::kBytes;
  // the attribute belongs to the current device: set on every launch
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<blocks, kSumThreads, smem, stream>>>(f, go, outS, outP, rgroups, f.piece_scratch);
  if (rgroups > 1) {
    const int64_t per = (f.pieces - 1) * f.batch * f.dim * f.N;  // the summaries written
    const int64_t first = BWD ? f.batch * f.dim * f.N : 0;        // the backward's start at piece 1
    piece_combine_kernel<BWD><<<(unsigned)((per + 255) / 256), 256, 0, stream>>>(f.piece_scratch, rgroups, first,
                                                                                  per, outS, outP);
  }
  return cudaGetLastError();
}

template <bool BWD>
cudaError_t launch_summary(const ScanArgs& f, const void* dout, float* outS, float* outP, int io_dtype,
                           int bc_dtype, cudaStream_t stream) {
  if (io_dtype == MB200_F32) return launch_summary_t<float, float, BWD>(f, dout, outS, outP, stream);
  if (io_dtype == MB200_BF16) {
    if (bc_dtype == MB200_BF16)
      return launch_summary_t<__nv_bfloat16, __nv_bfloat16, BWD>(f, dout, outS, outP, stream);
    return launch_summary_t<__nv_bfloat16, float, BWD>(f, dout, outS, outP, stream);
  }
  if (bc_dtype == MB200_F16) return launch_summary_t<__half, __half, BWD>(f, dout, outS, outP, stream);
  return launch_summary_t<__half, float, BWD>(f, dout, outS, outP, stream);
}

}  // namespace

int summary_rgroups(const ScanArgs& f) {
  // Runs of one chunk where the piece allows, up to 16 run groups: the summaries' ex2 work is the
  // same whatever the split, and more, shorter runs keep every SM's slots full to the end (one
  // rank's 8-rank c5 shard: 640 -> 532 us per backward summary, against the former rule of about
  // four rounds of resident CTAs and at most 8 groups).
  if (f.pieces <= 1) return 1;
  int rg = (f.piece_chunks + kSumRuns - 1) / kSumRuns;
  if (rg > 16) rg = 16;
  return rg < 1 ? 1 : rg;
}

size_t summary_scratch_floats(const ScanArgs& f) {
  const int rg = summary_rgroups(f);
  if (rg <= 1) return 0;
  return (size_t)f.pieces * f.batch * f.dim * f.N * rg * 2;
}

cudaError_t launch_fwd_piece_summary(const ScanArgs& f, int io_dtype, int bc_dtype, cudaStream_t stream) {
  if (f.pieces <= 1 || f.batch == 0 || f.dim == 0) return cudaSuccess;
  return launch_summary<false>(f, nullptr, f.piece_e, f.piece_P, io_dtype, bc_dtype, stream);
}

cudaError_t launch_bwd_piece_summary(const BwdArgs& a, int io_dtype, int bc_dtype, cudaStream_t stream) {
  if (a.f.pieces <= 1 || a.f.batch == 0 || a.f.dim == 0) return cudaSuccess;
  return launch_summary<true>(a.f, a.dout, a.piece_G, a.piece_P, io_dtype, bc_dtype, stream);
}

}  // namespace mb200
