// scan_bwd.cu -- backward selective scan on sm_100a.
//
// Gradients of the recurrence of scan_fwd.cu (mamba-cpu csrc/selective_scan.cpp:168-248 states
// them as a sequential CPU loop): with G_t = dLoss/dh_t and gh_t = a_{t+1} G_{t+1} (gh after the
// last step = dlast_state),
//   G_t   = gh_t + dy_t C_t            dy_t = dout_t * silu(z_t)   (dout_t without z)
//   dC_t += dy_t h_t                   dB_t += G_t dt_t u_t         (summed over the group's channels)
//   x_t   = G_t a_t h_{t-1}            dA   += x_t dt_t
//   ddt_t = (sum_n x_t A + u_t sum_n G_t B_t) * softplus'(delta_t + bias)
//   du_t  = D dy_t + dt_t sum_n G_t B_t,   dD += dy_t u_t,   dz_t = dout_t y_t silu'(z_t)
//
// Work decomposition:
//   * the same warp layout as the forward (CW channels x S time segments of K steps per chunk);
//   * chunks are visited from the last to the first. Each chunk restarts from the state the
//     forward saved at its start (chunk_states), so no seqlen x dstate history is materialised;
//   * per state n: a forward shuffle scan rebuilds h inside the chunk (a_t kept in registers),
//     a reverse shuffle scan of (a, gh) pairs carries gh across segments and chunks, then each
//     lane walks its K steps backwards accumulating the gradients;
//   * dB/dC (sums over channels) are reduced deterministically: a reduce-scatter over the CW
//     channel lanes of the warp (shuffles), a sum over the warps of the CTA (shared memory), a
//     sum over the CTAs of a thread-block cluster (distributed shared memory), and finally a sum
//     over clusters by the reduce kernel below. dA / dD / ddelta_bias leave the kernel as
//     per-row partials and are summed over batch by the same reduce kernel.
#include <cooperative_groups.h>

#include "scan.cuh"

namespace cg = cooperative_groups;

namespace mb200 {

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kRedFloats = kMaxState * 2 * kChunk;  // one CTA's dB|dC chunk partial (2048)

constexpr int ilog2(int v) { return v <= 1 ? 0 : 1 + ilog2(v / 2); }

template <typename TI, typename TW, int S, bool HAS_Z>
__global__ void __launch_bounds__(kBwdWarps * 32, 2) scan_bwd_kernel(const BwdArgs a) {
  constexpr int K = kChunk / S;
  constexpr int CW = 32 / S;
  constexpr int CPC = kBwdWarps * CW;
  constexpr int R = ilog2(CW);  // reduce-scatter rounds over the channel lanes
  static_assert(S >= 2 && S <= 16, "segments per channel");
  static_assert((2 * K) >> R == 4, "each lane ends the reduce-scatter with one float4");

  __shared__ __align__(16) float red[kBwdWarps][kRedFloats];
  __shared__ __align__(16) float red_out[2][kRedFloats];

  cg::cluster_group cluster = cg::this_cluster();
  const int CL = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();

  const ScanArgs& f = a.f;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int c = lane / S;
  const int s = lane % S;
  const int64_t tile = blockIdx.x % f.tiles;
  const int64_t slice = blockIdx.x / f.tiles;
  const int64_t b = slice / f.ngroups;
  const int64_t g = slice % f.ngroups;
  const int64_t cluster_idx = tile / CL;
  const int64_t cig = tile * CPC + warp * CW + c;
  const bool valid = cig < f.dpg;
  const int64_t d = g * f.dpg + (valid ? cig : 0);
  const int64_t row = b * f.dim + d;
  const int64_t L = f.L;
  const int N = (int)f.N;
  const int nchunks = f.nchunks;

  const TI* urow = static_cast<const TI*>(f.u) + row * L;
  const TI* drow = static_cast<const TI*>(f.delta) + row * L;
  const TI* zrow = HAS_Z ? static_cast<const TI*>(f.z) + row * L : nullptr;
  const TI* dorow = static_cast<const TI*>(a.dout) + row * L;
  TI* durow = static_cast<TI*>(a.du) + row * L;
  TI* ddrow = static_cast<TI*>(a.ddelta) + row * L;
  TI* dzrow = HAS_Z ? static_cast<TI*>(a.dz) + row * L : nullptr;
  const TW* Bbase = static_cast<const TW*>(f.B) + b * f.sBb + g * f.sBg;
  const TW* Cbase = static_cast<const TW*>(f.C) + b * f.sCb + g * f.sCg;
  const float* Arow = f.A + d * N;
  const float Dv = f.D ? f.D[d] : 0.f;
  const float bias = f.delta_bias ? f.delta_bias[d] : 0.f;
  const bool vec_io = f.vec_io != 0;
  const bool vec_bc = f.vec_bc != 0;

  float gc[kMaxState];     // gh entering the current chunk from later timesteps
  float dAacc[kMaxState];  // this lane's share of dA for its row
#pragma unroll
  for (int n = 0; n < kMaxState; ++n) {
    gc[n] = (valid && a.dlast != nullptr && n < N) ? a.dlast[row * N + n] : 0.f;
    dAacc[n] = 0.f;
  }
  float dDacc = 0.f, dbacc = 0.f;
  int buf = 0;

  for (int k = nchunks - 1; k >= 0; --k) {
    const int64_t t0 = (int64_t)k * kChunk + s * K;
    const bool tail = t0 + K > L;
    float dt[K], dtu[K], dy[K], uu[K], dsp[K], gB[K], xA[K];
    float dzc[HAS_Z ? K : 1], y[HAS_Z ? K : 1];
    {
      float dl[K], dO[K];
      load_items<TI, K>(urow, t0, L, vec_io, 0.f, uu);
      load_items<TI, K>(drow, t0, L, vec_io, 0.f, dl);
      load_items<TI, K>(dorow, t0, L, vec_io, 0.f, dO);
      float zz[HAS_Z ? K : 1];
      if constexpr (HAS_Z) load_items<TI, K>(zrow, t0, L, vec_io, 0.f, zz);
#pragma unroll
      for (int i = 0; i < K; ++i) {
        const bool in = t0 + i < L;
        const float raw = dl[i] + bias;
        const float sp = f.softplus ? softplus_f(raw) : raw;
        dsp[i] = f.softplus ? sigmoid_f(raw) : 1.f;
        dt[i] = in ? sp : 0.f;
        dtu[i] = dt[i] * uu[i];
        float dyi = dO[i];
        if constexpr (HAS_Z) {
          const float zs = sigmoid_f(zz[i]);
          dyi = dO[i] * zz[i] * zs;
          dzc[i] = dO[i] * zs * (1.f + zz[i] * (1.f - zs));
          y[i] = Dv * uu[i];
        }
        dy[i] = valid ? dyi : 0.f;
        gB[i] = 0.f;
        xA[i] = 0.f;
      }
    }

#pragma unroll
    for (int n = 0; n < kMaxState; ++n) {
      if (n < N) {
        const float An = Arow[n];
        const float A2n = An * kLog2e;
        const float hck = k > 0 ? a.states[(row * nchunks + (k - 1)) * N + n] : 0.f;
        float Bn[K], Cn[K], av[K], hs[K];
        load_bc_items<TW, K>(Bbase + n * f.sBn, f.sBl, t0, L, vec_bc, Bn);
        load_bc_items<TW, K>(Cbase + n * f.sCn, f.sCl, t0, L, vec_bc, Cn);
#pragma unroll
        for (int i = 0; i < K; ++i) av[i] = ex2(dt[i] * A2n);
        if (tail) {
#pragma unroll
          for (int i = 0; i < K; ++i)
            if (t0 + i >= L) av[i] = 1.f;
        }
        // -- forward: rebuild h inside the chunk
        float h0, Aloc = av[0];
        if constexpr (S > 1) {
          float Al = av[0], Bl = dtu[0] * Bn[0];
#pragma unroll
          for (int i = 1; i < K; ++i) {
            Bl = fmaf(av[i], Bl, dtu[i] * Bn[i]);
            Al *= av[i];
          }
          Aloc = Al;
#pragma unroll
          for (int off = 1; off < S; off <<= 1) {
            const float Ap = __shfl_up_sync(kFull, Al, off, S);
            const float Bp = __shfl_up_sync(kFull, Bl, off, S);
            if (s >= off) {
              Bl = fmaf(Al, Bp, Bl);
              Al *= Ap;
            }
          }
          float Ae = __shfl_up_sync(kFull, Al, 1, S);
          float Be = __shfl_up_sync(kFull, Bl, 1, S);
          if (s == 0) {
            Ae = 1.f;
            Be = 0.f;
          }
          h0 = fmaf(Ae, hck, Be);
        } else {
          h0 = hck;
        }
        {
          float h = h0;
#pragma unroll
          for (int i = 0; i < K; ++i) {
            h = fmaf(av[i], h, dtu[i] * Bn[i]);
            hs[i] = h;
            if constexpr (HAS_Z) y[i] = fmaf(h, Cn[i], y[i]);
          }
        }
        // -- reverse: gh entering this lane's segment from later timesteps
        float gh;
        if constexpr (S > 1) {
          float Gl = 0.f;
#pragma unroll
          for (int i = K - 1; i >= 0; --i) Gl = av[i] * fmaf(dy[i], Cn[i], Gl);
          float Ar = Aloc, Gr = Gl;
#pragma unroll
          for (int off = 1; off < S; off <<= 1) {
            const float An_ = __shfl_down_sync(kFull, Ar, off, S);
            const float Gn_ = __shfl_down_sync(kFull, Gr, off, S);
            if (s + off < S) {
              Gr = fmaf(Ar, Gn_, Gr);
              Ar *= An_;
            }
          }
          float Ae = __shfl_down_sync(kFull, Ar, 1, S);
          float Ge = __shfl_down_sync(kFull, Gr, 1, S);
          if (s == S - 1) {
            Ae = 1.f;
            Ge = 0.f;
          }
          gh = fmaf(Ae, gc[n], Ge);
        } else {
          gh = gc[n];
        }
        float v[2 * K];  // [dB items | dC items] of this lane's channel
#pragma unroll
        for (int i = K - 1; i >= 0; --i) {
          const float gg = fmaf(dy[i], Cn[i], gh);
          v[K + i] = dy[i] * hs[i];
          const float hp = i > 0 ? hs[i - 1] : h0;
          const float x = gg * (av[i] * hp);
          dAacc[n] = fmaf(x, dt[i], dAacc[n]);
          xA[i] = fmaf(x, An, xA[i]);
          gB[i] = fmaf(gg, Bn[i], gB[i]);
          v[i] = gg * dtu[i];
          gh = gg * av[i];
        }
        if constexpr (S > 1)
          gc[n] = __shfl_sync(kFull, gh, 0, S);
        else
          gc[n] = gh;
        // -- reduce-scatter dB|dC over the CW channel lanes holding the same timesteps
        int io = 0;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int mask = S << r;
          const bool upper = (lane & mask) != 0;
          const int half = K >> r;  // values kept after this round (2K >> (r + 1))
#pragma unroll
          for (int j = 0; j < half; ++j) {
            const float send = upper ? v[j] : v[half + j];
            const float keep = upper ? v[half + j] : v[j];
            v[j] = keep + __shfl_xor_sync(kFull, send, mask);
          }
          if (r > 0 && upper) io += half;
        }
        const int q = (lane & S) ? 1 : 0;
        *reinterpret_cast<float4*>(&red[warp][(n * 2 + q) * kChunk + s * K + io]) =
            make_float4(v[0], v[1], v[2], v[3]);
      }
    }

    // -- sum over the warps of the CTA, then over the CTAs of the cluster
    __syncthreads();
    const int total4 = N * 2 * kChunk / 4;
    {
      float4* ro = reinterpret_cast<float4*>(red_out[buf]);
      for (int f4 = threadIdx.x; f4 < total4; f4 += blockDim.x) {
        float4 acc = reinterpret_cast<const float4*>(red[0])[f4];
#pragma unroll
        for (int w = 1; w < kBwdWarps; ++w) {
          const float4 o = reinterpret_cast<const float4*>(red[w])[f4];
          acc.x += o.x;
          acc.y += o.y;
          acc.z += o.z;
          acc.w += o.w;
        }
        ro[f4] = acc;
      }
    }
    cluster.sync();
    {
      const int per = (total4 + CL - 1) / CL;
      const int lo = crank * per;
      const int hi = min(total4, lo + per);
      for (int f4 = lo + threadIdx.x; f4 < hi; f4 += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < CL; ++r) {
          const float4* peer = reinterpret_cast<const float4*>(cluster.map_shared_rank(red_out[buf], r));
          const float4 o = peer[f4];
          acc.x += o.x;
          acc.y += o.y;
          acc.z += o.z;
          acc.w += o.w;
        }
        const int nq = f4 / (kChunk / 4);  // n * 2 + q
        const int t4 = f4 % (kChunk / 4);
        const int n = nq >> 1, q = nq & 1;
        float* dst = a.part_bc + (((slice * a.clusters + cluster_idx) * 2 + q) * N + n) * a.Lpad +
                     (int64_t)k * kChunk + t4 * 4;
        *reinterpret_cast<float4*>(dst) = acc;
      }
    }
    buf ^= 1;

    // -- per-timestep gradients of this lane's K steps
    {
      float du[K], dd[K];
#pragma unroll
      for (int i = 0; i < K; ++i) {
        const float ddt = (xA[i] + uu[i] * gB[i]) * dsp[i];
        du[i] = Dv * dy[i] + dt[i] * gB[i];
        dd[i] = ddt;
        if (t0 + i < L) {
          dbacc += ddt;
          dDacc += dy[i] * uu[i];
        }
      }
      if (valid) {
        store_items<TI, K>(durow, t0, L, vec_io, du);
        store_items<TI, K>(ddrow, t0, L, vec_io, dd);
        if constexpr (HAS_Z) {
#pragma unroll
          for (int i = 0; i < K; ++i) dd[i] = dzc[i] * y[i];
          store_items<TI, K>(dzrow, t0, L, vec_io, dd);
        }
      }
    }
  }

  // -- per-row partials of dA / dD / ddelta_bias: sum the S segment lanes of the channel
#pragma unroll
  for (int n = 0; n < kMaxState; ++n) {
    if (n < N) {
      float v = dAacc[n];
#pragma unroll
      for (int off = S / 2; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off, S);
      if (valid && s == 0) a.part_A[row * N + n] = v;
    }
  }
#pragma unroll
  for (int off = S / 2; off > 0; off >>= 1) {
    dDacc += __shfl_xor_sync(kFull, dDacc, off, S);
    dbacc += __shfl_xor_sync(kFull, dbacc, off, S);
  }
  if (valid && s == 0) {
    a.part_D[row] = dDacc;
    a.part_db[row] = dbacc;
  }
  // Peers may still be reading this CTA's red_out through distributed shared memory.
  cluster.sync();
}

template <typename TI, typename TW, int S>
cudaError_t launch_typed(BwdArgs a, int cluster, cudaStream_t stream) {
  constexpr int CPC = kBwdWarps * (32 / S);
  const int64_t tiles = (a.f.dpg + CPC - 1) / CPC;
  a.f.tiles = (int)(((tiles + cluster - 1) / cluster) * cluster);
  a.clusters = a.f.tiles / cluster;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.f.tiles * a.f.batch * a.f.ngroups));
  cfg.blockDim = dim3(kBwdWarps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.f.z != nullptr) return cudaLaunchKernelEx(&cfg, scan_bwd_kernel<TI, TW, S, true>, a);
  return cudaLaunchKernelEx(&cfg, scan_bwd_kernel<TI, TW, S, false>, a);
}

template <typename TI, typename TW>
cudaError_t launch_seg(const BwdArgs& a, int cluster, cudaStream_t stream) {
  if (bwd_segments(a.f.batch * a.f.dim) == 8) return launch_typed<TI, TW, 8>(a, cluster, stream);
  return launch_typed<TI, TW, 16>(a, cluster, stream);
}

// ---- reduction of the partials ---------------------------------------------------------------

template <typename TO>
__global__ void scan_bwd_reduce_kernel(const BwdArgs a, TO* dB, TO* dC, int64_t osb, int64_t osg,
                                       int64_t osn, int64_t osl, float* dA, float* dD, float* db,
                                       int64_t n_bc4, int64_t n_A, int64_t n_D) {
  const int64_t N = a.f.N, L = a.f.L, Lpad = a.Lpad;
  const int64_t L4 = Lpad / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_bc4 + n_A + n_D; i += stride) {
    if (i < n_bc4) {
      // (slice, q, n, t4)
      const int64_t t4 = i % L4;
      const int64_t n = (i / L4) % N;
      const int64_t q = (i / (L4 * N)) % 2;
      const int64_t slice = i / (L4 * N * 2);
      const int64_t t = t4 * 4;
      if (t >= L) continue;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int cl = 0; cl < a.clusters; ++cl) {
        const float4 o = *reinterpret_cast<const float4*>(
            a.part_bc + (((slice * a.clusters + cl) * 2 + q) * N + n) * Lpad + t);
        acc.x += o.x;
        acc.y += o.y;
        acc.z += o.z;
        acc.w += o.w;
      }
      const int64_t bb = slice / a.f.ngroups, gg = slice % a.f.ngroups;
      TO* dst = (q == 0 ? dB : dC) + bb * osb + gg * osg + n * osn;
      const float vals[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (t + j < L) dst[(t + j) * osl] = from_f32<TO>(vals[j]);
    } else if (i < n_bc4 + n_A) {
      const int64_t j = i - n_bc4;  // d * N + n
      float acc = 0.f;
      for (int64_t bb = 0; bb < a.f.batch; ++bb) acc += a.part_A[bb * a.f.dim * N + j];
      dA[j] = acc;
    } else {
      const int64_t dd = i - n_bc4 - n_A;
      float accD = 0.f, accb = 0.f;
      for (int64_t bb = 0; bb < a.f.batch; ++bb) {
        accD += a.part_D[bb * a.f.dim + dd];
        accb += a.part_db[bb * a.f.dim + dd];
      }
      if (dD) dD[dd] = accD;
      if (db) db[dd] = accb;
    }
  }
}

}  // namespace

int bwd_segments(int64_t rows) { return rows >= 4096 ? 8 : 16; }

int bwd_cluster_size(int64_t tiles) {
  if (tiles >= 8) return 8;
  if (tiles >= 4) return 4;
  if (tiles >= 2) return 2;
  return 1;
}

cudaError_t launch_scan_bwd(const BwdArgs& a, int io_dtype, int bc_dtype, int cluster,
                            cudaStream_t stream) {
  if (a.f.batch == 0 || a.f.dim == 0) return cudaSuccess;
  if (io_dtype == MB200_F32) return launch_seg<float, float>(a, cluster, stream);
  if (io_dtype == MB200_BF16) {
    if (bc_dtype == MB200_BF16) return launch_seg<__nv_bfloat16, __nv_bfloat16>(a, cluster, stream);
    return launch_seg<__nv_bfloat16, float>(a, cluster, stream);
  }
  if (bc_dtype == MB200_F16) return launch_seg<__half, __half>(a, cluster, stream);
  return launch_seg<__half, float>(a, cluster, stream);
}

cudaError_t launch_scan_bwd_reduce_strided(const BwdArgs& a, void* dB, void* dC, int dbc_dtype,
                                           int64_t osb, int64_t osg, int64_t osn, int64_t osl,
                                           float* dA, float* dD, float* db, bool batch_partials,
                                           cudaStream_t stream) {
  const int64_t slices = a.f.batch * a.f.ngroups;
  const int64_t n_bc4 = slices * 2 * a.f.N * (a.Lpad / 4);
  const int64_t n_A = batch_partials ? 0 : a.f.dim * a.f.N;
  const int64_t n_D = batch_partials ? 0 : a.f.dim;
  const int64_t total = n_bc4 + n_A + n_D;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (dbc_dtype == MB200_F32)
    scan_bwd_reduce_kernel<float><<<(unsigned)blocks, threads, 0, stream>>>(
        a, static_cast<float*>(dB), static_cast<float*>(dC), osb, osg, osn, osl, dA, dD, db, n_bc4, n_A, n_D);
  else if (dbc_dtype == MB200_BF16)
    scan_bwd_reduce_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, stream>>>(
        a, static_cast<__nv_bfloat16*>(dB), static_cast<__nv_bfloat16*>(dC), osb, osg, osn, osl, dA, dD, db,
        n_bc4, n_A, n_D);
  else
    scan_bwd_reduce_kernel<__half><<<(unsigned)blocks, threads, 0, stream>>>(
        a, static_cast<__half*>(dB), static_cast<__half*>(dC), osb, osg, osn, osl, dA, dD, db, n_bc4, n_A, n_D);
  return cudaGetLastError();
}

}  // namespace mb200
