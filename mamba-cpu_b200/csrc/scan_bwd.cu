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
//     lane walks its K steps backwards accumulating the gradients. The state loop is not unrolled
//     (the body stays in the instruction cache); its per-state carries (gh entering the chunk and
//     the lane's dA partial) live in Tensor Memory (TMEM);
//   * dB/dC (sums over channels) are reduced deterministically: a sum over the CW channel lanes
//     of the warp through Tensor Memory (each lane stores its values in its own TMEM lane and reads
//     back a 16x256b fragment that holds all channel lanes of its segments), a sum over the warps
//     of the CTA (shared memory), a
//     sum over the CTAs of a thread-block cluster (distributed shared memory), and finally a sum
//     over clusters by the reduce kernel below. dA / dD / ddelta_bias leave the kernel as
//     per-row partials and are summed over batch by the same reduce kernel.
// Data movement: the B/C tile and the restart states of a chunk are staged in shared memory by
// the bulk-copy engine one chunk ahead (double buffer, mbarrier completion); each lane's u /
// delta / dout / z items are prefetched one chunk ahead into registers.
#include <cooperative_groups.h>

#include <atomic>
#include <cmath>

#include "scan.cuh"
#include "quad.cuh"
#include "segscan.cuh"
#include "stage.cuh"
#include "tmem.cuh"

namespace cg = cooperative_groups;

namespace mb200 {

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kRedFloats = kMaxState * 2 * kChunk;  // one CTA's dB|dC chunk partial (2048)

constexpr int ilog2(int v) { return v <= 1 ? 0 : 1 + ilog2(v / 2); }

constexpr int kMaxCluster = 8;  // bwd_cluster_size never returns more

// Split cluster barrier: every thread of every CTA of the cluster arrives (its earlier shared
// memory writes released to the cluster), and waits until all have arrived (acquire).
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMEM columns per CTA: per thread, the adjoint gh entering the current chunk (columns 0..15),
// the dA partial of each state (16..31), the chunk's u, softplus' and dz factor items (32.., 3 x K
// columns) that the output stage reads back, and (64..79) the staging area of the dB / dC sum
// over a warp's channels. At most 3 CTAs are resident per SM: 384 of the 512 columns.
constexpr uint32_t kTmemCols = 128;
constexpr int kColDA = kMaxState;
constexpr int kColItems = 2 * kMaxState;
constexpr int kColRS = 64;

template <typename TW, int CPC>
struct BwdSmem {
  TW bc[2][2][kMaxState][TileRow<TW>::kStride];   // [buf][B|C][n][staged t]
  float hst[2][CPC][kMaxState];                   // [buf][channel][n]: state at the chunk start
  float red[kBwdWarps][kRedFloats];               // [warp]: dB|dC partials of the chunk
  float red_out[2][kRedFloats];                   // CTA sums of a chunk, double-buffered for cluster readers
  float A[CPC][kMaxState];
  uint64_t bar[2];
  uint32_t tmem_base;
};

// A lane's K items of u, delta, dout and z for one chunk, as loaded (converted when used). With
// 2-byte items the next chunk's items are loaded at the end of the current chunk's state loop,
// so their latency overlaps the reductions and the output stage instead of stalling the next
// chunk's start. With 4-byte items that costs more registers than it saves (measured): those
// rows are prefetched into L2 one chunk ahead and loaded when the chunk starts.
template <typename TI, int K>
struct ChunkItems {
  static constexpr bool kCarry = sizeof(TI) == 2;
  Quad<TI> u[kCarry ? K / 4 : 1], d[kCarry ? K / 4 : 1], o[kCarry ? K / 4 : 1], z[kCarry ? K / 4 : 1];
};

template <typename TI, int K, bool HAS_Z>
__device__ __forceinline__ void load_chunk_items(ChunkItems<TI, K>& it, const TI* urow, const TI* drow,
                                                 const TI* dorow, const TI* zrow, int64_t t0, int64_t L, bool vec) {
  if constexpr (ChunkItems<TI, K>::kCarry) {
#pragma unroll
    for (int q = 0; q < K / 4; ++q) {
      const int64_t t = t0 + 4 * q;
      if (vec) {
        it.u[q] = ld_quad_stream(urow + t);
        it.d[q] = ld_quad_stream(drow + t);
        it.o[q] = ld_quad_stream(dorow + t);
        if constexpr (HAS_Z) it.z[q] = ld_quad_stream(zrow + t);
      } else {
        it.u[q] = ld_quad_masked(urow, t, L, 1);
        it.d[q] = ld_quad_masked(drow, t, L, 1);
        it.o[q] = ld_quad_masked(dorow, t, L, 1);
        if constexpr (HAS_Z) it.z[q] = ld_quad_masked(zrow, t, L, 1);
      }
    }
  }
}

template <typename TI, int K>
__device__ __forceinline__ void unpack_items(const Quad<TI> (&q)[K / 4], float (&x)[K]) {
#pragma unroll
  for (int i = 0; i < K / 4; ++i) {
    const float4 v = to_float4(q[i]);
    x[4 * i] = v.x;
    x[4 * i + 1] = v.y;
    x[4 * i + 2] = v.z;
    x[4 * i + 3] = v.w;
  }
}

template <typename TI, typename TW, int S, bool HAS_Z, bool STAGED, bool MASKED>
__device__ __forceinline__ void bwd_chunk(const BwdArgs& a, BwdSmem<TW, kBwdWarps * (32 / S)>& sm, int buf, int k,
                                          int64_t row, int64_t slice, int64_t cluster_idx, int cl_c, bool valid,
                                          int lane, int warp, int c, int s, const TW* Bbase, const TW* Cbase,
                                          float Dv, float bias, const TI* urow, const TI* drow, const TI* dorow,
                                          const TI* zrow, float& dDacc, float& dbacc, int& rbuf,
                                          uint32_t tcar, ChunkItems<TI, kChunk / S>& items, bool next_vec,
                                          cg::cluster_group& cluster) {
  constexpr int K = kChunk / S;
  const ScanArgs& f = a.f;
  const int64_t L = f.L;
  const int N = (int)f.N;
  const int64_t t0 = (int64_t)k * kChunk + s * K;

  // The lane's items (loaded by the previous chunk). u / delta / dout / z are read again at the
  // end of the chunk (L1 hits) instead of being kept live through the state loop.
  float dt[K], dtu[K], dy[K], gB[K], xA[K];
  float y[HAS_Z ? K : 1];
  float sdt = 0.f;
  {
    float uu[K], dl[K], dO[K], zz[K];
    if constexpr (ChunkItems<TI, K>::kCarry) {
      unpack_items<TI, K>(items.u, uu);
      unpack_items<TI, K>(items.d, dl);
      unpack_items<TI, K>(items.o, dO);
      if constexpr (HAS_Z) unpack_items<TI, K>(items.z, zz);
    } else {
      load_items<TI, K>(urow, t0, L, !MASKED, 0.f, uu);
      load_items<TI, K>(drow, t0, L, !MASKED, 0.f, dl);
      load_items<TI, K>(dorow, t0, L, !MASKED, 0.f, dO);
      if constexpr (HAS_Z) load_items<TI, K>(zrow, t0, L, !MASKED, 0.f, zz);
    }
    float dsp[K], dzf[K];  // softplus'(delta + bias); dout * silu'(z)
#pragma unroll
    for (int i = 0; i < K; ++i) {
      const float raw = dl[i] + bias;
      float dti = raw;
      dsp[i] = 1.f;
      if (f.softplus) dti = softplus_dsig(raw, dsp[i]);
      if (MASKED) dti = (t0 + i < L) ? dti : 0.f;
      dt[i] = dti;
      dtu[i] = dti * uu[i];
      sdt += dti;
      float dyi = dO[i];
      dzf[i] = 0.f;
      if constexpr (HAS_Z) {
        const float zs = sigmoid_f(zz[i]);
        dyi = dO[i] * zz[i] * zs;
        dzf[i] = dO[i] * zs * (1.f + zz[i] * (1.f - zs));
        y[i] = Dv * uu[i];
      }
      dy[i] = valid ? dyi : 0.f;
      gB[i] = 0.f;
      xA[i] = 0.f;
    }
    // park the items the output stage needs in TMEM (the pair loop's first wait::st completes
    // these stores)
    tmem_st_n<K>(tcar + kColItems, uu);
    tmem_st_n<K>(tcar + kColItems + K, dsp);
    if constexpr (HAS_Z) tmem_st_n<K>(tcar + kColItems + 2 * K, dzf);
  }

  const TW* tB = &sm.bc[buf][0][0][0];
  const TW* tC = &sm.bc[buf][1][0][0];

  // States are processed in pairs (n0, n0 + 1): the two states' dependency chains (local maps,
  // shuffle scans, the h and adjoint recurrences) are independent and interleave, which hides
  // their latencies; the per-step products that do not sit on a chain run as f32x2 pairs of
  // timesteps. An odd dstate pads the last pair with an inert state (A = B = C = 0).
  const int total4 = N * 2 * kChunk / 4;
#pragma unroll 1
  for (int n0 = 0; n0 < N; n0 += 2) {
    // this thread's carries of the pair (TMEM): gh entering the chunk, dA partial
    float gcn[2], dAc[2];
    tmem_wait_st();  // the previous pair's carry stores have landed
    tmem_ld2(tcar + n0, gcn[0], gcn[1]);
    tmem_ld2(tcar + kColDA + n0, dAc[0], dAc[1]);
    float An[2], A2n[2], hck[2];
    float Bn[2][K], Cn[2][K], av[2][K], bv[2][K], hs[2][K], gg[2][K];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = n0 + j;
      const bool live = n < N;
      An[j] = live ? sm.A[cl_c][n] : 0.f;
      A2n[j] = An[j] * kLog2e;
      // Invalid (padding) lanes must stay finite: they contribute dy = 0 to the dB/dC sums, and
      // 0 * NaN from an unwritten restart-state slot would poison them.
      hck[j] = 0.f;
      if (k > 0 && valid && live) {
        if constexpr (STAGED)
          hck[j] = sm.hst[buf][cl_c][n];
        else
          hck[j] = a.states[(row * f.nchunks + (k - 1)) * N + n];
      } else if (k == 0 && valid && live && f.h_init != nullptr) {
        hck[j] = f.h_init[row * N + n];
      }
      if (!live) {
#pragma unroll
        for (int i = 0; i < K; ++i) Bn[j][i] = Cn[j][i] = 0.f;
      } else if constexpr (STAGED) {
        constexpr int kRS = TileRow<TW>::kStride;
        const int tpos = TileRow<TW>::pos(s * K);
        load_cached_smem<TW, K>(tB + n * kRS + tpos, Bn[j]);
        load_cached_smem<TW, K>(tC + n * kRS + tpos, Cn[j]);
      } else {
        load_bc_items<TW, K>(Bbase + n * f.sBn, f.sBl, t0, L, MASKED ? false : (f.vec_bc != 0), Bn[j]);
        load_bc_items<TW, K>(Cbase + n * f.sCn, f.sCl, t0, L, MASKED ? false : (f.vec_bc != 0), Cn[j]);
      }
      const float2 a2 = make_float2(A2n[j], A2n[j]);
#pragma unroll
      for (int i = 0; i < K; i += 2) {
        const float2 x = __fmul2_rn(make_float2(dt[i], dt[i + 1]), a2);
        av[j][i] = ex2(x.x);
        av[j][i + 1] = ex2(x.y);
        const float2 b = __fmul2_rn(make_float2(dtu[i], dtu[i + 1]), make_float2(Bn[j][i], Bn[j][i + 1]));
        bv[j][i] = b.x;
        bv[j][i + 1] = b.y;
      }
      if (MASKED) {
#pragma unroll
        for (int i = 0; i < K; ++i)
          if (t0 + i >= L) av[j][i] = 1.f;
      }
    }
    // -- forward: rebuild h inside the chunk
    float Aloc[2], h0[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) Aloc[j] = seg_decay(An[j], sdt);  // the segment's total decay
    if constexpr (S > 1) {
      float Al[2], Bl[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        Al[j] = Aloc[j];
        Bl[j] = bv[j][0];
      }
#pragma unroll
      for (int i = 1; i < K; ++i) {
#pragma unroll
        for (int j = 0; j < 2; ++j) Bl[j] = fmaf(av[j][i], Bl[j], bv[j][i]);
      }
      scan_up2<S>(s, Al, Bl);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float Ae = __shfl_up_sync(kFull, Al[j], 1, S);
        float Be = __shfl_up_sync(kFull, Bl[j], 1, S);
        if (s == 0) {
          Ae = 1.f;
          Be = 0.f;
        }
        h0[j] = fmaf(Ae, hck[j], Be);
      }
    } else {
      h0[0] = hck[0];
      h0[1] = hck[1];
    }
    {
      float h[2] = {h0[0], h0[1]};
#pragma unroll
      for (int i = 0; i < K; ++i) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          h[j] = fmaf(av[j][i], h[j], bv[j][i]);
          hs[j][i] = h[j];
        }
      }
    }
    if constexpr (HAS_Z) {
#pragma unroll
      for (int i = 0; i < K; i += 2) {
        float2 yy = make_float2(y[i], y[i + 1]);
#pragma unroll
        for (int j = 0; j < 2; ++j)
          yy = __ffma2_rn(make_float2(hs[j][i], hs[j][i + 1]), make_float2(Cn[j][i], Cn[j][i + 1]), yy);
        y[i] = yy.x;
        y[i + 1] = yy.y;
      }
    }
    // -- reverse: gh entering this lane's segment from later timesteps
    float gh[2], Ar[2] = {1.f, 1.f}, Gr[2] = {0.f, 0.f};
    tmem_wait_ld();
    if constexpr (S > 1) {
      float Gl[2] = {0.f, 0.f};
#pragma unroll
      for (int i = K - 1; i >= 0; --i) {
#pragma unroll
        for (int j = 0; j < 2; ++j) Gl[j] = av[j][i] * fmaf(dy[i], Cn[j][i], Gl[j]);
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        Ar[j] = Aloc[j];
        Gr[j] = Gl[j];
      }
      scan_down2<S>(s, Ar, Gr);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float Ae = __shfl_down_sync(kFull, Ar[j], 1, S);
        float Ge = __shfl_down_sync(kFull, Gr[j], 1, S);
        if (s == S - 1) {
          Ae = 1.f;
          Ge = 0.f;
        }
        gh[j] = fmaf(Ae, gcn[j], Ge);
      }
    } else {
      gh[0] = gcn[0];
      gh[1] = gcn[1];
    }
    // adjoint chain: G_t = gh_t + dy_t C_t, gh_{t-1} = a_t G_t
#pragma unroll
    for (int i = K - 1; i >= 0; --i) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        gg[j][i] = fmaf(dy[i], Cn[j][i], gh[j]);
        gh[j] = gg[j][i] * av[j][i];
      }
    }
    // carries into the previous chunk: gh entering it (the scanned map of the whole chunk
    // applied to gcn) and this lane's dA partial
    {
      float ghc[2] = {gh[0], gh[1]};
      if constexpr (S > 1) {
#pragma unroll
        for (int j = 0; j < 2; ++j) ghc[j] = __shfl_sync(kFull, fmaf(Ar[j], gcn[j], Gr[j]), 0, S);
      }
      tmem_st2(tcar + n0, ghc[0], ghc[1]);
    }
    // -- per state: the gradient terms of the K steps (f32x2 over timestep pairs), then the
    //    sum of dB|dC over the CW channel lanes holding the same timesteps
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = n0 + j;
      const float2 an2 = make_float2(An[j], An[j]);
      float2 dA2 = make_float2(0.f, 0.f);
      float v[2 * K];  // [dB items | dC items] of this lane's channel
#pragma unroll
      for (int i = 0; i < K; i += 2) {
        const float2 g2 = make_float2(gg[j][i], gg[j][i + 1]);
        const float2 h2 = make_float2(hs[j][i], hs[j][i + 1]);
        // a_t h_{t-1} = h_t - b_t
        const float2 xx = __fmul2_rn(g2, __fadd2_rn(h2, make_float2(-bv[j][i], -bv[j][i + 1])));
        dA2 = __ffma2_rn(xx, make_float2(dt[i], dt[i + 1]), dA2);
        const float2 xa = __ffma2_rn(xx, an2, make_float2(xA[i], xA[i + 1]));
        xA[i] = xa.x;
        xA[i + 1] = xa.y;
        const float2 gb = __ffma2_rn(g2, make_float2(Bn[j][i], Bn[j][i + 1]), make_float2(gB[i], gB[i + 1]));
        gB[i] = gb.x;
        gB[i + 1] = gb.y;
        const float2 vb = __fmul2_rn(g2, make_float2(dtu[i], dtu[i + 1]));
        const float2 vc = __fmul2_rn(make_float2(dy[i], dy[i + 1]), h2);
        v[i] = vb.x;
        v[i + 1] = vb.y;
        v[K + i] = vc.x;
        v[K + i + 1] = vc.y;
      }
      dAc[j] += dA2.x + dA2.y;
      if constexpr (S == 8) {
        // Sum of v over the warp's 4 channel lanes (lane = channel * 8 + segment) through TMEM:
        // each lane stores its 16 values in its own TMEM lane, then two 16x256b loads hand lane
        // t the rows of all 4 channels of segment t / 4 at columns 2 (t % 4) + {0, 1} (dB items)
        // and 8 + 2 (t % 4) + {0, 1} (dC items). Channels are added in order 0, 1, 2, 3.
        tmem_st16(tcar + kColRS, v);
        tmem_wait_st();
        float lo[8], hi[8];
        tmem_ld16x256b_x2(tcar + kColRS, lo);                 // channels 0, 1
        tmem_ld16x256b_x2(tcar + kColRS + (16u << 16), hi);   // channels 2, 3
        tmem_wait_ld();
        const float2 sb = __fadd2_rn(__fadd2_rn(__fadd2_rn(make_float2(lo[0], lo[1]), make_float2(lo[2], lo[3])),
                                                make_float2(hi[0], hi[1])),
                                     make_float2(hi[2], hi[3]));
        const float2 sc = __fadd2_rn(__fadd2_rn(__fadd2_rn(make_float2(lo[4], lo[5]), make_float2(lo[6], lo[7])),
                                                make_float2(hi[4], hi[5])),
                                     make_float2(hi[6], hi[7]));
        const int pos = (lane >> 2) * K + 2 * (lane & 3);
        if (n < N) {
          *reinterpret_cast<float2*>(&sm.red[warp][(n * 2) * kChunk + pos]) = sb;
          *reinterpret_cast<float2*>(&sm.red[warp][(n * 2 + 1) * kChunk + pos]) = sc;
        }
      } else {
        // 2 channel lanes per segment (lane = channel * 16 + segment): the same TMEM transpose
        // with 8 columns. Lane t receives both channels of segments t / 4 and t / 4 + 8 at
        // columns 2 (t % 4) + {0, 1}: dB items (t % 4 < 2) or dC items, 2 (t % 2) + {0, 1}.
        tmem_st_n<2 * K>(tcar + kColRS, v);
        tmem_wait_st();
        float lo[4], hi[4];
        tmem_ld16x256b_x1(tcar + kColRS, lo);                 // channel 0: segments g, g + 8
        tmem_ld16x256b_x1(tcar + kColRS + (16u << 16), hi);   // channel 1
        tmem_wait_ld();
        const float2 s0 = __fadd2_rn(make_float2(lo[0], lo[1]), make_float2(hi[0], hi[1]));
        const float2 s1 = __fadd2_rn(make_float2(lo[2], lo[3]), make_float2(hi[2], hi[3]));
        const int g = lane >> 2, m = lane & 3;
        const int base = (n * 2 + (m >> 1)) * kChunk + 2 * (m & 1);
        if (n < N) {
          *reinterpret_cast<float2*>(&sm.red[warp][base + g * K]) = s0;
          *reinterpret_cast<float2*>(&sm.red[warp][base + (g + 8) * K]) = s1;
        }
      }
    }
    tmem_st2(tcar + kColDA + n0, dAc[0], dAc[1]);
  }
  // (the first chunk of a later sequence piece loads the chunk before it for nothing: in bounds,
  // and cheaper than another live value in this loop)
  if (k > 0) load_chunk_items<TI, K, HAS_Z>(items, urow, drow, dorow, zrow, t0 - kChunk, L, next_vec);
  // -- sum the chunk's partials over the warps of the CTA. red is rewritten only in the next
  //    chunk, after the cluster barrier below, which every thread reaches after this sum.
  __syncthreads();
  {
    float4* ro = reinterpret_cast<float4*>(sm.red_out[rbuf]);
    for (int f4 = threadIdx.x; f4 < total4; f4 += blockDim.x) {
      float4 acc = reinterpret_cast<const float4*>(sm.red[0])[f4];
#pragma unroll
      for (int w = 1; w < kBwdWarps; ++w) {
        const float4 o = reinterpret_cast<const float4*>(sm.red[w])[f4];
        acc.x += o.x;
        acc.y += o.y;
        acc.z += o.z;
        acc.w += o.w;
      }
      ro[f4] = acc;
    }
  }

  // -- the per-timestep gradients of this lane's K steps
  auto output_stage = [&]() {
    float uu[K], dsp[K], dzf[K];
    tmem_ld_n<K>(tcar + kColItems, uu);
    tmem_ld_n<K>(tcar + kColItems + K, dsp);
    if constexpr (HAS_Z) tmem_ld_n<K>(tcar + kColItems + 2 * K, dzf);
    tmem_wait_ld();
    float du[K], dd[K];
#pragma unroll
    for (int i = 0; i < K; ++i) {
      const float ddt = (xA[i] + uu[i] * gB[i]) * dsp[i];
      du[i] = Dv * dy[i] + dt[i] * gB[i];
      dd[i] = ddt;
      if (!MASKED || t0 + i < L) {
        dbacc += ddt;
        dDacc += dy[i] * uu[i];
      }
    }
    if (valid) {
      TI* durow = static_cast<TI*>(a.du) + row * L;
      TI* ddrow = static_cast<TI*>(a.ddelta) + row * L;
      if (MASKED) {
        store_items<TI, K>(durow, t0, L, false, du);
        store_items<TI, K>(ddrow, t0, L, false, dd);
      } else {
        store_stream<TI, K>(durow + t0, du);
        store_stream<TI, K>(ddrow + t0, dd);
      }
      if constexpr (HAS_Z) {
#pragma unroll
        for (int i = 0; i < K; ++i) dd[i] = dzf[i] * y[i];
        TI* dzrow = static_cast<TI*>(a.dz) + row * L;
        if (MASKED)
          store_items<TI, K>(dzrow, t0, L, false, dd);
        else
          store_stream<TI, K>(dzrow + t0, dd);
      }
    }
  };
  // -- sum over the CTAs of the cluster. With 4-byte items: arrive once this CTA's sums are in
  //    red_out, write the per-timestep gradients while the other CTAs catch up, then wait and
  //    read theirs. With 2-byte items (next chunk's items held in registers) that order spills
  //    (measured slower): full barrier, peer sums, then the gradients.
  constexpr bool kOverlap = !ChunkItems<TI, K>::kCarry;
  cluster_arrive_release();
  if constexpr (kOverlap) output_stage();
  cluster_wait_acquire();
  {
    const int CL = (int)cluster.num_blocks();
    const int crank = (int)cluster.block_rank();
    const int per = (total4 + CL - 1) / CL;
    const int lo = crank * per;
    const int hi = min(total4, lo + per);
    auto dst_of = [&](int f4) {  // this slice's cluster partial of float4 f4 (n * 2 + q, t4)
      const int nq = f4 / (kChunk / 4);
      const int t4 = f4 % (kChunk / 4);
      const int n = nq >> 1, q = nq & 1;
      return a.part_bc + (((slice * a.clusters + cluster_idx) * 2 + q) * N + n) * a.Lpad + (int64_t)k * kChunk +
             t4 * 4;
    };
    if constexpr (ChunkItems<TI, K>::kCarry) {
      // 2-byte items: the next chunk's items are held in registers here, so one peer load at a
      // time (more loads in flight spill)
      for (int f4 = lo + threadIdx.x; f4 < hi; f4 += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < CL; ++r) {
          const float4 o = reinterpret_cast<const float4*>(cluster.map_shared_rank(sm.red_out[rbuf], r))[f4];
          acc.x += o.x;
          acc.y += o.y;
          acc.z += o.z;
          acc.w += o.w;
        }
        *reinterpret_cast<float4*>(dst_of(f4)) = acc;
      }
    } else {
      // Each thread sums one half (a float2) of a float4 over the peers, in rank order, with the
      // loads of four peers in flight at a time (distributed shared memory round trips are long).
      for (int h2 = 2 * lo + threadIdx.x; h2 < 2 * hi; h2 += blockDim.x) {
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int r0 = 0; r0 < kMaxCluster; r0 += 4) {
          float2 o[4];
#pragma unroll
          for (int r = 0; r < 4; ++r)
            if (r0 + r < CL)
              o[r] = reinterpret_cast<const float2*>(cluster.map_shared_rank(sm.red_out[rbuf], r0 + r))[h2];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            if (r0 + r < CL) {
              acc.x += o[r].x;
              acc.y += o[r].y;
            }
          }
        }
        *reinterpret_cast<float2*>(dst_of(h2 >> 1) + (h2 & 1) * 2) = acc;
      }
    }
  }
  rbuf ^= 1;
  if constexpr (!kOverlap) output_stage();
}

template <typename TI, typename TW, int S, bool HAS_Z, bool STRIDED>
__global__ void __launch_bounds__(kBwdWarps * 32, 3) scan_bwd_kernel(const BwdArgs a) {
  constexpr int K = kChunk / S;
  constexpr int CW = 32 / S;
  constexpr int CPC = kBwdWarps * CW;
  static_assert(S == 8 || S == 16, "segments per channel: the TMEM channel sum handles 8 and 16");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  BwdSmem<TW, CPC>& sm = *reinterpret_cast<BwdSmem<TW, CPC>*>(smem_raw);

  cg::cluster_group cluster = cg::this_cluster();
  const int CL = (int)cluster.num_blocks();

  const ScanArgs& f = a.f;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int c = lane / S;
  const int s = lane % S;
  // blockIdx.x = (piece * slices + slice) * tiles + tile; a cluster's CTAs share piece and slice
  const unsigned bx = blockIdx.x, ntiles = (unsigned)f.tiles, nslices = (unsigned)(f.batch * f.ngroups);
  const int64_t tile = bx % ntiles;  // 32-bit index arithmetic: grids stay below 2^31 CTAs
  const int64_t slice = (bx / ntiles) % nslices;
  const int piece = (int)(bx / ntiles / nslices);
  const int k_lo = piece * f.piece_chunks;
  const int k_hi = min(f.nchunks, k_lo + f.piece_chunks);
  const int64_t rows = f.batch * f.dim;
  const int64_t b = slice / f.ngroups;
  const int64_t g = slice % f.ngroups;
  const int64_t cluster_idx = tile / CL;
  const int64_t tile_c0 = tile * CPC;  // first channel (in group) of this CTA
  const int64_t cig = tile_c0 + warp * CW + c;
  const bool valid = cig < f.dpg;
  const int cl_c = valid ? warp * CW + c : 0;  // CTA slot whose staged rows this lane reads
  const int64_t d = g * f.dpg + (valid ? cig : 0);
  const int64_t row = b * f.dim + d;
  const int64_t L = f.L;
  const int N = (int)f.N;
  const int64_t nvalid = f.dpg - tile_c0 < CPC ? (f.dpg - tile_c0 > 0 ? f.dpg - tile_c0 : 0) : CPC;

  // u / delta / z rows: dense (row * L) or, in the STRIDED instantiations, strided views (batch
  // and dim strides of their own); separate instantiations keep the dense kernels' registers.
  const TI* urow = static_cast<const TI*>(f.u) + (STRIDED ? b * f.sub + d * f.sud : row * L);
  const TI* drow = static_cast<const TI*>(f.delta) + (STRIDED ? b * f.sdb + d * f.sdd : row * L);
  const TI* zrow = HAS_Z ? static_cast<const TI*>(f.z) + (STRIDED ? b * f.szb + d * f.szd : row * L) : nullptr;
  const TI* dorow = static_cast<const TI*>(a.dout) + row * L;
  const TW* Bbase = static_cast<const TW*>(f.B) + b * f.sBb + g * f.sBg;
  const TW* Cbase = static_cast<const TW*>(f.C) + b * f.sCb + g * f.sCg;
  const float Dv = f.D ? f.D[d] : 0.f;
  const float bias = f.delta_bias ? f.delta_bias[d] : 0.f;
  const bool staged = f.vec_bc != 0;

  // TMEM for the per-thread carries, the parked items and the channel-sum staging (warp 0
  // allocates kTmemCols = 128 columns; at most 3 CTAs are co-resident, 384 of the SM's 512)
  if (warp == 0) tmem_alloc(&sm.tmem_base, kTmemCols);
  for (int i = threadIdx.x; i < CPC * N; i += blockDim.x) {
    const int ch = i / N, n = i % N;
    const int64_t dd = g * f.dpg + (tile_c0 + ch < f.dpg ? tile_c0 + ch : 0);
    sm.A[ch][n] = f.A[dd * N + n];
  }
  if (staged && threadIdx.x == 0) {
    mbar_init(&sm.bar[0], 1);
    mbar_init(&sm.bar[1], 1);
    mbar_fence_init();
  }
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tcar = tmem_lane_addr(sm.tmem_base, warp, 0);
  {
    // carries: gh entering the last chunk = dlast_state, dA partials = 0
    float init[kMaxState];
#pragma unroll
    for (int n = 0; n < kMaxState; ++n)
      init[n] = (valid && n < N && a.dlast != nullptr) ? a.dlast[row * N + n] : 0.f;
    // an earlier piece starts from the adjoint the later pieces leave: dlast carried through their
    // decays plus their adjoints from a zero carry (linear in the carry)
    if (valid) {
      for (int q = f.pieces - 1; q > piece; --q) {
#pragma unroll
        for (int n = 0; n < kMaxState; ++n) {
          if (n < N) {
            const int64_t at = ((int64_t)q * rows + row) * N + n;
            init[n] = fmaf(a.piece_P[at], init[n], a.piece_G[at]);
          }
        }
      }
    }
    tmem_st16(tcar, init);
#pragma unroll
    for (int n = 0; n < kMaxState; ++n) init[n] = 0.f;
    tmem_st16(tcar + kColDA, init);
  }

  // first row (global index) of this CTA's channels, for the restart-state copies
  const int64_t row_c0 = b * f.dim + g * f.dpg + tile_c0;
  auto issue = [&](int k, int buf) {  // warp 0: B/C tile and restart states of chunk k
    constexpr uint32_t half_bytes = kChunk / 2 * sizeof(TW);
    constexpr uint32_t st_bytes = kMaxState * sizeof(float);
    const bool with_states = k > 0 && N == kMaxState;
    const int nst = with_states ? (int)nvalid : 0;
    if (lane == 0) mbar_arrive_expect_tx(&sm.bar[buf], 4 * N * half_bytes + nst * st_bytes);
    __syncwarp();
    fence_proxy_async();
    for (int j = lane; j < 4 * N + nst; j += 32) {
      if (j < 4 * N) {  // B/C rows in two halves (TileRow layout)
        const int r = j >> 1, hf = j & 1;
        const bool isC = r >= N;
        const int n = isC ? r - N : r;
        const TW* src = (isC ? Cbase + n * f.sCn : Bbase + n * f.sBn) + (int64_t)k * kChunk + hf * (kChunk / 2);
        bulk_g2s(&sm.bc[buf][isC ? 1 : 0][n][TileRow<TW>::pos(hf * (kChunk / 2))], src, half_bytes, &sm.bar[buf]);
      } else {
        const int ch = j - 4 * N;
        bulk_g2s(&sm.hst[buf][ch][0], a.states + ((row_c0 + ch) * f.nchunks + (k - 1)) * kMaxState, st_bytes,
                 &sm.bar[buf]);
      }
    }
    if (k > 0 && N != kMaxState) {  // restart states not 64-byte rows: plain loads (all lanes of warp 0)
      for (int i = lane; i < (int)nvalid * N; i += 32) {
        const int ch = i / N, n = i % N;
        sm.hst[buf][ch][n] = a.states[((row_c0 + ch) * f.nchunks + (k - 1)) * N + n];
      }
    }
  };

  float dDacc = 0.f, dbacc = 0.f;
  int rbuf = 0;
  const bool vec_io = f.vec_io != 0;
  const int nfull = (vec_io && staged) ? (int)(L / kChunk) : 0;

  ChunkItems<TI, K> items;
  if (k_hi > k_lo)
    load_chunk_items<TI, K, HAS_Z>(items, urow, drow, dorow, zrow, (int64_t)(k_hi - 1) * kChunk + s * K, L,
                                   k_hi - 1 < nfull);
  // This CTA's piece of the row: chunks [k_lo, k_hi). The partial last chunk (and every chunk of
  // an unaligned row) goes first: masked, direct loads.
  for (int k = k_hi - 1; k >= max(k_lo, nfull); --k) {
    bwd_chunk<TI, TW, S, HAS_Z, false, true>(a, sm, 0, k, row, slice, cluster_idx, cl_c, valid, lane, warp, c, s,
                                             Bbase, Cbase, Dv, bias, urow, drow, dorow, zrow, dDacc, dbacc, rbuf,
                                             tcar, items, k - 1 < nfull, cluster);
  }
  // Full chunks, last to first: B/C + restart states staged one chunk ahead by the bulk-copy
  // engine; the lane's own items of the next chunk are loaded at the end of the current one (2-byte
  // items) or prefetched into L2 (4-byte items).
  const int kf = min(k_hi, nfull) - 1;  // the piece's last full chunk
  if (kf >= k_lo) {
    if (warp == 0) issue(kf, kf & 1);
    // With dstate < 16 issue() stores the restart states with plain stores, which the first
    // chunk reads right away (later chunks' stores are ordered by the barrier ending each chunk;
    // with dstate 16 they come by bulk copy, ordered by the mbarrier).
    if (N != kMaxState) __syncthreads();
  }
  for (int k = kf; k >= k_lo; --k) {
    const int buf = k & 1;
    if (k > k_lo) {
      if constexpr (!ChunkItems<TI, K>::kCarry) {
        const int64_t t1 = (int64_t)(k - 1) * kChunk + s * K;
        prefetch_l2(urow + t1);
        prefetch_l2(drow + t1);
        prefetch_l2(dorow + t1);
        if constexpr (HAS_Z) prefetch_l2(zrow + t1);
      }
      if (warp == 0) issue(k - 1, buf ^ 1);
    }
    // Uses of bar[buf], from the piece's last full chunk downwards: chunk k is use number (kf-k)/2.
    mbar_wait(&sm.bar[buf], (uint32_t)(((kf - k) >> 1) & 1));
    bwd_chunk<TI, TW, S, HAS_Z, true, false>(a, sm, buf, k, row, slice, cluster_idx, cl_c, valid, lane, warp, c, s,
                                             Bbase, Cbase, Dv, bias, urow, drow, dorow, zrow, dDacc, dbacc, rbuf,
                                             tcar, items, true, cluster);
    // bwd_chunk ends with a cluster barrier wait after its last shared-memory read of this
    // buffer (and of red), so the next iteration may refill it.
  }

  // -- the adjoint entering the first step is the gradient of the initial state (every segment
  //    lane of a channel holds it)
  if (a.dh_init != nullptr && piece == 0) {
    float ghp[kMaxState];
    tmem_wait_st();
    tmem_ld16(tcar, ghp);
    tmem_wait_ld();
    if (valid && s == 0) {
#pragma unroll
      for (int n = 0; n < kMaxState; ++n)
        if (n < N) a.dh_init[row * N + n] = ghp[n];
    }
  }
  // -- per-row partials of dA / dD / ddelta_bias: sum the S segment lanes of the channel
  {
    float dAp[kMaxState];
    tmem_wait_st();
    tmem_ld16(tcar + kColDA, dAp);
    tmem_wait_ld();
#pragma unroll
    for (int n = 0; n < kMaxState; ++n) {
      float v = dAp[n];
#pragma unroll
      for (int off = S / 2; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off, S);
      if (valid && s == 0 && n < N) a.part_A[((int64_t)piece * rows + row) * N + n] = v;
    }
  }
#pragma unroll
  for (int off = S / 2; off > 0; off >>= 1) {
    dDacc += __shfl_xor_sync(kFull, dDacc, off, S);
    dbacc += __shfl_xor_sync(kFull, dbacc, off, S);
  }
  if (valid && s == 0) {
    a.part_D[(int64_t)piece * rows + row] = dDacc;
    a.part_db[(int64_t)piece * rows + row] = dbacc;
  }
  // Peers may still be reading this CTA's red_out through distributed shared memory.
  tmem_fence_before_sync();
  cluster.sync();
  // every thread of the CTA is done with TMEM: the allocating warp frees it
  tmem_fence_after_sync();
  if (warp == 0) tmem_dealloc(sm.tmem_base, kTmemCols);
}

template <typename TI, typename TW, int S>
cudaError_t launch_typed(BwdArgs a, int cluster, cudaStream_t stream) {
  constexpr int CPC = kBwdWarps * (32 / S);
  const int64_t tiles = (a.f.dpg + CPC - 1) / CPC;
  a.f.tiles = (int)(((tiles + cluster - 1) / cluster) * cluster);
  a.clusters = a.f.tiles / cluster;
  constexpr size_t smem = sizeof(BwdSmem<TW, CPC>);
  const bool strided = io_rows_strided(a.f);
  auto kern = a.f.z != nullptr ? (strided ? scan_bwd_kernel<TI, TW, S, true, true> : scan_bwd_kernel<TI, TW, S, true, false>)
                               : (strided ? scan_bwd_kernel<TI, TW, S, false, true> : scan_bwd_kernel<TI, TW, S, false, false>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.f.tiles * a.f.batch * a.f.ngroups * a.f.pieces));
  cfg.blockDim = dim3(kBwdWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <typename TI, typename TW>
cudaError_t launch_seg(const BwdArgs& a, int cluster, cudaStream_t stream) {
  if (bwd_segments(a.f.batch * a.f.dim, a.f.nchunks) == 8) return launch_typed<TI, TW, 8>(a, cluster, stream);
  return launch_typed<TI, TW, 16>(a, cluster, stream);
}

// ---- reduction of the partials ---------------------------------------------------------------

template <typename TO>
__global__ void scan_bwd_reduce_kernel(const BwdArgs a, TO* dB, TO* dC, int64_t osb, int64_t osg, int64_t osn,
                                       int64_t osl, float* dA, float* dD, float* db, int64_t n_bc4, int64_t n_A,
                                       int64_t n_D) {
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
#pragma unroll 4
      for (int cl = 0; cl < a.clusters; ++cl) {  // unrolled: four loads in flight, adds in order
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
      for (int64_t pb = 0; pb < a.f.batch * a.f.pieces; ++pb) acc += a.part_A[pb * a.f.dim * N + j];
      dA[j] = acc;
    } else {
      const int64_t dd = i - n_bc4 - n_A;
      float accD = 0.f, accb = 0.f;
      for (int64_t pb = 0; pb < a.f.batch * a.f.pieces; ++pb) {  // (piece, batch) partials
        accD += a.part_D[pb * a.f.dim + dd];
        accb += a.part_db[pb * a.f.dim + dd];
      }
      if (dD) dD[dd] = accD;
      if (db) db[dd] = accb;
    }
  }
}

}  // namespace

int bwd_segments(int64_t rows, int nchunks) {
  // 16 segments per channel (2 channels per warp) give short rows of small problems more warps;
  // long rows (64 chunks and more) keep 8 and are split into sequence pieces when they are few.
  return rows >= 4096 || nchunks >= 64 ? 8 : 16;
}

cudaError_t read_fault_bwd(int* out) { return read_fault_word(out); }

int sm_count() {
  static std::atomic<int> sms{0};
  int v = sms.load();
  if (v == 0) {
    int dev = 0, n = 0;
    v = (cudaGetDevice(&dev) == cudaSuccess &&
         cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
            ? n
            : 148;
    sms.store(v);
  }
  return v;
}

std::atomic<int> g_forced_pieces{0};

void set_forced_pieces(int n) { g_forced_pieces.store(n > 0 ? n : 0); }
int forced_pieces() { return g_forced_pieces.load(); }

int seq_pieces(int64_t ctas, int nchunks, bool backward) {
  // Pieces trade a summary pass over all pieces but one (relative cost s per element: measured
  // 0.23 of the backward kernel's, 0.8 of the forward's, whose recurrence is most of its work)
  // against the idle share of the resident slots (3 CTAs per SM) in the grid's last round:
  //   cost(G) = (1 + s (G - 1) / G) * ceil(G w) / (G w),   w = CTAs of whole rows / slots,
  // which also charges grids under one round for their empty slots. G runs from 1 to 8 with at
  // least 4 chunks per piece. (Config 5 on one GPU: the backward takes 2 pieces, 28.2 -> 25.9 ms,
  // the forward none; one rank's shard at 8 ranks: 5 pieces both.)
  int G = g_forced_pieces.load();
  if (G <= 0) {
    if (ctas <= 0 || nchunks < 2) return 1;
    const double s = backward ? 0.23 : 0.8;
    const double w = (double)ctas / ((double)sm_count() * 3);
    double best = 0.0;
    G = 1;
    for (int c = 1; c <= 8 && (c == 1 || c <= nchunks / 4); ++c) {
      const double fill = c * w;
      const double cost = (1.0 + s * (c - 1) / c) * std::ceil(fill) / fill;
      if (c == 1 || cost < best * 0.98) {  // a split must gain at least 2 %
        best = cost;
        G = c;
      }
    }
  }
  if (G > nchunks) G = nchunks;
  return G < 1 ? 1 : G;
}

int bwd_cluster_size(int64_t tiles, int64_t slices) {
  // Larger clusters divide the dB/dC partials written per slice (fewer cluster partials for the
  // reduce kernel) but constrain where CTAs may be placed, which costs more the more waves of
  // resident CTAs (3 per SM) the grid takes. Measured, backward ms with 1 / 2 / 4 / 8 CTAs per
  // cluster: config 2 (0.86 waves) 0.289 / 0.262 / 0.247 / 0.243; config 5 at L 16384 (1.44
  // waves) 7.42 / 7.27 / 7.12 / 7.65 (L 65536: 28.88 with 2, 28.40 with 4); the config-4 layer
  // shape (4.6 waves) 2.396 with 2, 2.434 with 4; config 5 in 2 sequence pieces (2.9 waves) 25.9
  // with 2, 30.7 with 4. Hence 8 up to one wave, 4 up to two, else 2;
  // one wave of 8-CTA clusters holds at most 48 clusters here (384 CTAs: a cluster stays inside
  // one GPC), so larger one-wave grids take 4.
  const int sms = sm_count();
  const int64_t ctas = tiles * slices;
  const int cap = ctas <= 384 ? kMaxCluster : ctas <= (int64_t)sms * 6 ? 4 : 2;
  int cl = 1;
  while (cl * 2 <= cap && tiles >= cl * 2) cl *= 2;
  return cl;
}

cudaError_t launch_scan_bwd(const BwdArgs& a, int io_dtype, int bc_dtype, int cluster, cudaStream_t stream) {
  if (a.f.batch == 0 || a.f.dim == 0) return cudaSuccess;
  if (io_dtype == MB200_F32) return launch_seg<float, float>(a, cluster, stream);
  if (io_dtype == MB200_BF16) {
    if (bc_dtype == MB200_BF16) return launch_seg<__nv_bfloat16, __nv_bfloat16>(a, cluster, stream);
    return launch_seg<__nv_bfloat16, float>(a, cluster, stream);
  }
  if (bc_dtype == MB200_F16) return launch_seg<__half, __half>(a, cluster, stream);
  return launch_seg<__half, float>(a, cluster, stream);
}

cudaError_t launch_scan_bwd_reduce_strided(const BwdArgs& a, void* dB, void* dC, int dbc_dtype, int64_t osb,
                                           int64_t osg, int64_t osn, int64_t osl, float* dA, float* dD, float* db,
                                           bool batch_partials, cudaStream_t stream) {
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
