// scan_fwd.cu -- forward selective scan on sm_100a.
//
// Computes, for every row (batch b, channel d) and timestep t (mamba-cpu
// csrc/selective_scan.cpp:120-145 states the same recurrence as a sequential CPU loop):
//   dt_t = softplus(delta_t + bias_d)            (or delta_t + bias_d without softplus)
//   h_t  = exp(dt_t * A_d) * h_{t-1} + dt_t * u_t * B_t      (dstate lanes of h, h_{-1} = 0)
//   y_t  = <h_t, C_t> + D_d * u_t ;  out_t = y_t * silu(z_t)  (the gate only when z is given)
//
// Work decomposition: one lane per (channel, NS states), walking the sequence in order.
//   * A CTA owns CPC channels of one (batch, group) slice and walks their rows in chunks of 64
//     timesteps. Per chunk, its threads first stage the per-element terms dt and dt*u of all
//     CPC rows and the B / C tile (dstate x 64, shared by every channel of the slice) in shared
//     memory, in fp32, so softplus and the input conversions run once per element.
//   * Each recurrence lane then runs its states through the 64 steps sequentially: there is no
//     cross-lane scan at all. exp(dt * A) is one SFU ex2 per (t, n); the multiplies around it
//     are packed two timesteps at a time into the Blackwell f32x2 FMA/FMUL instructions.
//   * y_t needs the sum over all states of a channel, which lives in kLPC different lanes. Each
//     lane writes its partial sums for the chunk to shared memory; after a barrier the threads
//     add the partials of four consecutive timesteps at a time, apply D and the gate, and store
//     16-byte (fp32) / 8-byte (bf16) pieces of the output rows.
//   * Global loads for chunk k + 1 (u, delta, z and the B / C tile) are issued into registers
//     before chunk k's recurrence starts and consumed after it, so their latency is hidden
//     behind the recurrence; u and z then wait in shared memory for the output stage.
// Accuracy of long memories: the SFU ex2 is not correctly rounded, and near 1 its error has a
// consistent sign, so a state with |dt * A| << 1 would accumulate a relative drift of the order
// of L ulp through thousands of chained factors. Each lane therefore also keeps the running
// product P of its ex2 factors over the chunk and, at the chunk end, replaces the chunk's decay
// of the carried state by the accurately rounded expf(A * sum(dt)):
//   h_end += (expf(A * sum dt) - P) * h_start,
// so the error of the carried part stays at one rounding per chunk.
// The chunk-end states are optionally written to chunk_states, which the backward uses as
// restart points.
#include "quad.cuh"
#include "scan.cuh"

namespace mb200 {

namespace {

// fp32 shared-memory row stride: 272 bytes, so rows r, r + 1, ... start 16 bytes apart modulo the
// 128-byte bank window and eight lanes reading 16-byte pieces of eight rows never collide.
constexpr int kRowF = kChunk + 4;
constexpr int kThreads = kFwdWarps * 32;
constexpr int kQuads = kChunk / 4;  // 4-step groups per chunk

template <int NS>
struct FwdShape {
  static constexpr int kLPC = kMaxState / NS;                  // lanes per channel
  static constexpr int kCPW = 32 / kLPC;                       // channels per warp
  static constexpr int kCPC = kFwdWarps * kCPW;                // channels per CTA
  static constexpr int kTasks = kCPC * kQuads / kThreads;      // 4-element row pieces per thread
};

template <int NS>
struct FwdSmem {
  float dt[FwdShape<NS>::kCPC][kRowF];
  float dtu[FwdShape<NS>::kCPC][kRowF];
  float B[kMaxState][kRowF];
  float C[kMaxState][kRowF];
  float u[FwdShape<NS>::kCPC][kRowF];  // u and z of the chunk, for the output stage
  float z[FwdShape<NS>::kCPC][kRowF];
  float y[FwdShape<NS>::kCPC][FwdShape<NS>::kLPC][kRowF];  // per-lane partial sums of y
};

__device__ __forceinline__ float4 ld4s(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4s(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

// Operands of one 4-step group of one lane: the decays a = exp(dt A), the inputs b = dt u B and
// the C values of the lane's states.
template <int NS>
struct GroupOps {
  float a[NS][4];
  float2 b[NS][2];
  float4 c[NS];
};

// Loads group q's dt, dt*u, B, C from shared memory and evaluates its decays and inputs.
template <int NS, bool WRITE_OUT, bool MASKED>
__device__ __forceinline__ void group_ops(const FwdSmem<NS>& sm, int cl, int p, int q, const float2 (&A2)[NS],
                                          int lim, float2& sd, GroupOps<NS>& g) {
  using Sh = FwdShape<NS>;
  const float4 d4 = ld4s(&sm.dt[cl][4 * q]);
  const float4 u4 = ld4s(&sm.dtu[cl][4 * q]);
  sd = __fadd2_rn(sd, lo2(d4));
  sd = __fadd2_rn(sd, hi2(d4));
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int n = p + j * Sh::kLPC;
    const float4 B4 = ld4s(&sm.B[n][4 * q]);
    if (WRITE_OUT) g.c[j] = ld4s(&sm.C[n][4 * q]);
    const float2 x01 = __fmul2_rn(lo2(d4), A2[j]);
    const float2 x23 = __fmul2_rn(hi2(d4), A2[j]);
    g.a[j][0] = ex2(x01.x);
    g.a[j][1] = ex2(x01.y);
    g.a[j][2] = ex2(x23.x);
    g.a[j][3] = ex2(x23.y);
    if (MASKED) {  // steps past seqlen are the identity (their dt * u is 0)
#pragma unroll
      for (int e = 0; e < 4; ++e) g.a[j][e] = 4 * q + e < lim ? g.a[j][e] : 1.f;
    }
    g.b[j][0] = __fmul2_rn(lo2(u4), lo2(B4));
    g.b[j][1] = __fmul2_rn(hi2(u4), hi2(B4));
  }
}

// One chunk of the recurrence for one lane. lim = number of real timesteps in the chunk.
// Software-pipelined by one group: the shared-memory loads and SFU exponentials of group q + 1
// are issued before the FMA chain of group q, so their latencies overlap it.
template <int NS, bool WRITE_OUT, bool MASKED>
__device__ __forceinline__ void recur_chunk(FwdSmem<NS>& sm, int cl, int p, const float2 (&A2)[NS], float (&h)[NS],
                                            float2 (&P)[NS], float2& sd, int lim) {
  GroupOps<NS> cur;
  group_ops<NS, WRITE_OUT, MASKED>(sm, cl, p, 0, A2, lim, sd, cur);
#pragma unroll 4
  for (int q = 0; q < kQuads; ++q) {
    GroupOps<NS> nxt;
    if (q + 1 < kQuads) group_ops<NS, WRITE_OUT, MASKED>(sm, cl, p, q + 1, A2, lim, sd, nxt);
    float2 y01 = make_float2(0.f, 0.f), y23 = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      float2 h01, h23;
      h01.x = fmaf(cur.a[j][0], h[j], cur.b[j][0].x);
      h01.y = fmaf(cur.a[j][1], h01.x, cur.b[j][0].y);
      h23.x = fmaf(cur.a[j][2], h01.y, cur.b[j][1].x);
      h23.y = fmaf(cur.a[j][3], h23.x, cur.b[j][1].y);
      h[j] = h23.y;
      P[j] = __fmul2_rn(P[j], make_float2(cur.a[j][0], cur.a[j][1]));
      P[j] = __fmul2_rn(P[j], make_float2(cur.a[j][2], cur.a[j][3]));
      if (WRITE_OUT) {
        y01 = __ffma2_rn(h01, lo2(cur.c[j]), y01);
        y23 = __ffma2_rn(h23, hi2(cur.c[j]), y23);
      }
    }
    if (WRITE_OUT) st4s(&sm.y[cl][p][4 * q], make_float4(y01.x, y01.y, y23.x, y23.y));
    if (q + 1 < kQuads) cur = nxt;
  }
}

template <typename TI, typename TW, int NS, bool HAS_Z, bool WRITE_OUT, bool STRIDED>
__global__ void __launch_bounds__(kThreads, 3) scan_fwd_kernel(const ScanArgs a) {
  using Sh = FwdShape<NS>;
  constexpr int kTasks = Sh::kTasks;
  constexpr int kMats = WRITE_OUT ? 2 : 1;                          // B (and C)
  constexpr int kBCTasks = kMats * kMaxState * kQuads / kThreads;   // B / C tile pieces per thread
  static_assert(kTasks >= 1 && kBCTasks >= 1, "task split");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  FwdSmem<NS>& sm = *reinterpret_cast<FwdSmem<NS>*>(smem_raw);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  // blockIdx.x = (piece * slices + slice) * tiles + tile
  const unsigned bx = blockIdx.x, ntiles = (unsigned)a.tiles, nslices = (unsigned)(a.batch * a.ngroups);
  const int64_t tile = bx % ntiles;  // 32-bit index arithmetic: grids stay below 2^31 CTAs
  const int64_t slice = (bx / ntiles) % nslices;
  const int piece = (int)(bx / ntiles / nslices);
  const int64_t b = slice / a.ngroups;
  const int64_t g = slice % a.ngroups;
  const int64_t c0 = tile * Sh::kCPC;  // first channel (inside the group) of this CTA
  const int nvalid = (int)(a.dpg - c0 < Sh::kCPC ? a.dpg - c0 : Sh::kCPC);
  const int64_t d0 = g * a.dpg + c0;   // first channel (global)
  const int64_t row0 = b * a.dim + d0;
  const int64_t L = a.L;
  const int N = (int)a.N;
  const bool vec_io = a.vec_io != 0;
  const bool vec_bc = a.vec_bc != 0;
  const bool softplus = a.softplus != 0;
  const TW* Bb = static_cast<const TW*>(a.B) + b * a.sBb + g * a.sBg;
  const TW* Cb = static_cast<const TW*>(a.C) + b * a.sCb + g * a.sCg;

  // ---- recurrence lane: channel slot cl, states p, p + kLPC, ...
  const int cl = warp * Sh::kCPW + lane / Sh::kLPC;
  const int p = lane % Sh::kLPC;
  const bool lvalid = cl < nvalid;
  float Aj[NS], h[NS], h0[NS];
  float2 A2[NS], P[NS];
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const int n = p + j * Sh::kLPC;
    Aj[j] = (lvalid && n < N) ? a.A[(d0 + cl) * N + n] : 0.f;
    A2[j] = make_float2(Aj[j] * kLog2e, Aj[j] * kLog2e);
    h[j] = (lvalid && n < N && a.h_init != nullptr) ? a.h_init[(row0 + cl) * N + n] : 0.f;
    P[j] = make_float2(1.f, 1.f);
  }
  // A later piece starts from the state the earlier pieces leave: h_init carried through their
  // decays, plus their end states from zero (the recurrence is affine in its initial state).
  const int64_t rows = a.batch * a.dim;
  if (lvalid) {
    for (int q = 0; q < piece; ++q) {
#pragma unroll
      for (int j = 0; j < NS; ++j) {
        const int n = p + j * Sh::kLPC;
        if (n < N) {
          const int64_t at = ((int64_t)q * rows + row0 + cl) * N + n;
          h[j] = fmaf(a.piece_P[at], h[j], a.piece_e[at]);
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NS; ++j) h0[j] = h[j];
  float2 sd = make_float2(0.f, 0.f);

  // ---- row-piece tasks (staging and output): piece i covers channel tc[i], steps 4 * tq[i] + 0..3
  int tc[kTasks], tq[kTasks];
  float Dv[kTasks], bias[kTasks];
#pragma unroll
  for (int i = 0; i < kTasks; ++i) {
    const int q = tid + kThreads * i;
    tc[i] = q / kQuads;
    tq[i] = q % kQuads;
    const bool ok = tc[i] < nvalid;
    Dv[i] = (ok && a.D) ? a.D[d0 + tc[i]] : 0.f;
    bias[i] = (ok && a.delta_bias) ? a.delta_bias[d0 + tc[i]] : 0.f;
  }

  Quad<TI> ru[kTasks], rd[kTasks], rz[HAS_Z ? kTasks : 1];
  Quad<TW> rbc[kBCTasks];

  // Issue the global loads of chunk k into registers (no use of the results yet).
  auto load_chunk = [&](int k) {
    const int64_t t0 = (int64_t)k * kChunk;
    const bool full = t0 + kChunk <= L;
#pragma unroll
    for (int i = 0; i < kTasks; ++i) {
      const int64_t t = t0 + 4 * tq[i];
      if (tc[i] < nvalid) {
        // row (b, d0 + tc[i]) of u / delta / z: dense, or strided views in the STRIDED instantiations
        const int64_t dch = d0 + tc[i];
        const int64_t off = (row0 + tc[i]) * L;
        const TI* u = static_cast<const TI*>(a.u) + (STRIDED ? b * a.sub + dch * a.sud : off);
        const TI* dl = static_cast<const TI*>(a.delta) + (STRIDED ? b * a.sdb + dch * a.sdd : off);
        const TI* zr = HAS_Z ? static_cast<const TI*>(a.z) + (STRIDED ? b * a.szb + dch * a.szd : off) : nullptr;
        if (full && vec_io) {
          ru[i] = ld_quad_stream(u + t);
          rd[i] = ld_quad_stream(dl + t);
          if constexpr (HAS_Z) rz[i] = ld_quad_stream(zr + t);
        } else {
          ru[i] = ld_quad_masked(u, t, L, 1);
          rd[i] = ld_quad_masked(dl, t, L, 1);
          if constexpr (HAS_Z) rz[i] = ld_quad_masked(zr, t, L, 1);
        }
      } else {
        ru[i] = zero_quad<TI>();
        rd[i] = zero_quad<TI>();
        if constexpr (HAS_Z) rz[i] = zero_quad<TI>();
      }
    }
#pragma unroll
    for (int i = 0; i < kBCTasks; ++i) {
      const int r = tid + kThreads * i;
      const int mat = r / (kMaxState * kQuads);
      const int n = (r / kQuads) % kMaxState;
      const int64_t t = t0 + 4 * (r % kQuads);
      if (n < N) {
        const TW* src = mat ? Cb + n * a.sCn : Bb + n * a.sBn;
        const int64_t sl = mat ? a.sCl : a.sBl;
        rbc[i] = (full && vec_bc) ? ld_quad_cached(src + t) : ld_quad_masked(src, t, L, sl);
      } else {
        rbc[i] = zero_quad<TW>();
      }
    }
  };

  // Convert chunk k's loaded pieces and stage dt, dt * u and the B / C tile in shared memory.
  auto stage_chunk = [&](int k) {
    const int64_t t0 = (int64_t)k * kChunk;
#pragma unroll
    for (int i = 0; i < kTasks; ++i) {
      const float4 u = to_float4(ru[i]);
      const float4 dl = to_float4(rd[i]);
      const int64_t t = t0 + 4 * tq[i];
      const bool ok = tc[i] < nvalid;
      float e[4] = {dl.x, dl.y, dl.z, dl.w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        float v = e[m] + bias[i];
        v = softplus ? softplus_f(v) : v;
        e[m] = (ok && t + m < L) ? v : 0.f;
      }
      const float4 dt = make_float4(e[0], e[1], e[2], e[3]);
      st4s(&sm.dt[tc[i]][4 * tq[i]], dt);
      st4s(&sm.dtu[tc[i]][4 * tq[i]], make_float4(dt.x * u.x, dt.y * u.y, dt.z * u.z, dt.w * u.w));
      if constexpr (WRITE_OUT) st4s(&sm.u[tc[i]][4 * tq[i]], u);
      if constexpr (HAS_Z) st4s(&sm.z[tc[i]][4 * tq[i]], to_float4(rz[i]));
    }
#pragma unroll
    for (int i = 0; i < kBCTasks; ++i) {
      const int r = tid + kThreads * i;
      const int mat = r / (kMaxState * kQuads);
      const int n = (r / kQuads) % kMaxState;
      float* dst = mat ? &sm.C[n][4 * (r % kQuads)] : &sm.B[n][4 * (r % kQuads)];
      st4s(dst, to_float4(rbc[i]));
    }
  };

  // y of chunk k: sum the lanes' partials, add D * u, gate, store.
  auto write_out = [&](int k) {
    const int64_t t0 = (int64_t)k * kChunk;
    const bool full = t0 + kChunk <= L;
#pragma unroll
    for (int i = 0; i < kTasks; ++i) {
      if (tc[i] >= nvalid) continue;
      float4 y = ld4s(&sm.y[tc[i]][0][4 * tq[i]]);
      float2 ylo = lo2(y), yhi = hi2(y);
#pragma unroll
      for (int l = 1; l < Sh::kLPC; ++l) {
        const float4 o = ld4s(&sm.y[tc[i]][l][4 * tq[i]]);
        ylo = __fadd2_rn(ylo, lo2(o));
        yhi = __fadd2_rn(yhi, hi2(o));
      }
      const float4 u = ld4s(&sm.u[tc[i]][4 * tq[i]]);
      ylo = __ffma2_rn(make_float2(Dv[i], Dv[i]), lo2(u), ylo);
      yhi = __ffma2_rn(make_float2(Dv[i], Dv[i]), hi2(u), yhi);
      float4 o = make_float4(ylo.x, ylo.y, yhi.x, yhi.y);
      if constexpr (HAS_Z) {
        const float4 z = ld4s(&sm.z[tc[i]][4 * tq[i]]);
        o.x *= silu_f(z.x);
        o.y *= silu_f(z.y);
        o.z *= silu_f(z.z);
        o.w *= silu_f(z.w);
      }
      TI* orow = static_cast<TI*>(a.out) + (row0 + tc[i]) * L;
      const int64_t t = t0 + 4 * tq[i];
      if (full && vec_io)
        st_quad_stream(orow + t, o);
      else
        st_quad_masked(orow, t, L, o);
    }
  };

  const int nch = a.nchunks;
  const int k_lo = piece * a.piece_chunks;
  const int k_hi = min(nch, k_lo + a.piece_chunks);
  load_chunk(k_lo);
  stage_chunk(k_lo);
  __syncthreads();
  for (int k = k_lo; k < k_hi; ++k) {
    if (k + 1 < k_hi) load_chunk(k + 1);
    const int64_t t0 = (int64_t)k * kChunk;
    const int lim = (int)(L - t0 < kChunk ? L - t0 : kChunk);
    if (lim == kChunk)
      recur_chunk<NS, WRITE_OUT, false>(sm, cl, p, A2, h, P, sd, lim);
    else
      recur_chunk<NS, WRITE_OUT, true>(sm, cl, p, A2, h, P, sd, lim);

    // Chunk end: accurately rounded decay of the carried state (see the file comment). The
    // adjustment is skipped where it is not finite (overflowed or NaN states keep the plain
    // recurrence's value, as the reference's sequential loop would produce).
    const float sdt = sd.x + sd.y;
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const float exact = sdt == 0.f ? 1.f : expf(Aj[j] * sdt);
      const float adj = (exact - P[j].x * P[j].y) * h0[j];
      if (isfinite(adj)) h[j] += adj;
      h0[j] = h[j];
      P[j] = make_float2(1.f, 1.f);
    }
    sd = make_float2(0.f, 0.f);
    if (a.chunk_states != nullptr && lvalid) {
      float* st = a.chunk_states + ((row0 + cl) * nch + k) * N;
#pragma unroll
      for (int j = 0; j < NS; ++j) {
        const int n = p + j * Sh::kLPC;
        if (n < N) st[n] = h[j];
      }
    }
    __syncthreads();  // partial sums complete; everyone is done reading this chunk's tiles
    if constexpr (WRITE_OUT) write_out(k);
    if (k + 1 < k_hi) stage_chunk(k + 1);
    __syncthreads();
  }
  if (a.last_state != nullptr && lvalid && piece == a.pieces - 1) {
    float* st = a.last_state + (row0 + cl) * N;
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const int n = p + j * Sh::kLPC;
      if (n < N) st[n] = h[j];
    }
  }
}

template <typename TI, typename TW, int NS, bool HAS_Z, bool WRITE_OUT, bool STRIDED>
cudaError_t launch_one(const ScanArgs& a, dim3 grid, cudaStream_t stream) {
  auto kern = scan_fwd_kernel<TI, TW, NS, HAS_Z, WRITE_OUT, STRIDED>;
  constexpr size_t smem = sizeof(FwdSmem<NS>);
  // The attribute belongs to the current device: set it on every launch (a host-side call of a
  // few microseconds), so a process that runs on several GPUs gets it on each of them.
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

template <typename TI, typename TW, int NS>
cudaError_t launch_typed(ScanArgs a, bool write_out, cudaStream_t stream) {
  constexpr int CPC = FwdShape<NS>::kCPC;
  a.tiles = (int)((a.dpg + CPC - 1) / CPC);
  const dim3 grid((unsigned)(a.tiles * a.batch * a.ngroups * a.pieces));
  if (io_rows_strided(a)) {
    if (!write_out) return launch_one<TI, TW, NS, false, false, true>(a, grid, stream);
    if (a.z != nullptr) return launch_one<TI, TW, NS, true, true, true>(a, grid, stream);
    return launch_one<TI, TW, NS, false, true, true>(a, grid, stream);
  }
  if (!write_out) return launch_one<TI, TW, NS, false, false, false>(a, grid, stream);
  if (a.z != nullptr) return launch_one<TI, TW, NS, true, true, false>(a, grid, stream);
  return launch_one<TI, TW, NS, false, true, false>(a, grid, stream);
}

template <typename TI, typename TW>
cudaError_t launch_ns(const ScanArgs& a, bool write_out, cudaStream_t stream) {
  if (fwd_states_per_lane(a.batch * a.dim, a.nchunks) == 1) return launch_typed<TI, TW, 1>(a, write_out, stream);
  return launch_typed<TI, TW, 2>(a, write_out, stream);
}

}  // namespace

int fwd_states_per_lane(int64_t rows, int nchunks) {
  // Two states per lane halve the lanes (and the y partial sums) per channel; one state per lane
  // doubles the warps, which short rows of small problems need to fill 148 SMs. Long rows (64
  // chunks and more) keep two and are split into sequence pieces instead when they are few.
  return rows < 4096 && nchunks < 64 ? 1 : 2;
}

int64_t fwd_ctas(const ScanArgs& a) {
  const int64_t cpc = fwd_states_per_lane(a.batch * a.dim, a.nchunks) == 1 ? FwdShape<1>::kCPC : FwdShape<2>::kCPC;
  return (a.dpg + cpc - 1) / cpc * a.batch * a.ngroups;
}

cudaError_t read_fault_fwd(int* out) {
  *out = 0;  // the forward has no bounded waits
  return cudaSuccess;
}

namespace {

cudaError_t launch_dtypes(const ScanArgs& a, int io_dtype, int bc_dtype, bool write_out, cudaStream_t stream) {
  if (io_dtype == MB200_F32) return launch_ns<float, float>(a, write_out, stream);
  if (io_dtype == MB200_BF16) {
    if (bc_dtype == MB200_BF16) return launch_ns<__nv_bfloat16, __nv_bfloat16>(a, write_out, stream);
    return launch_ns<__nv_bfloat16, float>(a, write_out, stream);
  }
  if (bc_dtype == MB200_F16) return launch_ns<__half, __half>(a, write_out, stream);
  return launch_ns<__half, float>(a, write_out, stream);
}

}  // namespace

cudaError_t launch_scan_fwd(const ScanArgs& a, int io_dtype, int bc_dtype, bool write_out,
                            cudaStream_t stream) {
  if (a.batch == 0 || a.dim == 0) return cudaSuccess;
  if (a.pieces > 1) {  // summaries of pieces 0 .. pieces - 2, which the pieces after them start from
    const cudaError_t e = launch_fwd_piece_summary(a, io_dtype, bc_dtype, stream);
    if (e != cudaSuccess) return e;
  }
  return launch_dtypes(a, io_dtype, bc_dtype, write_out, stream);
}

}  // namespace mb200
