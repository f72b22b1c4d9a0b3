// ssd.cu -- Mamba-2 SSD chunk scan forward (mamba_chunk_scan_combined) on sm_100a tensor cores.
//
// Per (batch, head) the state is a headdim x dstate matrix with one scalar decay per step, so a
// chunk of Q = 128 steps is four small matrix products (the SSD chunk form of the recurrence,
// Dao & Gu 2024, "Transformers are SSMs", section 6):
//   G      = C B^T                          (Q x Q)           scores of step i against step j
//   M      = G o L,  L[i, j] = exp(cs_i - cs_j) dt_j  (j <= i), 0 above the diagonal
//   Y      = M X  +  diag(exp(cs)) C S_prev^T + D x          (Q x headdim)
//   S_next = exp(cs_Q) S_prev + X'^T B,  X'[j] = exp(cs_Q - cs_j) dt_j X[j]
// with cs the inclusive cumulative sum of dt A inside the chunk. The chunks of a (batch, head)
// are walked in order by one CTA, which carries S (float32, in registers) from chunk to chunk;
// CTAs split headdim into 32-wide tiles (S's columns are independent), so the grid is
// batch x nheads x headdim / 32.
//
// Tensor cores: every product is one tcgen05.mma (kind::f16, bf16 operands, float32 accumulators
// in Tensor Memory, M = 128) issued by one thread, operands in shared memory in the no-swizzle
// core-matrix layout (8 rows x 16 bytes per 128-byte core matrix), completion signalled on an
// mbarrier by tcgen05.commit. The bf16 copy of S that feeds C S^T is split in two (S = hi + lo,
// both bf16), so the carried state enters the product with ~16 significant bits; M and X' are
// rounded to bf16 once.
//
// Shared memory (PT = 32 headdim columns per CTA, 98 KB, two CTAs per SM):
//   sCM  [128 t][128 n]  C tile, then (once C B^T and C S^T are done) M [128 i][128 j]
//   sB   [128 t][128 n]  B tile; K-major operand of C B^T, MN-major operand of X'^T B
//   sX   [128 t][PT]     X tile (MN-major operand of M X)
//   sXs  [128 t][PT]     X' (MN-major operand of X'^T B)
//   sSh, sSl [128 n][PT] bf16 hi / lo parts of S (MN-major operand of C S^T)
// dstate is zero-padded to 128 (the padded columns of B stay zero, so S's padded rows stay zero).
// TMEM (256 columns): [0, 128) G, then M X; [128, 128 + PT) C S^T; [128 + PT, 128 + 2 PT) X'^T B.
// Thread i of the 128 reads row i of every accumulator (TMEM lane i).
#include "common.cuh"
#include "stage.cuh"
#include "tmem.cuh"

namespace mb200 {

namespace {

constexpr int kQ = 128;        // steps per chunk (the M of every product)
constexpr int kNP = 128;       // dstate padded
constexpr int kPT = 32;        // headdim columns per CTA
constexpr int kSsdThreads = 128;
constexpr uint32_t kSsdTmemCols = 256;

constexpr int kTileCM = kQ * kNP * 2;   // bytes
constexpr int kTileB = kQ * kNP * 2;
constexpr int kTileX = kQ * kPT * 2;
constexpr int kTileS = kNP * kPT * 2;
constexpr int kOffB = kTileCM;
constexpr int kOffX = kOffB + kTileB;
constexpr int kOffXs = kOffX + kTileX;
constexpr int kOffSh = kOffXs + kTileX;
constexpr int kOffSl = kOffSh + kTileS;
constexpr int kOffF = kOffSl + kTileS;             // float area
constexpr int kFloats = 2 * kQ + 8 + kPT;          // dt, cs, warp sums, D
constexpr int kOffBar = kOffF + kFloats * 4;
constexpr int kSsdSmem = kOffBar + 16;

struct SsdArgs {
  const __nv_bfloat16* x;
  const float* dt;
  const float* A;
  const __nv_bfloat16* B;
  const __nv_bfloat16* C;
  const float* D;
  const __nv_bfloat16* z;
  const float* dt_bias;
  const float* init;
  __nv_bfloat16* out;
  float* final_states;
  int64_t L, H, P, G, N;
  int64_t xbs, xls, xhs, zbs, zls, zhs, Bbs, Bls, Bgs, Cbs, Cls, Cgs, dtbs, dtls;
  float dt_min, dt_max;
  int softplus, D_per_dim;
  int ntiles;  // P / kPT
};

// Byte offset of the 16-byte piece (row r, column chunk c8 = column / 8) of a core-matrix tiled
// bf16 tile with `cols` columns: core matrix (r / 8, c8) holds rows r..r+7 x 8 columns, 128 bytes.
__device__ __forceinline__ uint32_t core16(int r, int c8, int cols) {
  return (uint32_t)(((r >> 3) * (cols >> 3) + c8) * 128 + (r & 7) * 16);
}

// Shared-memory matrix descriptor, no swizzle (sm_100 version 1): start address, leading byte
// offset (between core matrices adjacent along K) and stride byte offset (between core matrices
// adjacent along M / N), all in 16-byte units.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16: bf16 A and B, float32 accumulator, M x N, operand majors
// (0 = K-major, 1 = MN-major).
constexpr uint32_t idesc_bf16(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack_bf16(uint32_t w) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}

// A [rows][cols] bf16 tile piece by piece from global rows (row r at base + r * row_stride
// elements, 16-byte aligned), rows >= valid_rows zero-filled.
__device__ __forceinline__ void load_tile(uint32_t s_tile, const __nv_bfloat16* base, int64_t row_stride,
                                          int rows, int cols_loaded, int cols, int valid_rows, int tid) {
  const int nc8 = cols_loaded >> 3;
  for (int i = tid; i < rows * nc8; i += kSsdThreads) {
    const int r = i / nc8, c8 = i - r * nc8;
    const bool ok = r < valid_rows;
    const __nv_bfloat16* src = base + (ok ? (int64_t)r * row_stride : 0) + c8 * 8;
    cp_async16(s_tile + core16(r, c8, cols), src, ok ? 16u : 0u);
  }
}

__global__ void __launch_bounds__(kSsdThreads, 2) ssd_fwd_kernel(SsdArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x % a.ntiles;
  const int64_t bh = blockIdx.x / a.ntiles;
  const int64_t h = bh % a.H, b = bh / a.H;
  const int64_t g = h / (a.H / a.G);
  const int p0 = tile * kPT;

  float* sdt = reinterpret_cast<float*>(smem + kOffF);
  float* scs = sdt + kQ;
  float* swarp = scs + kQ;
  float* sD = swarp + 8;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kOffBar + 8);
  const uint32_t s0 = smem_u32(smem);
  const uint32_t sCM = s0, sB = s0 + kOffB, sX = s0 + kOffX, sXs = s0 + kOffXs, sSh = s0 + kOffSh,
                 sSl = s0 + kOffSl;

  if (warp == 0) tmem_alloc(tslot, kSsdTmemCols);
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  const int N = (int)a.N;
  const int nc8 = N / 8;                       // 16-byte pieces of a B / C row
  const int ksteps = (N + 15) / 16;            // K steps of the dstate contractions
  // zero the padded dstate columns of B (kept zero) and, if dstate is an odd multiple of 8, the
  // piece of C the last K step reads past dstate (re-zeroed every chunk, as M overwrites it)
  for (int i = tid; i < kQ * (16 - nc8); i += kSsdThreads) {
    const int r = i / (16 - nc8), c8 = nc8 + i % (16 - nc8);
    *reinterpret_cast<uint4*>(smem + kOffB + core16(r, c8, kNP)) = make_uint4(0, 0, 0, 0);
  }
  if (tid < kPT) {
    float dv = 0.f;
    if (a.D != nullptr) dv = a.D_per_dim ? a.D[h * a.P + p0 + tid] : a.D[h];
    sD[tid] = dv;
  }
  // S row n = tid (float32), initial state or zeros
  float S[kPT];
  {
    const int n = tid;
#pragma unroll
    for (int p = 0; p < kPT; ++p)
      S[p] = (a.init != nullptr && n < N) ? a.init[((b * a.H + h) * a.P + p0 + p) * a.N + n] : 0.f;
  }
  const float A2 = a.A[h] * kLog2e;
  const float bias = a.dt_bias != nullptr ? a.dt_bias[h] : 0.f;

  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tbase = *tslot;
  const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);  // this warp's lanes

  constexpr uint32_t kIdG = idesc_bf16(kQ, kQ, 0, 0);
  constexpr uint32_t kIdY = idesc_bf16(kQ, kPT, 0, 1);
  constexpr uint32_t kIdS = idesc_bf16(kNP, kPT, 1, 1);
  constexpr uint32_t kLboK = 128, kSboK = (kNP / 8) * 128;      // K-major 128-column tiles
  constexpr uint32_t kLboP = (kPT / 8) * 128, kSboP = 128;      // MN-major PT-column tiles
  constexpr uint32_t kColYo = kQ, kColSl = kQ + kPT;

  uint32_t phase = 0;
  const int64_t nchunks = (a.L + kQ - 1) / kQ;
  for (int64_t k = 0; k < nchunks; ++k) {
    const int64_t t0 = k * kQ;
    const int valid = (int)(a.L - t0 < kQ ? a.L - t0 : kQ);

    // ---- S_prev as bf16 hi + lo (row n = tid), the chunk's tiles, dt and its cumulative sum
    {
      const int n = tid;
#pragma unroll
      for (int c8 = 0; c8 < kPT / 8; ++c8) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float v0 = S[c8 * 8 + 2 * q], v1 = S[c8 * 8 + 2 * q + 1];
          hi[q] = pack_bf16(v0, v1);
          const float2 hv = unpack_bf16(hi[q]);
          lo[q] = pack_bf16(v0 - hv.x, v1 - hv.y);
        }
        *reinterpret_cast<uint4*>(smem + kOffSh + core16(n, c8, kPT)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(smem + kOffSl + core16(n, c8, kPT)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
    }
    load_tile(sCM, a.C + b * a.Cbs + t0 * a.Cls + g * a.Cgs, a.Cls, kQ, N, kNP, valid, tid);
    load_tile(sB, a.B + b * a.Bbs + t0 * a.Bls + g * a.Bgs, a.Bls, kQ, N, kNP, valid, tid);
    load_tile(sX, a.x + b * a.xbs + t0 * a.xls + h * a.xhs + p0, a.xls, kQ, kPT, kPT, valid, tid);
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (nc8 & 1)  // C columns [dstate, dstate + 8) of the last K step
      *reinterpret_cast<uint4*>(smem + core16(tid, nc8, kNP)) = make_uint4(0, 0, 0, 0);
    float cs;
    {
      float dtv = 0.f;
      if (tid < valid) {
        float raw = a.dt[b * a.dtbs + (t0 + tid) * a.dtls + h] + bias;
        if (a.softplus) raw = softplus_f(raw);
        dtv = fminf(fmaxf(raw, a.dt_min), a.dt_max);
      }
      sdt[tid] = dtv;
      float v = dtv * A2;  // log2 units
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (lane == 31) swarp[warp] = v;
      __syncthreads();
      for (int w = 0; w < warp; ++w) v += swarp[w];
      cs = v;
      scs[tid] = v;
    }
    cp_async_wait_all();
    fence_proxy_async();
    tmem_fence_before_sync();
    __syncthreads();
    const float cs_end = scs[kQ - 1];

    // ---- G = C B^T and Yo = C S^T (hi, then lo)
    if (tid == 0) {
      tmem_fence_after_sync();
      for (int s = 0; s < ksteps; ++s)
        umma_bf16(tbase, sdesc(sCM + s * 256, kLboK, kSboK), sdesc(sB + s * 256, kLboK, kSboK), kIdG, s > 0);
      for (int s = 0; s < ksteps; ++s)
        umma_bf16(tbase + kColYo, sdesc(sCM + s * 256, kLboK, kSboK), sdesc(sSh + s * 2 * kLboP, kLboP, kSboP), kIdY,
                  s > 0);
      for (int s = 0; s < ksteps; ++s)
        umma_bf16(tbase + kColYo, sdesc(sCM + s * 256, kLboK, kSboK), sdesc(sSl + s * 2 * kLboP, kLboP, kSboP), kIdY,
                  1);
      umma_commit(bar);
    }
    mbar_wait(bar, phase);
    phase ^= 1;
    tmem_fence_after_sync();

    // ---- M = G o L (row i = tid) over C's tile, and X' = w X
    {
      const int i = tid;
#pragma unroll 1
      for (int q = 0; q < kQ / 16; ++q) {
        uint4 w0 = make_uint4(0, 0, 0, 0), w1 = make_uint4(0, 0, 0, 0);
        if (q <= 2 * warp + 1) {  // warp-uniform: some row of this warp reaches column 16 q
          float gv[16];
          tmem_ld16(trow + q * 16, gv);
          tmem_wait_ld();
          uint32_t pk[8];
#pragma unroll
          for (int jj = 0; jj < 16; jj += 2) {
            const int j = q * 16 + jj;
            const float4 cj = *reinterpret_cast<const float4*>(&scs[j & ~3]);
            const float c0 = (jj & 2) ? cj.z : cj.x, c1 = (jj & 2) ? cj.w : cj.y;
            const float m0 = j <= i ? gv[jj] * ex2(cs - c0) * sdt[j] : 0.f;
            const float m1 = j + 1 <= i ? gv[jj + 1] * ex2(cs - c1) * sdt[j + 1] : 0.f;
            pk[jj / 2] = pack_bf16(m0, m1);
          }
          w0 = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          w1 = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
        *reinterpret_cast<uint4*>(smem + core16(i, 2 * q, kQ)) = w0;
        *reinterpret_cast<uint4*>(smem + core16(i, 2 * q + 1, kQ)) = w1;
      }
      const float wx = ex2(cs_end - cs) * sdt[i];
#pragma unroll
      for (int c8 = 0; c8 < kPT / 8; ++c8) {
        const uint4 v = *reinterpret_cast<const uint4*>(smem + kOffX + core16(i, c8, kPT));
        const uint32_t in[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16(in[e]);
          o[e] = pack_bf16(f.x * wx, f.y * wx);
        }
        *reinterpret_cast<uint4*>(smem + kOffXs + core16(i, c8, kPT)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    fence_proxy_async();
    tmem_fence_before_sync();
    __syncthreads();

    // ---- Yd = M X (into G's columns) and Sl = X'^T B
    if (tid == 0) {
      tmem_fence_after_sync();
      for (int s = 0; s < kQ / 16; ++s)
        umma_bf16(tbase, sdesc(sCM + s * 256, kLboK, kSboK), sdesc(sX + s * 2 * kLboP, kLboP, kSboP), kIdY, s > 0);
      for (int s = 0; s < kQ / 16; ++s)
        umma_bf16(tbase + kColSl, sdesc(sB + s * 2 * kSboK, kSboK, 128), sdesc(sXs + s * 2 * kLboP, kLboP, kSboP),
                  kIdS, s > 0);
      umma_commit(bar);
    }
    mbar_wait(bar, phase);
    phase ^= 1;
    tmem_fence_after_sync();

    // ---- outputs of row i = tid, and the carried state (row n = tid)
    {
      float yo[kPT], yd[kPT], sl[kPT];
      tmem_ld16(trow + kColYo, *reinterpret_cast<float(*)[16]>(&yo[0]));
      tmem_ld16(trow + kColYo + 16, *reinterpret_cast<float(*)[16]>(&yo[16]));
      tmem_ld16(trow, *reinterpret_cast<float(*)[16]>(&yd[0]));
      tmem_ld16(trow + 16, *reinterpret_cast<float(*)[16]>(&yd[16]));
      tmem_ld16(trow + kColSl, *reinterpret_cast<float(*)[16]>(&sl[0]));
      tmem_ld16(trow + kColSl + 16, *reinterpret_cast<float(*)[16]>(&sl[16]));
      tmem_wait_ld();
      const int i = tid;
      if (i < valid) {
        const float eo = ex2(cs);
        const int64_t t = t0 + i;
        __nv_bfloat16* orow = a.out + ((b * a.L + t) * a.H + h) * a.P + p0;
        const __nv_bfloat16* zrow = a.z != nullptr ? a.z + b * a.zbs + t * a.zls + h * a.zhs + p0 : nullptr;
#pragma unroll
        for (int c8 = 0; c8 < kPT / 8; ++c8) {
          const uint4 xv = *reinterpret_cast<const uint4*>(smem + kOffX + core16(i, c8, kPT));
          const uint32_t xin[4] = {xv.x, xv.y, xv.z, xv.w};
          uint32_t zin[4] = {0, 0, 0, 0};
          if (zrow != nullptr) {
            const uint4 zv = __ldg(reinterpret_cast<const uint4*>(zrow + c8 * 8));
            zin[0] = zv.x, zin[1] = zv.y, zin[2] = zv.z, zin[3] = zv.w;
          }
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int p = c8 * 8 + 2 * e;
            const float2 xf = unpack_bf16(xin[e]);
            float y0 = fmaf(eo, yo[p], yd[p]) + sD[p] * xf.x;
            float y1 = fmaf(eo, yo[p + 1], yd[p + 1]) + sD[p + 1] * xf.y;
            if (zrow != nullptr) {
              const float2 zf = unpack_bf16(zin[e]);
              y0 *= silu_f(zf.x);
              y1 *= silu_f(zf.y);
            }
            o[e] = pack_bf16(y0, y1);
          }
          *reinterpret_cast<uint4*>(orow + c8 * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      const float decay = ex2(cs_end);
#pragma unroll
      for (int p = 0; p < kPT; ++p) S[p] = fmaf(decay, S[p], sl[p]);
    }
    tmem_fence_before_sync();
    __syncthreads();
  }

  if (a.final_states != nullptr && tid < N) {
#pragma unroll
    for (int p = 0; p < kPT; ++p) a.final_states[((b * a.H + h) * a.P + p0 + p) * a.N + tid] = S[p];
  }
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, kSsdTmemCols);
}

}  // namespace

cudaError_t read_fault_ssd(int* out) { return read_fault_word(out); }

}  // namespace mb200

using namespace mb200;

extern "C" {

MB200_API int mb200_ssd_chunk_scan_fwd(const mb200_ssd_params* p, void* stream) {
  if (p == nullptr) return MB200_ERR_NULL_POINTER;
  if (p->x == nullptr || p->dt == nullptr || p->A == nullptr || p->B == nullptr || p->C == nullptr ||
      p->out == nullptr)
    return MB200_ERR_NULL_POINTER;
  if (p->batch < 0 || p->seqlen < 0 || p->nheads < 0 || p->headdim <= 0 || p->ngroups <= 0 || p->dstate <= 0)
    return MB200_ERR_BAD_SHAPE;
  if (p->nheads % p->ngroups != 0) return MB200_ERR_BAD_SHAPE;
  if (p->x_dtype != MB200_BF16) return p->x_dtype == MB200_F32 || p->x_dtype == MB200_F16 ? MB200_ERR_UNSUPPORTED
                                                                                          : MB200_ERR_BAD_DTYPE;
  if (p->dstate % 8 != 0 || p->dstate > kNP || p->headdim % kPT != 0 || p->headdim > 256)
    return MB200_ERR_UNSUPPORTED;
  // 16-byte pieces: row starts of x, z, B, C and out aligned
  const bool al = aligned16(p->x) && aligned16(p->B) && aligned16(p->C) && aligned16(p->out) &&
                  (p->z == nullptr || aligned16(p->z)) && p->x_batch_stride % 8 == 0 && p->x_seqlen_stride % 8 == 0 &&
                  p->x_head_stride % 8 == 0 && p->B_batch_stride % 8 == 0 && p->B_seqlen_stride % 8 == 0 &&
                  p->B_group_stride % 8 == 0 && p->C_batch_stride % 8 == 0 && p->C_seqlen_stride % 8 == 0 &&
                  p->C_group_stride % 8 == 0 &&
                  (p->z == nullptr ||
                   (p->z_batch_stride % 8 == 0 && p->z_seqlen_stride % 8 == 0 && p->z_head_stride % 8 == 0));
  if (!al) return MB200_ERR_BAD_LAYOUT;
  reset_launches();
  const int64_t ntiles = p->headdim / kPT;
  const int64_t ctas = p->batch * p->nheads * ntiles;
  if (ctas == 0) return MB200_OK;
  if (ctas > 0x7fffffff) return MB200_ERR_UNSUPPORTED;
  SsdArgs a;
  a.x = static_cast<const __nv_bfloat16*>(p->x);
  a.dt = p->dt;
  a.A = p->A;
  a.B = static_cast<const __nv_bfloat16*>(p->B);
  a.C = static_cast<const __nv_bfloat16*>(p->C);
  a.D = p->D;
  a.z = static_cast<const __nv_bfloat16*>(p->z);
  a.dt_bias = p->dt_bias;
  a.init = p->initial_states;
  a.out = static_cast<__nv_bfloat16*>(p->out);
  a.final_states = p->final_states;
  a.L = p->seqlen, a.H = p->nheads, a.P = p->headdim, a.G = p->ngroups, a.N = p->dstate;
  a.xbs = p->x_batch_stride, a.xls = p->x_seqlen_stride, a.xhs = p->x_head_stride;
  a.zbs = p->z_batch_stride, a.zls = p->z_seqlen_stride, a.zhs = p->z_head_stride;
  a.Bbs = p->B_batch_stride, a.Bls = p->B_seqlen_stride, a.Bgs = p->B_group_stride;
  a.Cbs = p->C_batch_stride, a.Cls = p->C_seqlen_stride, a.Cgs = p->C_group_stride;
  a.dtbs = p->dt_batch_stride, a.dtls = p->dt_seqlen_stride;
  a.dt_min = p->dt_min, a.dt_max = p->dt_max;
  a.softplus = p->dt_softplus != 0;
  a.D_per_dim = p->D_per_dim != 0;
  a.ntiles = (int)ntiles;
  cudaError_t e = cudaFuncSetAttribute(ssd_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSsdSmem);
  if (e != cudaSuccess) return MB200_ERR_CUDA;
  ssd_fwd_kernel<<<(unsigned)ctas, kSsdThreads, kSsdSmem, static_cast<cudaStream_t>(stream)>>>(a);
  if (cudaGetLastError() != cudaSuccess) return MB200_ERR_CUDA;
  note_launches(1);
  return MB200_OK;
}

}  // extern "C"
