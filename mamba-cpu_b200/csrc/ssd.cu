// ssd.cu -- Mamba-2 SSD chunk scan forward (mamba_chunk_scan_combined) on sm_100a tensor cores.
//
// Per (batch, head) the state is a headdim x dstate matrix with one scalar decay per step, so a
// chunk of Q = 64 steps is four small matrix products (the SSD chunk form of the recurrence,
// Dao & Gu 2024, "Transformers are SSMs", section 6):
//   G      = C B^T                          (Q x Q)           scores of step i against step j
//   M      = G o L,  L[i, j] = exp(cs_i - cs_j) dt_j  (j <= i), 0 above the diagonal
//   Y      = M X  +  diag(exp(cs)) C S_prev^T + D x          (Q x headdim)
//   S_next = exp(cs_Q) S_prev + X'^T B,  X'[j] = exp(cs_Q - cs_j) dt_j X[j]
// with cs the inclusive cumulative sum of dt A inside the chunk. The chunks of a (batch, head)
// are walked in order by one CTA, which carries S (float32, in registers) from chunk to chunk;
// CTAs split headdim into 32-wide tiles (S's columns are independent), so the grid is
// batch x nheads x headdim / 32. A CTA is small (128 threads, ~53 KB of shared memory, 128 TMEM
// columns) so that four fit on an SM and a whole Mamba-2 layer's grid is resident at once.
//
// Tensor cores: every product is one tcgen05.mma (kind::f16, bf16 or fp16 operands -- the input's
// 16-bit type --, float32 accumulators
// in Tensor Memory) issued by one thread, operands in shared memory in the no-swizzle core-matrix
// layout (8 rows x 16 bytes per 128-byte core matrix), completion signalled on an mbarrier by
// tcgen05.commit. G, C S^T and M X have M = 64 (row m of the accumulator in TMEM lane
// (m % 16) + 32 (m / 16), i.e. lanes 0-15 of each warp's quarter); X'^T B has M = 128 (row n in
// lane n). The 16-bit copy of S that feeds C S^T is split in two (S = hi + lo), so the carried
// state enters the product with about twice the 16-bit type's precision; M and X' are rounded to
// the 16-bit type once.
//
// Shared memory (PT = 32 headdim columns per CTA). Every tile is stored as [column piece c8][row
// r][8 elements]: 16 bytes per (row, 8 columns), so core matrix (r / 8, c8) -- 8 rows x 16 bytes
// -- is 128 contiguous bytes, the rows of one column piece are contiguous, and the same bytes
// serve as a K-major operand (rows = M / N) or an MN-major one (rows = K). A 5-D TMA tensor map
// per input (8 elements, seqlen, column pieces, group / head, batch) writes exactly this order, so
// one bulk tensor copy loads a tile; rows past seqlen are zero-filled by the copy.
//   sCM  [16][64 t]      C tile, then (once C B^T and C S^T are done) M [64 i][64 j] in its
//                        first 8 pieces
//   sB   [16][64 t]      B tile; K-major operand of C B^T, MN-major operand of X'^T B
//   sX   [PT/8][64 t]    X tile (MN-major operand of M X)
//   sSh, sSl [PT/8][128 n]  16-bit hi / lo parts of S (MN-major operand of C S^T); X' [PT/8][64 t]
//                        reuses sSl once C S^T is done
// dstate is zero-padded to 128 (the padded columns of B stay zero, so S's padded rows stay zero).
// TMEM (128 columns): [0, 64) G, then M X in [0, PT); [64, 64 + PT) C S^T; [96, 128) X'^T B.
// The chunk's tiles are copied in while the previous chunk's outputs are written: the copies for
// chunk k + 1 are issued as soon as chunk k's last products have completed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "stage.cuh"
#include "tmem.cuh"

namespace mb200 {

namespace {

constexpr int kQ = 64;         // steps per chunk
constexpr int kNP = 128;       // dstate padded
constexpr int kPT = 32;        // headdim columns per CTA
constexpr int kSsdThreads = 128;
constexpr uint32_t kSsdTmemCols = 128;

constexpr int kTileCM = kQ * kNP * 2;   // bytes
constexpr int kTileB = kQ * kNP * 2;
constexpr int kTileX = kQ * kPT * 2;
constexpr int kTileS = kNP * kPT * 2;
constexpr int kOffB = kTileCM;
constexpr int kOffX = kOffB + kTileB;
constexpr int kOffSh = kOffX + kTileX;
constexpr int kOffSl = kOffSh + kTileS;
constexpr int kOffXs = kOffSl;                     // X' reuses the lo part of S
constexpr int kOffF = kOffSl + kTileS;             // float area
constexpr int kFloats = 3 * kQ + 8 + kPT;          // dt, cs, sequence ids (int), warp sums, D
constexpr int kOffBar = kOffF + kFloats * 4;
constexpr int kSsdSmem = kOffBar + 32;

struct SsdArgs {
  const uint16_t* x;  // bf16 or fp16 bits (the F16 template argument)
  const float* dt;
  const float* A;
  const uint16_t* B;
  const uint16_t* C;
  const float* D;
  const uint16_t* z;
  const float* dt_bias;
  const float* init;
  uint16_t* out;
  float* final_states;
  int64_t L, H, P, G, N;
  int64_t xbs, xls, xhs, zbs, zls, zhs, Bbs, Bls, Bgs, Cbs, Cls, Cgs, dtbs, dtls;
  const int32_t* seq_idx;  // (batch, seqlen) or null
  int64_t sqbs, sqls;
  float dt_min, dt_max;
  int softplus, D_per_dim;
  int ntiles;  // P / kPT
};

// Byte offset of the 16-byte piece (row r, column piece c8 = column / 8) of a tile with `rows` rows.
__device__ __forceinline__ uint32_t core16(int r, int c8, int rows = kQ) { return (uint32_t)((c8 * rows + r) * 16); }

// Shared-memory matrix descriptor, no swizzle (sm_100 version 1): start address, leading byte
// offset (between core matrices adjacent along K) and stride byte offset (between core matrices
// adjacent along M / N), all in 16-byte units.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16: A and B both bf16 (format 1) or both fp16 (format 0), float32
// accumulator, M x N, operand majors (0 = K-major, 1 = MN-major).
constexpr uint32_t idesc_16(int M, int N, int a_mn, int b_mn, bool f16) {
  return (1u << 4) | ((f16 ? 0u : 1u) << 7) | ((f16 ? 0u : 1u) << 10) | ((uint32_t)a_mn << 15) |
         ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
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

// Two floats to / from a pair of 16-bit values (bf16, or fp16 when F16).
template <bool F16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (F16) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}
template <bool F16>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if constexpr (F16)
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  else
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}

// Wait for the mbarrier phase with the given parity (tensor-core or copy completion): try_wait
// with a suspend-time hint, so a waiting warp sleeps (and leaves its issue slots to the other
// CTAs of the SM) until the phase completes; bounded by 2 s of GPU time (%globaltimer). On timeout
// the fault word records it and the kernel carries on.
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_wait_spin(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const uint64_t t_start = global_ns();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity), "r"(1000000u)
        : "memory");
    if (done) return;
    if (global_ns() - t_start > 2000000000ull) break;
  }
  atomicOr(&g_mb200_fault, kFaultWaitTimeout);
}

// One 5-D bulk tensor copy (TMA, no multicast) of the box at coordinates c0..c4 into shared memory,
// completing on `bar` (transaction bytes).
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            int c4, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_u32(bar))
      : "memory");
}

struct SsdMaps {
  CUtensorMap B, C, x;
};

// Thread roles (128 threads, 4 warps): S row n = tid (TMEM lane n of X'^T B). The 64-row
// accumulators live in lanes 0-15 of each warp's quarter, so lane l < 16 of warp w owns chunk row
// i = 16 w + l (masked decay matrix, outputs) and lane l >= 16 owns row 16 w + l - 16 of X'.
// SEQ: packed sequences (seq_idx); the other instantiation drops the sequence masks. F16: fp16
// x / z / B / C (and fp16 operands of every product) instead of bf16.
template <bool SEQ, bool F16>
__global__ void __launch_bounds__(kSsdThreads, 4) ssd_fwd_kernel(SsdArgs a, const __grid_constant__ SsdMaps maps) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool lo16 = lane < 16;
  const int crow = 16 * warp + (lane & 15);  // this thread's chunk row (M phase, outputs or X')
  const int tile = blockIdx.x % a.ntiles;
  const int64_t bh = blockIdx.x / a.ntiles;
  const int64_t h = bh % a.H, b = bh / a.H;
  const int64_t g = h / (a.H / a.G);
  const int p0 = tile * kPT;

  float* sdt = reinterpret_cast<float*>(smem + kOffF);
  float* scs = sdt + kQ;
  int* sseq = reinterpret_cast<int*>(scs + kQ);  // sequence id of each step of the chunk
  float* swarp = reinterpret_cast<float*>(sseq + kQ);
  float* sD = swarp + 8;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);       // tensor-core completion
  uint64_t* tbar = reinterpret_cast<uint64_t*>(smem + kOffBar + 8);  // tile copies
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kOffBar + 16);
  const uint32_t s0 = smem_u32(smem);
  const uint32_t sCM = s0, sB = s0 + kOffB, sX = s0 + kOffX, sXs = s0 + kOffXs, sSh = s0 + kOffSh,
                 sSl = s0 + kOffSl;
  const int N = (int)a.N;
  const int nc8 = N / 8;                       // 16-byte pieces of a B / C row
  const int ksteps = (N + 15) / 16;            // K steps of the dstate contractions
  const int64_t nchunks = (a.L + kQ - 1) / kQ;
  const uint32_t tile_bytes = (uint32_t)(2 * kQ * 16 * nc8 + kTileX);

  if (warp == 0) tmem_alloc(tslot, kSsdTmemCols);
  // zero the padded dstate columns of B and C (the copies never write them; M overwrites C's
  // first 8 pieces, which are re-zeroed where needed in the chunk loop)
  for (int i = tid; i < kQ * 16; i += kSsdThreads) {
    const int r = i & (kQ - 1), c8 = i / kQ;
    if (c8 >= nc8) {
      *reinterpret_cast<uint4*>(smem + kOffB + core16(r, c8)) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(smem + core16(r, c8)) = make_uint4(0, 0, 0, 0);
    }
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(tbar, 1);
    mbar_fence_init();
  }
  fence_proxy_async();  // the zeroed pieces before the first copy and product
  __syncthreads();
  if (tid == 0 && nchunks > 0) {
    mbar_arrive_expect_tx(tbar, tile_bytes);
    tma_load_5d(sCM, &maps.C, 0, 0, 0, (int)g, (int)b, tbar);
    tma_load_5d(sB, &maps.B, 0, 0, 0, (int)g, (int)b, tbar);
    tma_load_5d(sX, &maps.x, 0, 0, p0 / 8, (int)h, (int)b, tbar);
  }
  if (tid < kPT) {
    float dv = 0.f;
    if (a.D != nullptr) dv = a.D_per_dim ? a.D[h * a.P + p0 + tid] : a.D[h];
    sD[tid] = dv;
  }
  // S row n = tid (float32): initial state or zeros
  float S[kPT];
#pragma unroll
  for (int p = 0; p < kPT; ++p)
    S[p] = (a.init != nullptr && tid < N) ? a.init[((b * a.H + h) * a.P + p0 + p) * a.N + tid] : 0.f;
  const float A2 = a.A[h] * kLog2e;
  const float bias = a.dt_bias != nullptr ? a.dt_bias[h] : 0.f;
  const uint16_t* zbase = a.z != nullptr ? a.z + b * a.zbs + h * a.zhs + p0 : nullptr;
  const float* dtbase = a.dt + b * a.dtbs + h;

  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tbase = *tslot;
  const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);  // this warp's lanes

  constexpr uint32_t kIdG = idesc_16(kQ, kQ, 0, 0, F16);
  constexpr uint32_t kIdY = idesc_16(kQ, kPT, 0, 1, F16);
  constexpr uint32_t kIdS = idesc_16(kNP, kPT, 1, 1, F16);
  // Column-piece-major tiles: core matrices 128 bytes apart along the rows, rows * 16 bytes
  // apart along the column pieces. K-major (rows = M / N): LBO = piece stride, SBO = 128;
  // MN-major (rows = K): LBO = 128, SBO = piece stride. A K step of 16 is two pieces (K-major)
  // or two 8-row groups (MN-major).
  constexpr uint32_t kPiece = kQ * 16;     // 64-row tiles (C, B, M, X, X')
  constexpr uint32_t kPieceS = kNP * 16;   // 128-row tiles (S)
  constexpr uint32_t kColYo = kQ, kColSl = kQ + kPT;

  // Packed sequences (seq_idx): the carried state belongs to sequence seq_prev (initial states to
  // sequence 0, as upstream); a step only sees steps and carried state of its own sequence.
  const int32_t* seqbase = SEQ ? a.seq_idx + b * a.sqbs : nullptr;
  int seq_prev = 0;

  uint32_t phase = 0, tphase = 0;
  float dt_raw = (tid < kQ && tid < a.L) ? dtbase[tid * a.dtls] : 0.f;
  for (int64_t k = 0; k < nchunks; ++k) {
    const int64_t t0 = k * kQ;
    const int valid = (int)(a.L - t0 < kQ ? a.L - t0 : kQ);

    // ---- S_prev as 16-bit hi + lo (row n = tid), this chunk's z (registers), dt and its sums
    uint4 zv[kPT / 8];
    if (lo16 && zbase != nullptr && crow < valid) {
#pragma unroll
      for (int c = 0; c < kPT / 8; ++c) zv[c] = __ldg(reinterpret_cast<const uint4*>(zbase + (t0 + crow) * a.zls) + c);
    }
#pragma unroll
    for (int c = 0; c < kPT / 8; ++c) {
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float v0 = S[c * 8 + 2 * q], v1 = S[c * 8 + 2 * q + 1];
        hi[q] = pack2<F16>(v0, v1);
        const float2 hv = unpack2<F16>(hi[q]);
        lo[q] = pack2<F16>(v0 - hv.x, v1 - hv.y);
      }
      const uint32_t off = core16(tid, c, kNP);
      *reinterpret_cast<uint4*>(smem + kOffSh + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(smem + kOffSl + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    if ((nc8 & 1) && nc8 < 8 && tid < kQ)  // C columns [dstate, dstate + 8) of the last K step (M overwrote them)
      *reinterpret_cast<uint4*>(smem + core16(tid, nc8)) = make_uint4(0, 0, 0, 0);
    if (tid < kQ) {  // warps 0 and 1: dt (softplus, clamp) and the cumulative sum of dt A
      float dtv = 0.f;
      if (tid < valid) {
        float raw = dt_raw + bias;
        if (a.softplus) raw = softplus_f(raw);
        dtv = fminf(fmaxf(raw, a.dt_min), a.dt_max);
      }
      sdt[tid] = dtv;
      if constexpr (SEQ) sseq[tid] = tid < valid ? seqbase[(t0 + tid) * a.sqls] : -1;
      float v = dtv * A2;  // log2 units
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (lane == 31) swarp[warp] = v;
      scs[tid] = v;  // warp-inclusive; warp 1 adds warp 0's total below
      dt_raw = (t0 + kQ + tid < a.L) ? dtbase[(t0 + kQ + tid) * a.dtls] : 0.f;  // the next chunk's
    }
    __syncthreads();
    if (tid >= 32 && tid < kQ) scs[tid] += swarp[0];
    mbar_wait_spin(tbar, tphase);  // this chunk's tiles have landed
    tphase ^= 1;
    fence_proxy_async();
    tmem_fence_before_sync();
    __syncthreads();
    const float cs_end = scs[kQ - 1];
    const float cs = scs[crow];
    const int seq_i = SEQ ? sseq[crow] : 0, seq_last = SEQ ? sseq[valid - 1] : 0;

    // ---- G = C B^T and Yo = C S^T (hi, then lo)
    if (tid == 0) {
      tmem_fence_after_sync();
      for (int s = 0; s < ksteps; ++s)
        umma_16(tbase, sdesc(sCM + s * 2 * kPiece, kPiece, 128), sdesc(sB + s * 2 * kPiece, kPiece, 128), kIdG,
                  s > 0);
      for (int s = 0; s < ksteps; ++s)
        umma_16(tbase + kColYo, sdesc(sCM + s * 2 * kPiece, kPiece, 128), sdesc(sSh + s * 256, 128, kPieceS), kIdY,
                  s > 0);
      for (int s = 0; s < ksteps; ++s)
        umma_16(tbase + kColYo, sdesc(sCM + s * 2 * kPiece, kPiece, 128), sdesc(sSl + s * 256, 128, kPieceS), kIdY,
                  1);
      umma_commit(bar);
    }
    mbar_wait_spin(bar, phase);
    phase ^= 1;
    tmem_fence_after_sync();

    // ---- lanes < 16: M = G o L (row i = crow) over C's tile; lanes >= 16: X' = w X (row crow)
    uint4 xv[kPT / 8];  // lanes < 16: this row's x, kept for the output stage
    {
      const int i = crow;
#pragma unroll 1
      for (int q = 0; q < kQ / 16; ++q) {
        uint4 w0 = make_uint4(0, 0, 0, 0), w1 = make_uint4(0, 0, 0, 0);
        if (q <= warp) {  // warp-uniform: rows 16 warp .. + 15 reach column 16 q
          float gv[16];
          tmem_ld16(trow + q * 16, gv);
          tmem_wait_ld();
          uint32_t pk[8];
#pragma unroll
          for (int jj = 0; jj < 16; jj += 4) {
            const int j = q * 16 + jj;
            const float4 cj = *reinterpret_cast<const float4*>(&scs[j]);
            const float4 dj = *reinterpret_cast<const float4*>(&sdt[j]);
            const int4 sj = SEQ ? *reinterpret_cast<const int4*>(&sseq[j]) : make_int4(0, 0, 0, 0);
            const float m0 = (j <= i && sj.x == seq_i) ? gv[jj] * ex2(cs - cj.x) * dj.x : 0.f;
            const float m1 = (j + 1 <= i && sj.y == seq_i) ? gv[jj + 1] * ex2(cs - cj.y) * dj.y : 0.f;
            const float m2 = (j + 2 <= i && sj.z == seq_i) ? gv[jj + 2] * ex2(cs - cj.z) * dj.z : 0.f;
            const float m3 = (j + 3 <= i && sj.w == seq_i) ? gv[jj + 3] * ex2(cs - cj.w) * dj.w : 0.f;
            pk[jj / 2] = pack2<F16>(m0, m1);
            pk[jj / 2 + 1] = pack2<F16>(m2, m3);
          }
          w0 = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          w1 = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
        if (lo16) {
          *reinterpret_cast<uint4*>(smem + core16(i, 2 * q)) = w0;
          *reinterpret_cast<uint4*>(smem + core16(i, 2 * q + 1)) = w1;
        }
      }
      // X' rows of the chunk's last sequence only: earlier sequences end inside the chunk
      const float wx = seq_i == seq_last ? ex2(cs_end - cs) * sdt[i] : 0.f;
#pragma unroll
      for (int c = 0; c < kPT / 8; ++c) {
        const uint32_t off = core16(i, c);
        xv[c] = *reinterpret_cast<const uint4*>(smem + kOffX + off);
        if (!lo16) {
          const uint32_t in[4] = {xv[c].x, xv[c].y, xv[c].z, xv[c].w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = unpack2<F16>(in[e]);
            o[e] = pack2<F16>(f.x * wx, f.y * wx);
          }
          *reinterpret_cast<uint4*>(smem + kOffXs + off) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
    fence_proxy_async();
    tmem_fence_before_sync();
    __syncthreads();

    // ---- Yd = M X (into G's columns) and Sl = X'^T B; then the next chunk's tile copies
    if (tid == 0) {
      tmem_fence_after_sync();
      for (int s = 0; s < kQ / 16; ++s)
        umma_16(tbase, sdesc(sCM + s * 2 * kPiece, kPiece, 128), sdesc(sX + s * 256, 128, kPiece), kIdY, s > 0);
      for (int s = 0; s < kQ / 16; ++s)
        umma_16(tbase + kColSl, sdesc(sB + s * 256, 128, kPiece), sdesc(sXs + s * 256, 128, kPiece), kIdS, s > 0);
      umma_commit(bar);
    }
    mbar_wait_spin(bar, phase);
    phase ^= 1;
    tmem_fence_after_sync();
    if (tid == 0 && k + 1 < nchunks) {
      const int tn = (int)(t0 + kQ);
      mbar_arrive_expect_tx(tbar, tile_bytes);
      tma_load_5d(sCM, &maps.C, 0, tn, 0, (int)g, (int)b, tbar);
      tma_load_5d(sB, &maps.B, 0, tn, 0, (int)g, (int)b, tbar);
      tma_load_5d(sX, &maps.x, 0, tn, p0 / 8, (int)h, (int)b, tbar);
    }

    // ---- outputs of row crow (lanes < 16), in two halves of 16 columns
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float yo[16], yd[16];
      tmem_ld16(trow + kColYo + 16 * hf, yo);
      tmem_ld16(trow + 16 * hf, yd);
      tmem_wait_ld();
      if (lo16 && crow < valid) {
        const float eo = seq_i == seq_prev ? ex2(cs) : 0.f;  // the carried state, if it is this row's sequence
        const int64_t t = t0 + crow;
        uint16_t* orow = a.out + ((b * a.L + t) * a.H + h) * a.P + p0 + 16 * hf;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint4 xq = xv[2 * hf + c];
          const uint32_t xin[4] = {xq.x, xq.y, xq.z, xq.w};
          uint32_t zin[4] = {0, 0, 0, 0};
          if (zbase != nullptr) {
            const uint4 zq = zv[2 * hf + c];
            zin[0] = zq.x, zin[1] = zq.y, zin[2] = zq.z, zin[3] = zq.w;
          }
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int p = c * 8 + 2 * e;
            const float2 xf = unpack2<F16>(xin[e]);
            float y0 = fmaf(eo, yo[p], yd[p]) + sD[16 * hf + p] * xf.x;
            float y1 = fmaf(eo, yo[p + 1], yd[p + 1]) + sD[16 * hf + p + 1] * xf.y;
            if (zbase != nullptr) {
              const float2 zf = unpack2<F16>(zin[e]);
              y0 *= silu_f(zf.x);
              y1 *= silu_f(zf.y);
            }
            o[e] = pack2<F16>(y0, y1);
          }
          *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
    // ---- the carried state (row n = tid)
    {
      const float decay = seq_last == seq_prev ? ex2(cs_end) : 0.f;  // a new sequence starts from zero
      float sl[16];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        tmem_ld16(trow + kColSl + 16 * hf, sl);
        tmem_wait_ld();
#pragma unroll
        for (int p = 0; p < 16; ++p) S[16 * hf + p] = fmaf(decay, S[16 * hf + p], sl[p]);
      }
    }
    seq_prev = seq_last;
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

// cuTensorMapEncodeTiled from the driver (through the runtime, no libcuda link).
// Looked up once per process (a function-local static: thread-safe initialisation).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    return nullptr;
  }();
  return fn;
}

// Tensor map of a bf16 / fp16 tensor seen as (8 elements, seqlen, pieces of 8 columns, group or head,
// batch) with element strides (1, s_l, 8, s_g, s_b); box (8, 128, box_pieces, 1, 1).
bool encode_map(CUtensorMap* m, const void* base, int64_t L, int64_t pieces, int64_t ng, int64_t nb, int64_t s_l,
                int64_t s_g, int64_t s_b, int box_pieces, bool f16) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[5] = {8, (cuuint64_t)L, (cuuint64_t)pieces, (cuuint64_t)ng, (cuuint64_t)nb};
  const cuuint64_t strides[4] = {(cuuint64_t)s_l * 2, 16, (cuuint64_t)s_g * 2, (cuuint64_t)s_b * 2};
  const cuuint32_t box[5] = {8, (cuuint32_t)kQ, (cuuint32_t)box_pieces, 1, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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
  if (p->x_dtype != MB200_BF16 && p->x_dtype != MB200_F16)
    return p->x_dtype == MB200_F32 ? MB200_ERR_UNSUPPORTED : MB200_ERR_BAD_DTYPE;
  const bool f16 = p->x_dtype == MB200_F16;
  if (p->dstate % 8 != 0 || p->dstate > kNP || p->headdim % kPT != 0 || p->headdim > 256 || p->seqlen > 0x7fffffff)
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
  a.x = static_cast<const uint16_t*>(p->x);
  a.dt = p->dt;
  a.A = p->A;
  a.B = static_cast<const uint16_t*>(p->B);
  a.C = static_cast<const uint16_t*>(p->C);
  a.D = p->D;
  a.z = static_cast<const uint16_t*>(p->z);
  a.dt_bias = p->dt_bias;
  a.init = p->initial_states;
  a.out = static_cast<uint16_t*>(p->out);
  a.final_states = p->final_states;
  a.L = p->seqlen, a.H = p->nheads, a.P = p->headdim, a.G = p->ngroups, a.N = p->dstate;
  a.xbs = p->x_batch_stride, a.xls = p->x_seqlen_stride, a.xhs = p->x_head_stride;
  a.zbs = p->z_batch_stride, a.zls = p->z_seqlen_stride, a.zhs = p->z_head_stride;
  a.Bbs = p->B_batch_stride, a.Bls = p->B_seqlen_stride, a.Bgs = p->B_group_stride;
  a.Cbs = p->C_batch_stride, a.Cls = p->C_seqlen_stride, a.Cgs = p->C_group_stride;
  a.dtbs = p->dt_batch_stride, a.dtls = p->dt_seqlen_stride;
  a.seq_idx = p->seq_idx, a.sqbs = p->seq_idx_batch_stride, a.sqls = p->seq_idx_seqlen_stride;
  a.dt_min = p->dt_min, a.dt_max = p->dt_max;
  a.softplus = p->dt_softplus != 0;
  a.D_per_dim = p->D_per_dim != 0;
  a.ntiles = (int)ntiles;
  SsdMaps maps;
  const int64_t L = p->seqlen > 0 ? p->seqlen : 1;
  if (!encode_map(&maps.B, p->B, L, p->dstate / 8, p->ngroups, p->batch, p->B_seqlen_stride, p->B_group_stride,
                  p->B_batch_stride, (int)(p->dstate / 8), f16) ||
      !encode_map(&maps.C, p->C, L, p->dstate / 8, p->ngroups, p->batch, p->C_seqlen_stride, p->C_group_stride,
                  p->C_batch_stride, (int)(p->dstate / 8), f16) ||
      !encode_map(&maps.x, p->x, L, p->headdim / 8, p->nheads, p->batch, p->x_seqlen_stride, p->x_head_stride,
                  p->x_batch_stride, kPT / 8, f16))
    return MB200_ERR_CUDA;
  const bool seq = p->seq_idx != nullptr;
  const auto kern = f16 ? (seq ? ssd_fwd_kernel<true, true> : ssd_fwd_kernel<false, true>)
                        : (seq ? ssd_fwd_kernel<true, false> : ssd_fwd_kernel<false, false>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSsdSmem);
  if (e != cudaSuccess) return MB200_ERR_CUDA;
  kern<<<(unsigned)ctas, kSsdThreads, kSsdSmem, static_cast<cudaStream_t>(stream)>>>(a, maps);
  if (cudaGetLastError() != cudaSuccess) return MB200_ERR_CUDA;
  note_launches(1);
  return MB200_OK;
}

}  // extern "C"
