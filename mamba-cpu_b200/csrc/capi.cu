// capi.cu -- extern "C" entry points of libmamba_b200.so (declared in include/mamba_b200.h).
//
// Each entry point validates its arguments on the host, derives the kernel argument block and
// enqueues the kernels on the caller's stream. Nothing is enqueued when validation fails.
#include <cuda_runtime.h>

#include "conv1d.cuh"
#include "decode.cuh"
#include "scan.cuh"

namespace mb200 {

static thread_local int g_launches = 0;
void note_launches(int n) { g_launches += n; }
void reset_launches() { g_launches = 0; }

namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool io_dtype_ok(int t) { return t == MB200_F32 || t == MB200_BF16 || t == MB200_F16; }

bool bc_dtype_ok(int io, int bc) { return bc == MB200_F32 || bc == io; }

// Shared validation of the forward parameter block; fills the kernel view.
int build_scan_args(const mb200_scan_fwd_params* p, bool need_out, ScanArgs* a) {
  if (p == nullptr) return MB200_ERR_NULL_POINTER;
  if (p->batch < 0 || p->dim < 0 || p->seqlen < 0 || p->dstate < 1 || p->ngroups < 1)
    return MB200_ERR_BAD_SHAPE;
  if (p->dim % p->ngroups != 0) return MB200_ERR_BAD_SHAPE;
  if (p->dstate > MB200_MAX_DSTATE) return MB200_ERR_UNSUPPORTED;
  if (!io_dtype_ok(p->io_dtype) || !bc_dtype_ok(p->io_dtype, p->bc_dtype)) return MB200_ERR_BAD_DTYPE;
  const bool empty = p->batch == 0 || p->dim == 0;
  if (!empty && (p->u == nullptr || p->delta == nullptr || p->A == nullptr || p->B == nullptr ||
                 p->C == nullptr || (need_out && p->out == nullptr)))
    return MB200_ERR_NULL_POINTER;
  const int es = dtype_size(p->io_dtype);
  const int bs = dtype_size(p->bc_dtype);
  a->u = p->u;
  a->delta = p->delta;
  a->A = p->A;
  a->B = p->B;
  a->C = p->C;
  a->D = p->D;
  a->z = p->z;
  a->delta_bias = p->delta_bias;
  a->out = p->out;
  a->last_state = p->last_state;
  a->chunk_states = p->chunk_states;
  a->h_init = p->initial_state;
  a->batch = p->batch;
  a->dim = p->dim;
  a->L = p->seqlen;
  a->N = p->dstate;
  a->ngroups = p->ngroups;
  a->dpg = p->dim / p->ngroups;
  a->sBb = p->B_batch_stride;
  a->sBg = p->B_group_stride;
  a->sBn = p->B_dstate_stride;
  a->sBl = p->B_seqlen_stride;
  a->sCb = p->C_batch_stride;
  a->sCg = p->C_group_stride;
  a->sCn = p->C_dstate_stride;
  a->sCl = p->C_seqlen_stride;
  a->tiles = 0;
  a->nchunks = (int)((p->seqlen + kChunk - 1) / kChunk);
  a->pieces = 1;
  a->piece_chunks = a->nchunks;
  a->piece_e = nullptr;
  a->piece_scratch = nullptr;
  a->piece_P = nullptr;
  a->softplus = p->delta_softplus != 0;
  const int64_t dense_b = p->dim * p->seqlen, dense_d = p->seqlen;
  auto pick = [](int64_t s, int64_t dense) { return s != 0 ? s : dense; };
  a->sub = pick(p->u_batch_stride, dense_b);
  a->sud = pick(p->u_dim_stride, dense_d);
  a->sdb = pick(p->delta_batch_stride, dense_b);
  a->sdd = pick(p->delta_dim_stride, dense_d);
  a->szb = pick(p->z_batch_stride, dense_b);
  a->szd = pick(p->z_dim_stride, dense_d);
  const int64_t io_strides[6] = {a->sub, a->sud, a->sdb, a->sdd, a->szb, a->szd};
  bool io_rows16 = true;
  for (int64_t v : io_strides) {
    if (v < 0) return MB200_ERR_BAD_LAYOUT;
    io_rows16 = io_rows16 && (v * es) % 16 == 0;
  }
  const bool io_al = aligned16(p->u) && aligned16(p->delta) && aligned16(p->z) && aligned16(p->out);
  a->vec_io = io_al && io_rows16 && ((p->seqlen * es) % 16 == 0);
  const bool bc_al = aligned16(p->B) && aligned16(p->C);
  auto row16 = [&](int64_t s) { return (s * bs) % 16 == 0; };
  a->vec_bc = bc_al && p->B_seqlen_stride == 1 && p->C_seqlen_stride == 1 && row16(p->B_batch_stride) &&
              row16(p->B_group_stride) && row16(p->B_dstate_stride) && row16(p->C_batch_stride) &&
              row16(p->C_group_stride) && row16(p->C_dstate_stride);
  return MB200_OK;
}

// Sequence pieces for a grid whose whole rows give `ctas` CTAs: (pieces, chunks per piece), with
// no empty piece.
void piece_split(int64_t ctas, int nchunks, bool backward, int* pieces, int* piece_chunks) {
  int G = nchunks > 1 ? seq_pieces(ctas, nchunks, backward) : 1;
  int pc = G > 1 ? (nchunks + G - 1) / G : nchunks;
  if (G > 1) G = (nchunks + pc - 1) / pc;
  *pieces = G;
  *piece_chunks = pc;
}

struct FwdLayout {
  size_t e, P, scratch, total;
  int pieces, piece_chunks;
};

FwdLayout fwd_layout(const ScanArgs& a) {
  FwdLayout w = {};
  w.pieces = 1;
  w.piece_chunks = a.nchunks;
  // Short rows of small problems (the one-state-per-lane layout) stay whole unless a count is
  // forced: there the summary pass's own chain is as long as the pieces it would save (BASELINE
  // config 1, b=1 d=1536 l=2048: 71.7 us whole, 93.2 us in the 2 pieces the cost model picks).
  const bool short_rows = fwd_states_per_lane(a.batch * a.dim, a.nchunks) == 1;
  if (a.batch > 0 && a.dim > 0 && (!short_rows || forced_pieces() > 0))
    piece_split(fwd_ctas(a), a.nchunks, false, &w.pieces, &w.piece_chunks);
  const size_t per = sizeof(float) * (size_t)(w.pieces - 1) * a.batch * a.dim * a.N;
  ScanArgs t = a;
  t.pieces = w.pieces;
  t.piece_chunks = w.piece_chunks;
  size_t off = 0;
  w.e = off;
  off = align_up(off + per, 256);
  w.P = off;
  off = align_up(off + per, 256);
  w.scratch = off;
  off = align_up(off + sizeof(float) * summary_scratch_floats(t), 256);
  w.total = w.pieces > 1 ? off : 0;
  return w;
}

struct BwdLayout {
  size_t states, part_bc, part_A, part_D, part_db, piece_G, piece_P, scratch, total;
  int cluster, pieces, piece_chunks;
  int64_t clusters, Lpad;
};

BwdLayout bwd_layout(const ScanArgs& f, bool need_states, bool batch_partials) {
  BwdLayout w = {};
  const int S = bwd_segments(f.batch * f.dim, f.nchunks);
  const int64_t cpc = kBwdWarps * (32 / S);
  const int64_t tiles = (f.dpg + cpc - 1) / cpc;
  const int64_t slices = f.batch * f.ngroups;
  // batch_partials writes the caller's per-batch partial buffers directly: whole rows only
  w.pieces = 1;
  w.piece_chunks = f.nchunks;
  if (!batch_partials && f.batch > 0 && f.dim > 0)
    piece_split(tiles * slices, f.nchunks, true, &w.pieces, &w.piece_chunks);
  w.cluster = bwd_cluster_size(tiles, slices * w.pieces);
  w.clusters = (tiles + w.cluster - 1) / w.cluster;
  w.Lpad = (int64_t)f.nchunks * kChunk;
  const int64_t rows = f.batch * f.dim;
  const int64_t G = w.pieces;
  size_t off = 0;
  w.states = off;
  if (need_states) off = align_up(off + sizeof(float) * rows * f.nchunks * f.N, 256);
  w.part_bc = off;
  off = align_up(off + sizeof(float) * slices * w.clusters * 2 * f.N * w.Lpad, 256);
  w.part_A = off;
  if (!batch_partials) off = align_up(off + sizeof(float) * G * rows * f.N, 256);
  w.part_D = off;
  if (!batch_partials) off = align_up(off + sizeof(float) * G * rows, 256);
  w.part_db = off;
  if (!batch_partials) off = align_up(off + sizeof(float) * G * rows, 256);
  w.piece_G = off;
  if (G > 1) off = align_up(off + sizeof(float) * G * rows * f.N, 256);
  w.piece_P = off;
  if (G > 1) off = align_up(off + sizeof(float) * G * rows * f.N, 256);
  ScanArgs t = f;
  t.pieces = w.pieces;
  t.piece_chunks = w.piece_chunks;
  w.scratch = off;
  if (G > 1) off = align_up(off + sizeof(float) * summary_scratch_floats(t), 256);
  w.total = off;
  return w;
}

int run_fwd(const mb200_scan_fwd_params* p, ScanArgs a, const FwdLayout& w, char* ws, cudaStream_t stream) {
  a.pieces = w.pieces;
  a.piece_chunks = w.piece_chunks;
  if (w.pieces > 1) {
    a.piece_e = reinterpret_cast<float*>(ws + w.e);
    a.piece_P = reinterpret_cast<float*>(ws + w.P);
    a.piece_scratch = reinterpret_cast<float*>(ws + w.scratch);
  }
  if (launch_scan_fwd(a, p->io_dtype, p->bc_dtype, true, stream) != cudaSuccess) return MB200_ERR_CUDA;
  if (a.batch > 0 && a.dim > 0) note_launches(w.pieces > 1 ? 2 : 1);
  return MB200_OK;
}

int check_bwd(const mb200_scan_bwd_params* p, ScanArgs* f) {
  if (p == nullptr) return MB200_ERR_NULL_POINTER;
  int st = build_scan_args(&p->fwd, false, f);
  if (st != MB200_OK) return st;
  if (p->dbc_dtype != MB200_F32 && p->dbc_dtype != p->fwd.bc_dtype) return MB200_ERR_BAD_DTYPE;
  const bool empty = f->batch == 0 || f->dim == 0;
  if (!empty && (p->dout == nullptr || p->du == nullptr || p->ddelta == nullptr || p->dB == nullptr ||
                 p->dC == nullptr || (p->fwd.z != nullptr && p->dz == nullptr)))
    return MB200_ERR_NULL_POINTER;
  if (f->dim > 0 && p->dA == nullptr) return MB200_ERR_NULL_POINTER;
  const bool io_al = aligned16(p->dout) && aligned16(p->du) && aligned16(p->ddelta) && aligned16(p->dz);
  if (!io_al) f->vec_io = 0;
  return MB200_OK;
}

int run_bwd(const mb200_scan_bwd_params* p, ScanArgs f, char* ws, const BwdLayout& w, bool batch_partials,
            float* pA, float* pD, float* pdb, int64_t osb, int64_t osg, int64_t osn, int64_t osl,
            cudaStream_t stream) {
  BwdArgs a = {};
  a.f = f;
  a.dout = p->dout;
  a.dlast = p->dlast_state;
  a.du = p->du;
  a.ddelta = p->ddelta;
  a.dz = p->dz;
  a.dh_init = p->dinitial_state;
  a.part_bc = reinterpret_cast<float*>(ws + w.part_bc);
  a.part_A = batch_partials ? pA : reinterpret_cast<float*>(ws + w.part_A);
  a.part_D = batch_partials ? pD : reinterpret_cast<float*>(ws + w.part_D);
  a.part_db = batch_partials ? pdb : reinterpret_cast<float*>(ws + w.part_db);
  a.Lpad = w.Lpad;
  a.clusters = (int)w.clusters;
  a.f.pieces = w.pieces;
  a.f.piece_chunks = w.piece_chunks;
  if (w.pieces > 1) {
    a.piece_G = reinterpret_cast<float*>(ws + w.piece_G);
    a.piece_P = reinterpret_cast<float*>(ws + w.piece_P);
    a.f.piece_scratch = reinterpret_cast<float*>(ws + w.scratch);
  }
  int launches = 0;
  if (p->fwd.chunk_states != nullptr) {
    a.states = p->fwd.chunk_states;
  } else {
    // Restart states are not available: run the forward recurrence once without outputs.
    ScanArgs s = f;
    s.out = nullptr;
    s.last_state = nullptr;
    s.chunk_states = reinterpret_cast<float*>(ws + w.states);
    a.states = s.chunk_states;
    if (f.batch > 0 && f.dim > 0 && f.nchunks > 1) {
      if (launch_scan_fwd(s, p->fwd.io_dtype, p->fwd.bc_dtype, false, stream) != cudaSuccess)
        return MB200_ERR_CUDA;
      ++launches;
    }
  }
  a.f.out = nullptr;
  a.f.last_state = nullptr;
  a.f.chunk_states = nullptr;
  if (f.batch > 0 && f.dim > 0) {
    if (w.pieces > 1) {
      if (launch_bwd_piece_summary(a, p->fwd.io_dtype, p->fwd.bc_dtype, stream) != cudaSuccess) return MB200_ERR_CUDA;
      ++launches;
    }
    if (launch_scan_bwd(a, p->fwd.io_dtype, p->fwd.bc_dtype, w.cluster, stream) != cudaSuccess)
      return MB200_ERR_CUDA;
    ++launches;
  }
  if (launch_scan_bwd_reduce_strided(a, p->dB, p->dC, p->dbc_dtype, osb, osg, osn, osl, p->dA, p->dD,
                                     p->ddelta_bias, batch_partials, stream) != cudaSuccess)
    return MB200_ERR_CUDA;
  ++launches;
  note_launches(launches);
  return MB200_OK;
}

}  // namespace

}  // namespace mb200

using namespace mb200;

extern "C" {

MB200_API size_t mb200_selective_scan_fwd_workspace_size(const mb200_scan_fwd_params* p) {
  ScanArgs a;
  if (build_scan_args(p, true, &a) != MB200_OK) return 0;
  return fwd_layout(a).total;
}

MB200_API int mb200_selective_scan_fwd_ws(const mb200_scan_fwd_params* p, void* workspace, size_t workspace_bytes,
                                          void* stream) {
  reset_launches();
  ScanArgs a;
  int st = build_scan_args(p, true, &a);
  if (st != MB200_OK) return st;
  const FwdLayout w = fwd_layout(a);
  if (w.total > 0 && (workspace == nullptr || workspace_bytes < w.total ||
                      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0))
    return MB200_ERR_WORKSPACE;
  return run_fwd(p, a, w, static_cast<char*>(workspace), static_cast<cudaStream_t>(stream));
}

MB200_API int mb200_selective_scan_fwd(const mb200_scan_fwd_params* p, void* stream) {
  reset_launches();
  ScanArgs a;
  int st = build_scan_args(p, true, &a);
  if (st != MB200_OK) return st;
  // the sequence-piece summaries (small grids only) live in a stream-ordered allocation
  const FwdLayout w = fwd_layout(a);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* ws = nullptr;
  if (w.total > 0 && cudaMallocAsync(&ws, w.total, s) != cudaSuccess) return MB200_ERR_CUDA;
  st = run_fwd(p, a, w, static_cast<char*>(ws), s);
  if (ws != nullptr && cudaFreeAsync(ws, s) != cudaSuccess && st == MB200_OK) st = MB200_ERR_CUDA;
  return st;
}

MB200_API void mb200_set_sequence_pieces(int pieces) { set_forced_pieces(pieces); }

MB200_API int mb200_sequence_pieces(int64_t ctas, int nchunks, int backward) {
  return seq_pieces(ctas, nchunks, backward != 0);
}

MB200_API size_t mb200_selective_scan_bwd_workspace_size(const mb200_scan_bwd_params* p) {
  ScanArgs f;
  if (check_bwd(p, &f) != MB200_OK) return 0;
  return bwd_layout(f, p->fwd.chunk_states == nullptr, false).total;
}

MB200_API int mb200_selective_scan_bwd(const mb200_scan_bwd_params* p, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  reset_launches();
  ScanArgs f;
  int st = check_bwd(p, &f);
  if (st != MB200_OK) return st;
  const BwdLayout w = bwd_layout(f, p->fwd.chunk_states == nullptr, false);
  if (w.total > 0 && (workspace == nullptr || workspace_bytes < w.total ||
                      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0))
    return MB200_ERR_WORKSPACE;
  const int64_t N = f.N, L = f.L;
  return run_bwd(p, f, static_cast<char*>(workspace), w, false, nullptr, nullptr, nullptr,
                 f.ngroups * N * L, N * L, L, 1, static_cast<cudaStream_t>(stream));
}

MB200_API int mb200_selective_scan_fwd_f32(const float* u, const float* delta, const float* A,
                                           const float* B, const float* C, const float* D,
                                           const float* z, const float* delta_bias, float* out,
                                           float* last_state, int64_t batch, int64_t dim,
                                           int64_t seqlen, int64_t dstate, int64_t ngroups,
                                           int delta_softplus, void* stream) {
  mb200_scan_fwd_params p = {};
  p.u = u;
  p.delta = delta;
  p.A = A;
  p.B = B;
  p.C = C;
  p.D = D;
  p.z = z;
  p.delta_bias = delta_bias;
  p.out = out;
  p.last_state = last_state;
  p.chunk_states = nullptr;
  p.batch = batch;
  p.dim = dim;
  p.seqlen = seqlen;
  p.dstate = dstate;
  p.ngroups = ngroups;
  // (batch, ngroups, seqlen, dstate): selective_scan.h:17
  p.B_batch_stride = p.C_batch_stride = ngroups * seqlen * dstate;
  p.B_group_stride = p.C_group_stride = seqlen * dstate;
  p.B_dstate_stride = p.C_dstate_stride = 1;
  p.B_seqlen_stride = p.C_seqlen_stride = dstate;
  p.io_dtype = MB200_F32;
  p.bc_dtype = MB200_F32;
  p.delta_softplus = delta_softplus;
  return mb200_selective_scan_fwd(&p, stream);
}

MB200_API int mb200_selective_scan_bwd_f32(
    const float* u, const float* delta, const float* A, const float* B, const float* C,
    const float* D, const float* z, const float* delta_bias, const float* dout,
    const float* dlast_state, float* du, float* ddelta, float* dA_part, float* dB, float* dC,
    float* dD_part, float* dz, float* ddelta_bias_part, int64_t batch, int64_t dim,
    int64_t seqlen, int64_t dstate, int64_t ngroups, int delta_softplus, void* stream) {
  reset_launches();
  mb200_scan_bwd_params p = {};
  p.fwd.u = u;
  p.fwd.delta = delta;
  p.fwd.A = A;
  p.fwd.B = B;
  p.fwd.C = C;
  p.fwd.D = D;
  p.fwd.z = z;
  p.fwd.delta_bias = delta_bias;
  p.fwd.batch = batch;
  p.fwd.dim = dim;
  p.fwd.seqlen = seqlen;
  p.fwd.dstate = dstate;
  p.fwd.ngroups = ngroups;
  p.fwd.B_batch_stride = p.fwd.C_batch_stride = ngroups * seqlen * dstate;
  p.fwd.B_group_stride = p.fwd.C_group_stride = seqlen * dstate;
  p.fwd.B_dstate_stride = p.fwd.C_dstate_stride = 1;
  p.fwd.B_seqlen_stride = p.fwd.C_seqlen_stride = dstate;
  p.fwd.io_dtype = MB200_F32;
  p.fwd.bc_dtype = MB200_F32;
  p.fwd.delta_softplus = delta_softplus;
  p.dout = dout;
  p.dlast_state = dlast_state;
  p.du = du;
  p.ddelta = ddelta;
  p.dz = dz;
  p.dA = dA_part;  // only checked for non-NULL; the partials go straight to the caller's buffers
  p.dB = dB;
  p.dC = dC;
  p.dD = dD_part;
  p.ddelta_bias = ddelta_bias_part;
  p.dbc_dtype = MB200_F32;
  ScanArgs f;
  int st = check_bwd(&p, &f);
  if (st != MB200_OK) return st;
  if (f.batch > 0 && f.dim > 0 && (dD_part == nullptr || ddelta_bias_part == nullptr))
    return MB200_ERR_NULL_POINTER;
  const BwdLayout w = bwd_layout(f, true, true);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* ws = nullptr;
  if (w.total > 0 && cudaMallocAsync(&ws, w.total, s) != cudaSuccess) return MB200_ERR_CUDA;
  st = run_bwd(&p, f, static_cast<char*>(ws), w, true, dA_part, dD_part, ddelta_bias_part,
               ngroups * seqlen * dstate, seqlen * dstate, 1, dstate, s);
  if (ws != nullptr && cudaFreeAsync(ws, s) != cudaSuccess && st == MB200_OK) st = MB200_ERR_CUDA;
  return st;
}

}  // extern "C"

namespace {

int build_conv_args(const mb200_conv1d_params* p, bool need_out, ConvArgs* a) {
  if (p == nullptr) return MB200_ERR_NULL_POINTER;
  if (p->batch < 0 || p->dim < 0 || p->seqlen < 0 || p->width < 1) return MB200_ERR_BAD_SHAPE;
  if (p->width > kConvMaxWidth) return MB200_ERR_UNSUPPORTED;
  if (!io_dtype_ok(p->x_dtype)) return MB200_ERR_BAD_DTYPE;
  if (p->activation != 0 && p->activation != 1) return MB200_ERR_BAD_SHAPE;
  const bool empty = p->batch == 0 || p->dim == 0;
  if (!empty && (p->x == nullptr || p->weight == nullptr || (need_out && p->out == nullptr)))
    return MB200_ERR_NULL_POINTER;
  const int64_t span = (int64_t)kConvThreads * (kConvRowBytes / dtype_size(p->x_dtype));
  a->x = p->x;
  a->w = p->weight;
  a->bias = p->bias;
  a->init = p->initial_states;
  a->out = p->out;
  a->final_states = p->final_states;
  a->batch = p->batch;
  a->dim = p->dim;
  a->L = p->seqlen;
  a->width = p->width;
  a->silu = p->activation;
  a->vec = aligned16(p->x) && aligned16(p->out) && (p->seqlen * dtype_size(p->x_dtype)) % 16 == 0;
  a->blocks_per_row = p->seqlen > 0 ? (p->seqlen + span - 1) / span : 1;
  return MB200_OK;
}

}  // namespace

extern "C" {

MB200_API int mb200_causal_conv1d_fwd(const mb200_conv1d_params* p, void* stream) {
  reset_launches();
  ConvArgs a;
  int st = build_conv_args(p, true, &a);
  if (st != MB200_OK) return st;
  if (launch_conv_fwd(a, p->x_dtype, static_cast<cudaStream_t>(stream)) != cudaSuccess) return MB200_ERR_CUDA;
  if (a.batch > 0 && a.dim > 0) note_launches(1);
  return MB200_OK;
}

MB200_API size_t mb200_causal_conv1d_bwd_workspace_size(const mb200_conv1d_params* p) {
  ConvArgs a;
  if (build_conv_args(p, false, &a) != MB200_OK) return 0;
  return align_up(sizeof(float) * (size_t)conv_bwd_partials(a) * (size_t)(a.width + 1), 256);
}

MB200_API int mb200_causal_conv1d_bwd(const mb200_conv1d_params* p, const void* dout, void* dx,
                                      float* dweight, float* dbias, void* dinitial_states,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  reset_launches();
  if (p == nullptr) return MB200_ERR_NULL_POINTER;
  ConvArgs a;
  int st = build_conv_args(p, false, &a);
  if (st != MB200_OK) return st;
  const bool empty = a.batch == 0 || a.dim == 0;
  if (!empty && (dout == nullptr || dx == nullptr)) return MB200_ERR_NULL_POINTER;
  if (a.dim > 0 && dweight == nullptr) return MB200_ERR_NULL_POINTER;
  const size_t need = mb200_causal_conv1d_bwd_workspace_size(p);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need ||
                   (reinterpret_cast<uintptr_t>(workspace) & 255) != 0))
    return MB200_ERR_WORKSPACE;
  a.vec = a.vec && aligned16(dout) && aligned16(dx);
  if (launch_conv_bwd(a, p->x_dtype, dout, dx, dweight, dbias, dinitial_states,
                      static_cast<float*>(workspace), static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return MB200_ERR_CUDA;
  note_launches(empty ? (a.dim > 0 ? 1 : 0) : 2);
  return MB200_OK;
}

MB200_API int mb200_selective_state_update(const mb200_state_update_params* p, void* stream) {
  reset_launches();
  if (p == nullptr) return MB200_ERR_NULL_POINTER;
  if (p->batch < 0 || p->dim < 0 || p->dstate < 1 || p->ngroups < 1 || (p->dim % p->ngroups) != 0)
    return MB200_ERR_BAD_SHAPE;
  if (p->dstate > MB200_DECODE_MAX_DSTATE) return MB200_ERR_UNSUPPORTED;
  if (!io_dtype_ok(p->io_dtype) || !bc_dtype_ok(p->io_dtype, p->bc_dtype) ||
      (p->state_dtype != MB200_F32 && p->state_dtype != p->io_dtype))
    return MB200_ERR_BAD_DTYPE;
  if (p->batch > 0 && p->dim > 0 &&
      (p->state == nullptr || p->x == nullptr || p->dt == nullptr || p->A == nullptr || p->B == nullptr ||
       p->C == nullptr || p->out == nullptr))
    return MB200_ERR_NULL_POINTER;
  if (launch_state_update(*p, static_cast<cudaStream_t>(stream)) != cudaSuccess) return MB200_ERR_CUDA;
  if (p->batch > 0 && p->dim > 0) note_launches(1);
  return MB200_OK;
}

MB200_API int mb200_causal_conv1d_update(const mb200_conv1d_update_params* p, void* stream) {
  reset_launches();
  if (p == nullptr) return MB200_ERR_NULL_POINTER;
  if (p->batch < 0 || p->dim < 0 || p->seqlen < 0 || p->width < 1 || p->state_len < p->width - 1)
    return MB200_ERR_BAD_SHAPE;
  if (p->width > kConvMaxWidth) return MB200_ERR_UNSUPPORTED;
  if (!io_dtype_ok(p->x_dtype)) return MB200_ERR_BAD_DTYPE;
  if (p->batch > 0 && p->dim > 0 &&
      (p->x == nullptr || p->conv_state == nullptr || p->weight == nullptr || p->out == nullptr))
    return MB200_ERR_NULL_POINTER;
  if (launch_conv_update(*p, static_cast<cudaStream_t>(stream)) != cudaSuccess) return MB200_ERR_CUDA;
  if (p->batch > 0 && p->dim > 0) note_launches(1);
  return MB200_OK;
}

MB200_API const char* mb200_status_string(int status) {
  switch (status) {
    case MB200_OK:
      return "ok";
    case MB200_ERR_NULL_POINTER:
      return "a required pointer is NULL";
    case MB200_ERR_BAD_SHAPE:
      return "invalid shape (negative size, dstate < 1, ngroups < 1 or dim not divisible by ngroups)";
    case MB200_ERR_BAD_DTYPE:
      return "unsupported dtype code or combination";
    case MB200_ERR_BAD_LAYOUT:
      return "unsupported stride or alignment";
    case MB200_ERR_UNSUPPORTED:
      return "request outside this build's limits (e.g. dstate > 16 or conv width > 8)";
    case MB200_ERR_WORKSPACE:
      return "workspace missing, misaligned or smaller than the *_workspace_size result";
    case MB200_ERR_CUDA:
      return "a CUDA runtime call failed";
    case MB200_ERR_SCRATCH_LIMIT:
      return "request needs more scratch than the no-allocation entry point's static buffer "
             "(MB200_NOALLOC_SCRATCH_BYTES); use mb200_selective_scan_bwd with a workspace";
    default:
      return "unknown status";
  }
}

MB200_API int mb200_version(void) { return (1 << 16) | 2; }

MB200_API int mb200_last_launch_count(void) { return g_launches; }

MB200_API int mb200_device_fault(int* fault) {
  if (fault == nullptr) return MB200_ERR_NULL_POINTER;
  int f0 = 0, f1 = 0, f2 = 0, f3 = 0;
  if (read_fault_fwd(&f0) != cudaSuccess || read_fault_bwd(&f1) != cudaSuccess || read_fault_peer(&f2) != cudaSuccess ||
      read_fault_ssd(&f3) != cudaSuccess)
    return MB200_ERR_CUDA;
  *fault = f0 | f1 | f2 | f3;
  return MB200_OK;
}

}  // extern "C"
