// scan.cuh -- kernel-side argument blocks and launcher declarations of the selective scan.
#pragma once

#include "common.cuh"

namespace mb200 {

// Warps per CTA of the forward / backward scan kernels.
constexpr int kFwdWarps = 4;
constexpr int kBwdWarps = 4;

// Kernel-side view of one selective-scan call. Built and validated on the host from
// mb200_scan_fwd_params / mb200_scan_bwd_params (capi.cu).
struct ScanArgs {
  const void* u;
  const void* delta;
  const float* A;
  const void* B;
  const void* C;
  const float* D;
  const void* z;
  const float* delta_bias;
  void* out;            // forward output (io dtype), NULL in the states-only pass
  float* last_state;    // (batch, dim, dstate) or NULL
  float* chunk_states;  // (batch, dim, nchunks, dstate) or NULL
  const float* h_init;  // (batch, dim, dstate) state before the first step, or NULL (zeros)
  int64_t batch, dim, L, N, ngroups, dpg;
  int64_t sBb, sBg, sBn, sBl, sCb, sCg, sCn, sCl;
  int64_t sub, sud, sdb, sdd, szb, szd;  // batch / dim element strides of u, delta, z
  int tiles;    // CTAs per (batch, group) slice
  int nchunks;  // ceil(L / kChunk)
  int softplus;
  int vec_io;   // u / delta / z / out rows allow 16-byte vector access
  int vec_bc;   // B / C are l-contiguous and aligned
  // Sequence pieces: every row is cut into `pieces` runs of `piece_chunks` chunks, each run by its
  // own CTAs (pieces = 1: whole rows). The piece summary kernel (pieces.cu) writes the end states
  // of pieces 0 .. pieces - 2 from a zero state (piece_e) and their decays (piece_P); the forward
  // starts piece p from h_init composed through the summaries of the pieces before it.
  int pieces;
  int piece_chunks;
  float* piece_e;  // (pieces - 1, batch * dim, N)
  float* piece_P;  // (pieces - 1, batch * dim, N)
  float* piece_scratch;  // summary_scratch_floats(*this) floats for the summary kernel, or NULL
};

// True when u, delta or z are not dense (batch, dim, seqlen) rows: the launchers then pick the
// kernels' STRIDED instantiations, which address rows through the batch / dim strides. The dense
// instantiations keep the plain row * seqlen addressing (and its register allocation).
inline bool io_rows_strided(const ScanArgs& a) {
  const int64_t db = a.dim * a.L, dd = a.L;
  return a.sub != db || a.sud != dd || a.sdb != db || a.sdd != dd ||
         (a.z != nullptr && (a.szb != db || a.szd != dd));
}

struct BwdArgs {
  ScanArgs f;
  const float* states;  // chunk_states of the forward (or of the states pass)
  const void* dout;
  const float* dlast;
  void* du;
  void* ddelta;
  void* dz;
  float* dh_init;   // (batch, dim, dstate) gradient with respect to f.h_init, or NULL
  float* part_bc;   // (batch*ngroups, clusters, 2, N, Lpad) cluster partial sums of dB | dC
  float* part_A;    // (batch, dim, N)
  float* part_D;    // (batch, dim)
  float* part_db;   // (batch, dim)
  int64_t Lpad;     // nchunks * kChunk
  int clusters;     // clusters per slice = tiles / cluster size
  // Sequence pieces of the backward (f.pieces / f.piece_chunks): the piece summary kernel writes,
  // for pieces 1 .. pieces - 1, the adjoint leaving the piece at its first step when the adjoint
  // entering it at its end is zero (piece_G) and the piece's decay (piece_P); the backward kernel
  // starts piece p's carry from dlast composed through the summaries of the pieces after it.
  // part_A / part_D / part_db then hold one partial per (piece, row).
  float* piece_G;   // (pieces, batch * dim, N); piece 0 unused
  float* piece_P;   // (pieces, batch * dim, N); piece 0 unused
};

// Sequence pieces per row for a forward / backward kernel whose whole rows give `ctas` CTAs: the
// count (1 to 8, at least 4 chunks per piece) that minimises the modelled time of the summary
// pass plus the grid's rounds of resident slots (3 CTAs per SM). mb200_set_sequence_pieces
// forces a count (tests).
int seq_pieces(int64_t ctas, int nchunks, bool backward);
void set_forced_pieces(int n);  // 0: automatic
int forced_pieces();             // the count set by set_forced_pieces (0: automatic)
int sm_count();
// CTAs of the forward over whole rows (its per-CTA channel count depends on the lane layout).
int64_t fwd_ctas(const ScanArgs& a);

// States per recurrence lane of the forward (1 or 2) and segments per channel of the backward
// that the launchers pick for a call.
int fwd_states_per_lane(int64_t rows, int nchunks);
// Read and clear the device fault word of the forward / backward kernels (synchronous).
cudaError_t read_fault_fwd(int* out);
cudaError_t read_fault_bwd(int* out);
cudaError_t read_fault_peer(int* out);
cudaError_t read_fault_ssd(int* out);
int bwd_segments(int64_t rows, int nchunks);
int bwd_cluster_size(int64_t tiles, int64_t slices);

cudaError_t launch_scan_fwd(const ScanArgs& a, int io_dtype, int bc_dtype, bool write_out,
                            cudaStream_t stream);
cudaError_t launch_scan_bwd(const BwdArgs& a, int io_dtype, int bc_dtype, int cluster,
                            cudaStream_t stream);
// Piece summaries (pieces.cu; nothing to do with pieces = 1): the forward's piece_e / piece_P of
// pieces 0 .. pieces - 2, the backward's piece_G / piece_P of pieces 1 .. pieces - 1.
cudaError_t launch_fwd_piece_summary(const ScanArgs& f, int io_dtype, int bc_dtype, cudaStream_t stream);
// Run groups per piece of the summary kernel (CTAs that share a piece, composed by a second
// kernel) and the scratch floats they need (pieces and piece_chunks already set).
int summary_rgroups(const ScanArgs& f);
size_t summary_scratch_floats(const ScanArgs& f);
cudaError_t launch_bwd_piece_summary(const BwdArgs& a, int io_dtype, int bc_dtype, cudaStream_t stream);
// Sums the cluster partials of dB/dC over clusters (written with element strides osb/osg/osn/osl
// for batch/group/state/seqlen) and dA/dD/ddelta_bias over batch (skipped with batch_partials,
// when the kernel wrote the caller's per-batch partial buffers directly).
cudaError_t launch_scan_bwd_reduce_strided(const BwdArgs& a, void* dB, void* dC, int dbc_dtype,
                                           int64_t osb, int64_t osg, int64_t osn, int64_t osl,
                                           float* dA, float* dD, float* db, bool batch_partials,
                                           cudaStream_t stream);

}  // namespace mb200
