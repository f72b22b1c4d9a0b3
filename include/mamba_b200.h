/*
 * mamba_b200.h -- C ABI of the B200 (sm_100a) Mamba-1 selective-scan and causal-conv1d library
 * (libmamba_b200.so).
 *
 * This is the drop-in boundary below the Python ops. It replaces the reference's nanobind module
 * `mamba_cpu._C` (SandyTheAdventurer/mamba-cpu, csrc/bindings.cpp) and the torch-CPU conv path:
 * plain pointers and sizes, no torch types, an int status instead of exceptions, and a CUDA stream
 * argument where the reference takes a thread count (`num_threads`, bindings.cpp:35,60).
 *
 * Conventions for every entry point:
 *  - Pointers are DEVICE pointers unless stated. NULL means an absent optional input, exactly as
 *    the reference's 0-for-None uintptr convention (bindings.cpp:10-15, selective_scan.h:20).
 *  - The caller allocates every output (selective_scan_interface.py:33-34, 72-79). Entry points
 *    that need scratch take a caller-provided workspace whose size is returned by the matching
 *    *_workspace_size function; they never allocate, except the *_f32 mirrors (below), which keep
 *    the reference's signature and therefore allocate their scratch stream-ordered
 *    (cudaMallocAsync / cudaFreeAsync on the given stream) as the reference allocates its own
 *    (selective_scan.cpp:322, 341-342).
 *  - Work is enqueued on `stream` (a cudaStream_t; NULL = the legacy default stream) and the call
 *    returns without synchronising. Argument errors are detected before anything is enqueued.
 *  - Kernels never trap: a bad argument is an error status, never a device fault.
 */
#ifndef MAMBA_B200_H
#define MAMBA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MB200_API __attribute__((visibility("default")))
#else
#define MB200_API
#endif

/* ---- status codes ------------------------------------------------------------------------ */
#define MB200_OK 0
#define MB200_ERR_NULL_POINTER 1 /* a required pointer is NULL */
#define MB200_ERR_BAD_SHAPE 2    /* negative size, dim % ngroups != 0, ... */
#define MB200_ERR_BAD_DTYPE 3    /* unknown or unsupported dtype code / combination */
#define MB200_ERR_BAD_LAYOUT 4   /* stride or alignment outside what the kernel accepts */
#define MB200_ERR_UNSUPPORTED 5  /* a valid request outside this build (e.g. dstate > 16) */
#define MB200_ERR_WORKSPACE 6    /* workspace NULL or smaller than *_workspace_size */
#define MB200_ERR_CUDA 7         /* a CUDA runtime call failed (launch error, allocation) */
#define MB200_ERR_SCRATCH_LIMIT 8 /* needs more than the no-allocation entry point's static scratch */

/* ---- dtype codes ------------------------------------------------------------------------- */
#define MB200_F32 0
#define MB200_BF16 1
#define MB200_F16 2

/* Largest dstate the scan kernels accept (Mamba-1 uses 16). */
#define MB200_MAX_DSTATE 16
/* Largest dstate of the decode step (mb200_selective_state_update; Mamba-2 uses 64 / 128). */
#define MB200_DECODE_MAX_DSTATE 256
/* Timesteps between the states the forward saves for the backward (chunk_states). */
#define MB200_CHUNK 64

/* ---- selective scan ---------------------------------------------------------------------- */

/*
 * Forward scan parameters. Shapes (elements; all dense unless a stride is given):
 *   u, delta, z      : (batch, dim, seqlen), dtype io_dtype; seqlen-contiguous rows, batch / dim
 *                      strides below (dense by default)
 *   out              : (batch, dim, seqlen), dtype io_dtype, contiguous
 *   A                : (dim, dstate) float32, contiguous
 *   B, C             : (batch, ngroups, dstate, seqlen), dtype bc_dtype, element strides given
 *                      below. seqlen stride 1 (the upstream layout) takes the vectorised path;
 *                      any other stride -- e.g. dstate (the reference kernel's (b, g, l, n)
 *                      layout, selective_scan.h:17) -- is accepted on a scalar-load path.
 *   D, delta_bias    : (dim) float32 or NULL
 *   last_state       : (batch, dim, dstate) float32 or NULL
 *   chunk_states     : (batch, dim, ceil(seqlen / MB200_CHUNK), dstate) float32 or NULL: the state
 *                      after every MB200_CHUNK timesteps, which the backward uses instead of
 *                      recomputing the forward from t = 0.
 *   initial_state    : (batch, dim, dstate) float32 or NULL: the state before the first step
 *                      (zeros when NULL, which is the reference's behaviour). Lets a sequence
 *                      be scanned in pieces, e.g. split across GPUs.
 * io_dtype in {F32, BF16, F16}; bc_dtype is F32 or equal to io_dtype.
 */
typedef struct mb200_scan_fwd_params {
  const void* u;
  const void* delta;
  const float* A;
  const void* B;
  const void* C;
  const float* D;
  const void* z;
  const float* delta_bias;
  void* out;
  float* last_state;
  float* chunk_states;
  const float* initial_state;
  int64_t batch, dim, seqlen, dstate, ngroups;
  int64_t B_batch_stride, B_group_stride, B_dstate_stride, B_seqlen_stride;
  int64_t C_batch_stride, C_group_stride, C_dstate_stride, C_seqlen_stride;
  int32_t io_dtype;
  int32_t bc_dtype;
  int32_t delta_softplus;
  int32_t reserved;
  /* Element strides of u, delta and z over batch and over dim; along seqlen they are contiguous.
   * 0 selects the dense value (dim * seqlen, seqlen); negative strides are rejected
   * (MB200_ERR_BAD_LAYOUT). Lets a caller hand over views -- the transposed delta projection,
   * one half of the in_proj output as z -- without copying them. The vectorised path needs
   * every row start 16-byte aligned; other strides run on the scalar-load path. The outputs and
   * the backward's dout, du, ddelta, dz stay dense. */
  int64_t u_batch_stride, u_dim_stride;
  int64_t delta_batch_stride, delta_dim_stride;
  int64_t z_batch_stride, z_dim_stride;
} mb200_scan_fwd_params;

/*
 * Backward scan parameters: the forward inputs (`fwd`; its out/last_state are ignored, its
 * chunk_states -- if not NULL -- must hold what the forward wrote) plus
 *   dout             : (batch, dim, seqlen) io_dtype
 *   dlast_state      : (batch, dim, dstate) float32 or NULL
 * and outputs
 *   du, ddelta       : (batch, dim, seqlen) io_dtype
 *   dz               : (batch, dim, seqlen) io_dtype; required iff fwd.z != NULL
 *   dA               : (dim, dstate) float32, summed over batch
 *   dB, dC           : (batch, ngroups, dstate, seqlen) contiguous, dtype dbc_dtype (F32 or
 *                      fwd.bc_dtype); overwritten
 *   dD, ddelta_bias  : (dim) float32, summed over batch; either may be NULL to skip it
 *   dinitial_state   : (batch, dim, dstate) float32 or NULL: gradient with respect to
 *                      fwd.initial_state (the adjoint entering the first step)
 * The reference returns dA/dD/ddelta_bias as per-batch partials that its Python layer sums
 * (selective_scan_interface.py:87); here the sum over batch happens on the device.
 */
typedef struct mb200_scan_bwd_params {
  mb200_scan_fwd_params fwd;
  const void* dout;
  const float* dlast_state;
  void* du;
  void* ddelta;
  void* dz;
  float* dA;
  void* dB;
  void* dC;
  float* dD;
  float* ddelta_bias;
  float* dinitial_state;
  int32_t dbc_dtype;
  int32_t reserved;
} mb200_scan_bwd_params;

/* Forward selective scan.
 * Replaces mamba_cpu::selective_scan_fwd_f32 (csrc/selective_scan.h:40, bound at
 * csrc/bindings.cpp:23-45) behind the op mamba_cpu::selective_scan_fwd
 * (src/mamba_cpu/ops/selective_scan_interface.py:16-40). */
MB200_API int mb200_selective_scan_fwd(const mb200_scan_fwd_params* p, void* stream);

/* Sequence pieces. When a call's whole rows give too few CTAs to fill the GPU (a small batch x dim,
 * e.g. one rank's shard of a dim-sharded problem), the scans cut every row into pieces of whole
 * 64-step chunks run by separate CTAs: a summary pass runs the recurrence of each piece from a
 * zero state (forward: pieces but the last; backward: the adjoint of pieces but the first), and
 * every piece then starts from its predecessors' composed state (the recurrence is affine in its
 * initial state). Results agree with whole rows to rounding. The forward keeps the summaries in a
 * workspace: mb200_selective_scan_fwd allocates it stream-ordered (cudaMallocAsync) when needed;
 * mb200_selective_scan_fwd_ws takes it from the caller. The backward's are part of its workspace.
 * No reference counterpart (the reference parallelises over rows only, csrc/selective_scan.cpp:
 * 320-324). */
/* Bytes of forward workspace for these parameters: 0 when rows are not split (or on bad
 * arguments). */
MB200_API size_t mb200_selective_scan_fwd_workspace_size(const mb200_scan_fwd_params* p);
/* mb200_selective_scan_fwd with a caller workspace (256-byte aligned, at least
 * mb200_selective_scan_fwd_workspace_size(p) bytes, need not be initialised). */
MB200_API int mb200_selective_scan_fwd_ws(const mb200_scan_fwd_params* p, void* workspace,
                                          size_t workspace_bytes, void* stream);
/* Force the pieces per row of later calls (0 restores the automatic choice). Process-wide; meant
 * for tests and tuning. */
MB200_API void mb200_set_sequence_pieces(int pieces);
/* The automatic choice (or the forced count) for the forward (backward = 0) or backward kernel
 * whose whole rows of `nchunks` chunks give `ctas` CTAs: the count G in 1..8 (at least 4 chunks per
 * piece) minimising (1 + s (G-1)/G) ceil(G w) / (G w), w = ctas / resident slots (3 per SM), s the
 * summary pass's cost per element relative to the kernel's (0.8 forward, 0.23 backward); a split
 * must gain 2 %. */
MB200_API int mb200_sequence_pieces(int64_t ctas, int nchunks, int backward);

/* Bytes of device workspace mb200_selective_scan_bwd needs for these parameters (0 on bad
 * arguments). Depends on shapes and on whether fwd.chunk_states is NULL, not on pointer values. */
MB200_API size_t mb200_selective_scan_bwd_workspace_size(const mb200_scan_bwd_params* p);

/* Backward selective scan. `workspace` must be 256-byte aligned and hold at least
 * mb200_selective_scan_bwd_workspace_size(p) bytes; it need not be initialised.
 * Replaces mamba_cpu::selective_scan_bwd_f32 (csrc/selective_scan.h:65, bound at
 * csrc/bindings.cpp:47-84) behind mamba_cpu::selective_scan_bwd
 * (src/mamba_cpu/ops/selective_scan_interface.py:48-87). */
MB200_API int mb200_selective_scan_bwd(const mb200_scan_bwd_params* p, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* Size of the static device scratch behind mb200_selective_scan_bwd_noalloc (16 MiB). */
#define MB200_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)

/* Backward selective scan that allocates nothing, for callers that can neither allocate device
 * memory nor provide a workspace (e.g. a host framework that owns all device memory and forbids
 * allocation inside its execute callbacks). This entry point has no counterpart in the reference.
 * It runs mb200_selective_scan_bwd with a workspace carved from a static device array of
 * MB200_NOALLOC_SCRATCH_BYTES that every GPU loading this library holds until the process exits.
 * Requests whose mb200_selective_scan_bwd_workspace_size exceeds that limit return
 * MB200_ERR_SCRATCH_LIMIT before anything is enqueued (with fwd.chunk_states given, about a
 * batch 4 x dim 1536 x seqlen 1024 problem fits; without it roughly half that).
 * The first call on each device resolves the array's device address (a runtime query) and should
 * come before any stream capture on that device; a failed lookup returns MB200_ERR_CUDA and is
 * retried by the next call (only a successful lookup is kept). All calls on a device share the array: calls
 * whose GPU work may overlap (other streams, other host threads) race and must be serialised by
 * the caller. Nothing in the array needs clearing between calls. */
MB200_API int mb200_selective_scan_bwd_noalloc(const mb200_scan_bwd_params* p, void* stream);

/* Exact mirror of the reference binding `selective_scan_fwd_f32` (csrc/bindings.cpp:23-45):
 * same argument order and meaning -- float32 everywhere, B/C in the reference kernel's
 * (batch, ngroups, seqlen, dstate) layout (selective_scan.h:17) -- with `stream` in place of
 * num_threads. last_state may be NULL. */
MB200_API int mb200_selective_scan_fwd_f32(const float* u, const float* delta, const float* A,
                                           const float* B, const float* C, const float* D,
                                           const float* z, const float* delta_bias, float* out,
                                           float* last_state, int64_t batch, int64_t dim,
                                           int64_t seqlen, int64_t dstate, int64_t ngroups,
                                           int delta_softplus, void* stream);

/* Exact mirror of the reference binding `selective_scan_bwd_f32` (csrc/bindings.cpp:47-84),
 * float32, B/C/dB/dC in (batch, ngroups, seqlen, dstate). As in the reference, dA_part (batch,
 * dim, dstate), dD_part (batch, dim) and ddelta_bias_part (batch, dim) are per-batch partials.
 * dB/dC are overwritten (the reference accumulates into zero-initialised buffers,
 * selective_scan.h:47, which gives the same result). Scratch is allocated stream-ordered. */
MB200_API int mb200_selective_scan_bwd_f32(
    const float* u, const float* delta, const float* A, const float* B, const float* C,
    const float* D, const float* z, const float* delta_bias, const float* dout,
    const float* dlast_state, float* du, float* ddelta, float* dA_part, float* dB, float* dC,
    float* dD_part, float* dz, float* ddelta_bias_part, int64_t batch, int64_t dim,
    int64_t seqlen, int64_t dstate, int64_t ngroups, int delta_softplus, void* stream);

/* ---- causal depthwise conv1d ------------------------------------------------------------- */

/*
 *   x, out        : (batch, dim, seqlen), dtype x_dtype (F32 / BF16 / F16), contiguous
 *   weight        : (dim, width) float32, 1 <= width <= 8
 *   bias          : (dim) float32 or NULL
 *   initial_states: (batch, dim, width - 1) x_dtype or NULL (zeros)
 *   final_states  : (batch, dim, width - 1) x_dtype or NULL: the last width-1 inputs of
 *                   [initial_states | x] (causal_conv1d.py:48-53)
 *   activation    : 0 = none, 1 = SiLU
 */
typedef struct mb200_conv1d_params {
  const void* x;
  const float* weight;
  const float* bias;
  const void* initial_states;
  void* out;
  void* final_states;
  int64_t batch, dim, seqlen, width;
  int32_t x_dtype;
  int32_t activation;
} mb200_conv1d_params;

/* Causal depthwise conv1d with optional SiLU. Replaces the F.conv1d path of
 * causal_conv1d_fn (src/mamba_cpu/ops/causal_conv1d.py:16-53). */
MB200_API int mb200_causal_conv1d_fwd(const mb200_conv1d_params* p, void* stream);

/* Backward of mb200_causal_conv1d_fwd (torch autograd's gradient of causal_conv1d.py:37-47):
 *   dout (batch, dim, seqlen) x_dtype -> dx (x_dtype), dweight (dim, width) f32,
 *   dbias (dim) f32 or NULL, dinitial_states (batch, dim, width-1) x_dtype or NULL. */
MB200_API size_t mb200_causal_conv1d_bwd_workspace_size(const mb200_conv1d_params* p);
MB200_API int mb200_causal_conv1d_bwd(const mb200_conv1d_params* p, const void* dout, void* dx,
                                      float* dweight, float* dbias, void* dinitial_states,
                                      void* workspace, size_t workspace_bytes, void* stream);

/* ---- decode steps (the reference runs these in plain PyTorch) --------------------------- */

/*
 * One selective-scan step per (batch, channel) updating `state` in place.
 * Replaces selective_state_update (src/mamba_cpu/ops/selective_state_update.py:5-57) for the
 * Mamba-1 layout; the multi-head layout is the same after flattening (heads*headdim -> dim):
 *   state (batch, dim, dstate) float32 or io_dtype (state_dtype); x, dt, z, out (batch, dim)
 *   io_dtype; A (dim, dstate) f32; B, C (batch, ngroups, dstate) bc_dtype contiguous;
 *   D, dt_bias (dim) f32 or NULL. dstate up to MB200_DECODE_MAX_DSTATE (the reference's PyTorch
 *   version takes any dstate; Mamba-2 heads use 64 or 128).
 */
typedef struct mb200_state_update_params {
  void* state;
  const void* x;
  const void* dt;
  const float* A;
  const void* B;
  const void* C;
  const float* D;
  const void* z;
  const float* dt_bias;
  void* out;
  int64_t batch, dim, dstate, ngroups;
  int32_t io_dtype, bc_dtype, state_dtype;
  int32_t dt_softplus;
} mb200_state_update_params;

MB200_API int mb200_selective_state_update(const mb200_state_update_params* p, void* stream);

/*
 * Decode conv step(s): causal_conv1d_update (src/mamba_cpu/ops/causal_conv1d.py:56-85).
 *   x, out (batch, dim, seqlen) x_dtype; conv_state (batch, dim, state_len) x_dtype, rolled in
 *   place by seqlen steps; state_len >= width - 1; weight (dim, width) f32; bias f32 or NULL.
 */
typedef struct mb200_conv1d_update_params {
  const void* x;
  void* conv_state;
  const float* weight;
  const float* bias;
  void* out;
  int64_t batch, dim, seqlen, state_len, width;
  int32_t x_dtype;
  int32_t activation;
} mb200_conv1d_update_params;

MB200_API int mb200_causal_conv1d_update(const mb200_conv1d_update_params* p, void* stream);

/* ---- Mamba-2 SSD chunk scan (forward) ------------------------------------------------------
 *
 * The reference lists the Mamba-2 SSD scan `mamba_chunk_scan_combined` as a roadmap item
 * (README.md:94) and has no implementation of it; this entry point computes the forward of
 * upstream mamba_ssm's function of that name (ssd_combined.py). Per (batch, head), with a scalar
 * decay A[h] shared by the head's headdim x dstate state:
 *   dt_t  = clamp(softplus?(dt[b, t, h] + dt_bias[h]), dt_min, dt_max)
 *   h_t   = exp(dt_t A[h]) h_{t-1} + dt_t x_t B_t^T        (headdim x dstate, fp32)
 *   y_t   = h_t C_t + D x_t ;   out_t = y_t * silu(z_t) when z is given
 * which is the Mamba-1 selective scan with channels = nheads * headdim, A broadcast over dstate
 * and delta broadcast over headdim (the reference's selective_scan_fwd_f32 on those inputs,
 * csrc/selective_scan.cpp:120-145, computes the same values).
 *   x, z, out       : (batch, seqlen, nheads, headdim) x_dtype; headdim contiguous, other strides
 *                     below (out dense). Row starts (x, z, out, B, C) 16-byte aligned.
 *   dt              : (batch, seqlen, nheads) float32, nheads contiguous, strides below
 *   A               : (nheads) float32; dt_bias (nheads) float32 or NULL
 *   B, C            : (batch, seqlen, ngroups, dstate) x_dtype, dstate contiguous; head h reads
 *                     group h / (nheads / ngroups)
 *   D               : (nheads) or (nheads, headdim) (D_per_dim = 1) float32, or NULL
 *   initial_states  : (batch, nheads, headdim, dstate) float32 or NULL (zeros)
 *   final_states    : (batch, nheads, headdim, dstate) float32 or NULL: the state after the last
 *                     step
 *   seq_idx         : (batch, seqlen) int32, non-decreasing along seqlen, or NULL: packed
 *                     sequences; no step sees another sequence's steps and the state restarts
 *                     from zero where the index changes. initial_states belong to sequence 0 (as
 *                     upstream: they are dropped if seq_idx[b, 0] != 0), final_states are the
 *                     last sequence's.
 * Limits of this build: x_dtype MB200_BF16 or MB200_F16 (x, z, B, C and out all of that type),
 * dstate a multiple of 8 up to 128, headdim a multiple of 32 up to 256 (MB200_ERR_UNSUPPORTED
 * otherwise). One kernel launch, no scratch memory.
 */
typedef struct mb200_ssd_params {
  const void* x;
  const float* dt;
  const float* A;
  const void* B;
  const void* C;
  const float* D;
  const void* z;
  const float* dt_bias;
  const float* initial_states;
  void* out;
  float* final_states;
  int64_t batch, seqlen, nheads, headdim, ngroups, dstate;
  int64_t x_batch_stride, x_seqlen_stride, x_head_stride;
  int64_t z_batch_stride, z_seqlen_stride, z_head_stride;
  int64_t B_batch_stride, B_seqlen_stride, B_group_stride;
  int64_t C_batch_stride, C_seqlen_stride, C_group_stride;
  int64_t dt_batch_stride, dt_seqlen_stride;
  const int32_t* seq_idx;
  int64_t seq_idx_batch_stride, seq_idx_seqlen_stride;
  float dt_min, dt_max;
  int32_t x_dtype;
  int32_t dt_softplus;
  int32_t D_per_dim;
  int32_t reserved;
} mb200_ssd_params;

MB200_API int mb200_ssd_chunk_scan_fwd(const mb200_ssd_params* p, void* stream);

/* ---- misc -------------------------------------------------------------------------------- */

/* ---- one-shot sum over the GPUs of a node through peer memory ------------------------------
 *
 * The dB / dC partial sums of a channel-sharded backward are combined across ranks by reading
 * every rank's partial over NVLink instead of a ring all-reduce (which at these sizes, ~0.5 MB,
 * is dominated by per-step latency). Every rank owns an exchange buffer of 2 * n floats (two
 * slots, used alternately) and a signal pad of `world` uint32, shared with the other ranks of
 * the node through CUDA IPC (plain peer mappings, no multicast objects):
 *
 *   mb200_peer_alloc / mb200_peer_free    zeroed device allocation (its own base, as IPC needs)
 *   mb200_ipc_handle / mb200_ipc_open     export / map an allocation of another process
 *   mb200_peer_sum_f32                    in place: a[0..na) | b[0..nb) := the sum over all ranks
 *                                         of their a | b (every rank gets the same bits: ranks
 *                                         are added in rank order)
 *
 * peer_bufs / peer_pads are DEVICE arrays of `world` pointers (this rank's own at index `rank`) to
 * the ranks' exchange buffers (8 * ceil((na + nb) / 4) floats each) and signal pads (world *
 * MB200_PEER_BLOCKS uint32 each, zeroed); `counters` is this rank's device array of
 * MB200_PEER_BLOCKS + 1 uint32, zeroed: the first MB200_PEER_BLOCKS are call numbers that only
 * these calls advance (they select the slot and the values the signals carry, so the call is
 * valid inside CUDA graphs), the last is a sticky timeout flag. One kernel of MB200_PEER_BLOCKS
 * CTAs per call; CTA j of a rank waits only for CTA j of the others. The wait for the other ranks
 * is bounded by timeout_us of GPU time (<= 0: 30 s); a CTA whose wait runs out writes NaN into
 * its share of a | b instead of the sum, sets bit 1 of the fault word of mb200_device_fault and
 * sets counters[MB200_PEER_BLOCKS] to 1 (left set; the caller reads it to refuse the result and
 * clears it). The signals stay in step, so a late rank's own call still sums correctly. All ranks
 * must make the same sequence of calls with the same sizes, and the calls of one rank on one set
 * of buffers must not overlap (issue them on one stream).
 */
#define MB200_IPC_HANDLE_BYTES 64
#define MB200_PEER_BLOCKS 148
MB200_API int mb200_peer_alloc(size_t bytes, void** dev_ptr);
MB200_API int mb200_peer_free(void* dev_ptr);
MB200_API int mb200_ipc_handle(void* dev_ptr, unsigned char handle[MB200_IPC_HANDLE_BYTES]);
MB200_API int mb200_ipc_open(const unsigned char handle[MB200_IPC_HANDLE_BYTES], void** dev_ptr);
MB200_API int mb200_ipc_close(void* dev_ptr);
MB200_API int mb200_peer_sum_f32(float* a, int64_t na, float* b, int64_t nb, float* const* peer_bufs,
                                 uint32_t* const* peer_pads, uint32_t* counters, int rank, int world,
                                 int64_t timeout_us, void* stream);

/* Static description of a status code. */
MB200_API const char* mb200_status_string(int status);

/* Library ABI version: (major << 16) | minor. */
MB200_API int mb200_version(void);

/* Number of kernel launches the most recent successful call on this host thread enqueued. */
MB200_API int mb200_last_launch_count(void);

/* Read and clear the device-side fault word of the current device (synchronises the device).
 * Kernels never trap: a bounded wait that gave up (a staged copy that did not arrive in ~2.5 s)
 * sets bit 0, a peer that did not signal within the timeout (mb200_peer_sum_f32) bit 1, and the
 * kernel finishes with unspecified outputs. *fault = 0 means no fault. */
MB200_API int mb200_device_fault(int* fault);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA_B200_H */
