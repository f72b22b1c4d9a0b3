/*
 * oracle.c -- float64 CPU restatement of the Mamba-1 selective scan and the causal
 * depthwise conv1d, used ONLY as the parity checker for the CUDA kernels.
 *
 * TEST INFRASTRUCTURE. Nothing in the product path (the CUDA library or the Python
 * package) links, loads or calls this file. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg use it.
 *
 * The math follows the reference implementation (SandyTheAdventurer/mamba-cpu), restated
 * in double precision with libm exp/log1p instead of the reference's polynomial exp:
 *   forward  : csrc/selective_scan.cpp:120-145 (fwd_row_body), :94-115 (row_ptrs, row_dt),
 *              :45 (softplus with threshold 20), :47 (sigmoid)
 *   backward : csrc/selective_scan.cpp:168-248 (bwd_row_body); the per-batch partials of
 *              dA / dD / ddelta_bias are summed over batch as
 *              src/mamba_cpu/ops/selective_scan_interface.py:87 does.
 *   conv1d   : src/mamba_cpu/ops/causal_conv1d.py:16-53 (left pad or initial_states,
 *              depthwise conv, optional SiLU, final states) and the gradient torch autograd
 *              derives for it.
 *   decode   : src/mamba_cpu/ops/selective_state_update.py:5-57 (Mamba-1 layout) and
 *              src/mamba_cpu/ops/causal_conv1d.py:56-85 (causal_conv1d_update).
 *
 * Layouts (all dense, row-major):
 *   u, delta, z, out, dout, du, ddelta, dz : (batch, dim, seqlen)
 *   A, dA                                   : (dim, dstate)
 *   B, C, dB, dC                            : (batch, ngroups, dstate, seqlen)  (l-contiguous,
 *                                             the upstream layout; the reference kernel's own
 *                                             (batch, ngroups, seqlen, dstate) is a transpose)
 *   D, delta_bias, dD, ddelta_bias          : (dim)
 *   last_state, dlast_state                 : (batch, dim, dstate)
 * Null pointers mean "absent" exactly as in the reference (selective_scan.h:20).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <unistd.h>

/* ---- a minimal parallel-for over [0, count) on pthreads (static contiguous chunks) ------ */

typedef void (*body_fn)(int64_t lo, int64_t hi, void* ctx);

typedef struct {
  body_fn fn;
  void* ctx;
  int64_t lo, hi;
} chunk_arg;

static void* chunk_main(void* p) {
  chunk_arg* a = (chunk_arg*)p;
  a->fn(a->lo, a->hi, a->ctx);
  return NULL;
}

static int g_threads = 0; /* 0 = one per online CPU */

void oracle_set_num_threads(int n) { g_threads = n; }

int oracle_num_threads(void) {
  if (g_threads > 0) return g_threads;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

static void parallel_for(int64_t count, body_fn fn, void* ctx) {
  int nt = oracle_num_threads();
  if (nt > 64) nt = 64;
  if ((int64_t)nt > count) nt = (int)count;
  if (nt <= 1) {
    if (count > 0) fn(0, count, ctx);
    return;
  }
  pthread_t tid[64];
  chunk_arg args[64];
  const int64_t per = count / nt, rem = count % nt;
  int64_t start = 0;
  for (int i = 0; i < nt; ++i) {
    args[i].fn = fn;
    args[i].ctx = ctx;
    args[i].lo = start;
    args[i].hi = start + per + (i < rem ? 1 : 0);
    start = args[i].hi;
    pthread_create(&tid[i], NULL, chunk_main, &args[i]);
  }
  for (int i = 0; i < nt; ++i) pthread_join(tid[i], NULL);
}

static double softplus_d(double x) { return x <= 20.0 ? log1p(exp(x)) : x; }
static double sigmoid_d(double x) { return 1.0 / (1.0 + exp(-x)); }

/* Channel d of batch b reads the B/C slice of its group: selective_scan.cpp:99. */
static int64_t bc_slice(int64_t b, int64_t d, int64_t dim, int64_t ngroups) {
  return b * ngroups + d / (dim / ngroups);
}

static double row_dt(const float* delta_row, double bias, int64_t t, int softplus) {
  double dt = (double)delta_row[t] + bias;
  return softplus ? softplus_d(dt) : dt;
}

/* Forward: selective_scan.cpp:120-145. out and last_state are float64. */
typedef struct {
  const float *u, *delta, *A, *B, *C, *D, *z, *delta_bias, *h_init;
  double *out, *last_state;
  int64_t batch, dim, seqlen, dstate, ngroups;
  int softplus;
} fwd_ctx;

static void fwd_rows(int64_t lo, int64_t hi, void* vctx) {
  const fwd_ctx* c = (const fwd_ctx*)vctx;
  const int64_t L = c->seqlen, N = c->dstate;
  double h[256];
  for (int64_t idx = lo; idx < hi; ++idx) {
    const int64_t b = idx / c->dim, d = idx % c->dim;
    const int64_t slice = bc_slice(b, d, c->dim, c->ngroups);
    const float* ur = c->u + idx * L;
    const float* dr = c->delta + idx * L;
    const float* zr = c->z ? c->z + idx * L : NULL;
    const float* Bs = c->B + slice * N * L;
    const float* Cs = c->C + slice * N * L;
    const double Dd = c->D ? (double)c->D[d] : 0.0;
    const double bias = c->delta_bias ? (double)c->delta_bias[d] : 0.0;
    for (int64_t n = 0; n < N; ++n) h[n] = c->h_init ? (double)c->h_init[idx * N + n] : 0.0;
    for (int64_t t = 0; t < L; ++t) {
      const double dt = row_dt(dr, bias, t, c->softplus);
      const double dtu = dt * (double)ur[t];
      double y = 0.0;
      for (int64_t n = 0; n < N; ++n) {
        h[n] = exp(dt * (double)c->A[d * N + n]) * h[n] + dtu * (double)Bs[n * L + t];
        y += h[n] * (double)Cs[n * L + t];
      }
      y += Dd * (double)ur[t];
      if (zr) {
        const double zt = (double)zr[t];
        y *= zt * sigmoid_d(zt);
      }
      c->out[idx * L + t] = y;
    }
    if (c->last_state)
      for (int64_t n = 0; n < N; ++n) c->last_state[idx * N + n] = h[n];
  }
}

/* h_init: (batch, dim, dstate) state before the first step, or NULL for zeros (an extension of
 * the reference, which always starts from zero; used to check sequence-sharded scans). */
int oracle_scan_fwd_init(const float* u, const float* delta, const float* A, const float* B,
                         const float* C, const float* D, const float* z, const float* delta_bias,
                         const float* h_init, double* out, double* last_state, int64_t batch,
                         int64_t dim, int64_t seqlen, int64_t dstate, int64_t ngroups, int softplus) {
  if (dstate > 256 || ngroups <= 0 || dim % ngroups) return 1;
  fwd_ctx c = {u, delta, A, B, C, D, z, delta_bias, h_init, out, last_state,
               batch, dim, seqlen, dstate, ngroups, softplus};
  parallel_for(batch * dim, fwd_rows, &c);
  return 0;
}

int oracle_scan_fwd(const float* u, const float* delta, const float* A, const float* B,
                    const float* C, const float* D, const float* z, const float* delta_bias,
                    double* out, double* last_state, int64_t batch, int64_t dim, int64_t seqlen,
                    int64_t dstate, int64_t ngroups, int softplus) {
  return oracle_scan_fwd_init(u, delta, A, B, C, D, z, delta_bias, NULL, out, last_state, batch, dim,
                              seqlen, dstate, ngroups, softplus);
}

/*
 * Backward: selective_scan.cpp:168-248 in float64, with the batch sums of
 * selective_scan_interface.py:87 folded in. dA, dD, ddelta_bias are (dim[,dstate]) totals.
 * dB / dC are overwritten (not accumulated into). dz may be NULL when z is NULL; dD and
 * ddelta_bias are always written, as the reference op always computes them.
 *
 * dB/dC sum over the channels of a (batch, group) slice (selective_scan.cpp:335-368). Here
 * each slice's channels are cut into a fixed number of blocks (independent of the thread
 * count); every block accumulates privately and the blocks are added in order at the end,
 * so the result is the same for any number of threads.
 */
#define BWD_BLOCKS_PER_SLICE 16

typedef struct {
  const float *u, *delta, *A, *B, *C, *D, *z, *delta_bias, *dout, *dlast, *h_init;
  double *du, *ddelta, *dz, *dh_init;
  double *dA_part, *dD_part, *db_part; /* per row */
  double* blk;                          /* (slices, blocks, 2, N, L) */
  int64_t batch, dim, seqlen, dstate, ngroups, blocks;
  int softplus;
} bwd_ctx;

static void bwd_blocks(int64_t lo, int64_t hi, void* vctx) {
  const bwd_ctx* c = (const bwd_ctx*)vctx;
  const int64_t L = c->seqlen, N = c->dstate, dim = c->dim;
  const int64_t dpg = dim / c->ngroups;
  double* hs = (double*)malloc(sizeof(double) * (size_t)(L * N > 0 ? L * N : 1));
  double gh[256], dA_acc[256];
  for (int64_t job = lo; job < hi; ++job) {
    const int64_t slice = job / c->blocks, blk = job % c->blocks;
    const int64_t b = slice / c->ngroups, g = slice % c->ngroups;
    const int64_t d_lo = g * dpg + (dpg * blk) / c->blocks;
    const int64_t d_hi = g * dpg + (dpg * (blk + 1)) / c->blocks;
    double* dBs = c->blk + ((slice * c->blocks + blk) * 2 + 0) * N * L;
    double* dCs = c->blk + ((slice * c->blocks + blk) * 2 + 1) * N * L;
    const float* Bs = c->B + slice * N * L;
    const float* Cs = c->C + slice * N * L;
    for (int64_t d = d_lo; d < d_hi; ++d) {
      const int64_t idx = b * dim + d;
      const float* ur = c->u + idx * L;
      const float* dr = c->delta + idx * L;
      const float* zr = c->z ? c->z + idx * L : NULL;
      const float* dor = c->dout + idx * L;
      const double Dd = c->D ? (double)c->D[d] : 0.0;
      const double bias = c->delta_bias ? (double)c->delta_bias[d] : 0.0;
      const float* Ar = c->A + d * N;
      /* Forward recompute keeping every state: selective_scan.cpp:182-190. */
      for (int64_t t = 0; t < L; ++t) {
        const double dt = row_dt(dr, bias, t, c->softplus);
        const double dtu = dt * (double)ur[t];
        for (int64_t n = 0; n < N; ++n) {
          const double hp = t > 0 ? hs[(t - 1) * N + n] : (c->h_init ? (double)c->h_init[idx * N + n] : 0.0);
          hs[t * N + n] = exp(dt * (double)Ar[n]) * hp + dtu * (double)Bs[n * L + t];
        }
      }
      /* Reverse adjoint scan: selective_scan.cpp:192-243. */
      for (int64_t n = 0; n < N; ++n) {
        gh[n] = c->dlast ? (double)c->dlast[idx * N + n] : 0.0;
        dA_acc[n] = 0.0;
      }
      double dD_acc = 0.0, dbias_acc = 0.0;
      for (int64_t t = L - 1; t >= 0; --t) {
        const double dt = row_dt(dr, bias, t, c->softplus);
        const double ut = (double)ur[t];
        const double dtu = dt * ut;
        const double* h = hs + t * N;
        double dy = (double)dor[t];
        if (zr) {
          double y = 0.0;
          for (int64_t n = 0; n < N; ++n) y += h[n] * (double)Cs[n * L + t];
          y += Dd * ut;
          const double zt = (double)zr[t];
          const double sg = sigmoid_d(zt);
          c->dz[idx * L + t] = (double)dor[t] * y * sg * (1.0 + zt * (1.0 - sg));
          dy = (double)dor[t] * zt * sg;
        }
        dD_acc += dy * ut;
        double ddt = 0.0, gB = 0.0;
        for (int64_t n = 0; n < N; ++n) {
          const double Bn = (double)Bs[n * L + t];
          const double Cn = (double)Cs[n * L + t];
          const double hp = t > 0 ? hs[(t - 1) * N + n] : (c->h_init ? (double)c->h_init[idx * N + n] : 0.0);
          const double g = gh[n] + dy * Cn;
          dCs[n * L + t] += dy * h[n];
          const double a = exp(dt * (double)Ar[n]);
          const double g_a = g * hp * a;
          dA_acc[n] += g_a * dt;
          ddt += g_a * (double)Ar[n] + g * ut * Bn;
          gB += g * Bn;
          dBs[n * L + t] += g * dtu;
          gh[n] = g * a;
        }
        c->du[idx * L + t] = dy * Dd + dt * gB;
        if (c->softplus) ddt *= sigmoid_d((double)dr[t] + bias);
        c->ddelta[idx * L + t] = ddt;
        dbias_acc += ddt;
      }
      for (int64_t n = 0; n < N; ++n) c->dA_part[idx * N + n] = dA_acc[n];
      if (c->dh_init)
        for (int64_t n = 0; n < N; ++n) c->dh_init[idx * N + n] = gh[n];
      c->dD_part[idx] = dD_acc;
      c->db_part[idx] = dbias_acc;
    }
  }
  free(hs);
}

/* h_init as in oracle_scan_fwd_init; dh_init (batch, dim, dstate) receives the gradient with
 * respect to it (may be NULL). */
int oracle_scan_bwd_init(const float* u, const float* delta, const float* A, const float* B,
                         const float* C, const float* D, const float* z, const float* delta_bias,
                         const float* h_init, const float* dout, const float* dlast_state, double* du,
                         double* ddelta, double* dA, double* dB, double* dC, double* dD, double* dz,
                         double* ddelta_bias, double* dh_init, int64_t batch, int64_t dim,
                         int64_t seqlen, int64_t dstate, int64_t ngroups, int softplus) {
  if (dstate > 256 || ngroups <= 0 || dim % ngroups) return 1;
  const int64_t L = seqlen, N = dstate;
  const int64_t rows = batch * dim;
  const int64_t slices = batch * ngroups;
  const int64_t dpg = dim / ngroups;
  const int64_t blocks = dpg < BWD_BLOCKS_PER_SLICE ? (dpg > 0 ? dpg : 1) : BWD_BLOCKS_PER_SLICE;
  bwd_ctx c;
  c.u = u; c.delta = delta; c.A = A; c.B = B; c.C = C; c.D = D; c.z = z;
  c.delta_bias = delta_bias; c.dout = dout; c.dlast = dlast_state; c.h_init = h_init;
  c.du = du; c.ddelta = ddelta; c.dz = dz; c.dh_init = dh_init;
  c.dA_part = (double*)calloc((size_t)(rows * N + 1), sizeof(double));
  c.dD_part = (double*)calloc((size_t)(rows + 1), sizeof(double));
  c.db_part = (double*)calloc((size_t)(rows + 1), sizeof(double));
  c.blk = (double*)calloc((size_t)(slices * blocks * 2 * N * L + 1), sizeof(double));
  c.batch = batch; c.dim = dim; c.seqlen = seqlen; c.dstate = dstate; c.ngroups = ngroups;
  c.blocks = blocks; c.softplus = softplus;
  if (!c.dA_part || !c.dD_part || !c.db_part || !c.blk) {
    free(c.dA_part); free(c.dD_part); free(c.db_part); free(c.blk);
    return 2;
  }
  parallel_for(slices * blocks, bwd_blocks, &c);
  for (int64_t s = 0; s < slices; ++s) {
    for (int64_t q = 0; q < 2; ++q) {
      double* dst = (q == 0 ? dB : dC) + s * N * L;
      for (int64_t i = 0; i < N * L; ++i) dst[i] = 0.0;
      for (int64_t k = 0; k < blocks; ++k) {
        const double* src = c.blk + ((s * blocks + k) * 2 + q) * N * L;
        for (int64_t i = 0; i < N * L; ++i) dst[i] += src[i];
      }
    }
  }
  for (int64_t d = 0; d < dim; ++d) {
    for (int64_t n = 0; n < N; ++n) {
      double acc = 0.0;
      for (int64_t b = 0; b < batch; ++b) acc += c.dA_part[(b * dim + d) * N + n];
      dA[d * N + n] = acc;
    }
    double sD = 0.0, sb = 0.0;
    for (int64_t b = 0; b < batch; ++b) {
      sD += c.dD_part[b * dim + d];
      sb += c.db_part[b * dim + d];
    }
    dD[d] = sD;
    ddelta_bias[d] = sb;
  }
  free(c.dA_part); free(c.dD_part); free(c.db_part); free(c.blk);
  return 0;
}

int oracle_scan_bwd(const float* u, const float* delta, const float* A, const float* B,
                    const float* C, const float* D, const float* z, const float* delta_bias,
                    const float* dout, const float* dlast_state, double* du, double* ddelta,
                    double* dA, double* dB, double* dC, double* dD, double* dz,
                    double* ddelta_bias, int64_t batch, int64_t dim, int64_t seqlen,
                    int64_t dstate, int64_t ngroups, int softplus) {
  return oracle_scan_bwd_init(u, delta, A, B, C, D, z, delta_bias, NULL, dout, dlast_state, du, ddelta,
                              dA, dB, dC, dD, dz, ddelta_bias, NULL, batch, dim, seqlen, dstate, ngroups,
                              softplus);
}

/* ---- causal depthwise conv1d: ops/causal_conv1d.py:16-53 ------------------------------- */

static double act_fwd(double x, int silu) { return silu ? x * sigmoid_d(x) : x; }
static double act_grad(double x, int silu) {
  if (!silu) return 1.0;
  const double s = sigmoid_d(x);
  return s * (1.0 + x * (1.0 - s));
}

typedef struct {
  const float *x, *w, *bias, *init, *dout;
  double *out, *final_states, *dx, *dw, *dbias, *dinit;
  int64_t batch, dim, seqlen, width;
  int silu;
} conv_ctx;

/* Value of [init | zeros, x] at x-index s (s < 0 reads the initial state / zero pad). */
static double conv_in(const float* xr, const float* ir, int64_t P, int64_t s) {
  if (s >= 0) return (double)xr[s];
  return ir ? (double)ir[P + s] : 0.0;
}

static void conv_fwd_rows(int64_t lo, int64_t hi, void* vctx) {
  const conv_ctx* c = (const conv_ctx*)vctx;
  const int64_t L = c->seqlen, W = c->width, P = W - 1;
  for (int64_t idx = lo; idx < hi; ++idx) {
    const int64_t d = idx % c->dim;
    const float* xr = c->x + idx * L;
    const float* ir = c->init ? c->init + idx * P : NULL;
    for (int64_t t = 0; t < L; ++t) {
      double acc = c->bias ? (double)c->bias[d] : 0.0;
      for (int64_t k = 0; k < W; ++k) acc += (double)c->w[d * W + k] * conv_in(xr, ir, P, t - P + k);
      c->out[idx * L + t] = act_fwd(acc, c->silu);
    }
    if (c->final_states)
      for (int64_t j = 0; j < P; ++j) c->final_states[idx * P + j] = conv_in(xr, ir, P, L - P + j);
  }
}

/* x (b,d,l); w (d,W); bias (d) or NULL; init (b,d,W-1) or NULL; out (b,d,l);
 * final_states (b,d,W-1) or NULL: the last W-1 entries of [init|zeros, x] (causal_conv1d.py:48-53). */
int oracle_conv1d_fwd(const float* x, const float* w, const float* bias, const float* init,
                      double* out, double* final_states, int64_t batch, int64_t dim,
                      int64_t seqlen, int64_t width, int silu) {
  if (width < 1 || width > 64) return 1;
  conv_ctx c = {x, w, bias, init, NULL, out, final_states, NULL, NULL, NULL, NULL,
                batch, dim, seqlen, width, silu};
  parallel_for(batch * dim, conv_fwd_rows, &c);
  return 0;
}

static void conv_bwd_channels(int64_t lo, int64_t hi, void* vctx) {
  const conv_ctx* c = (const conv_ctx*)vctx;
  const int64_t L = c->seqlen, W = c->width, P = W - 1, dim = c->dim;
  for (int64_t d = lo; d < hi; ++d) {
    double dwacc[64];
    for (int64_t k = 0; k < W; ++k) dwacc[k] = 0.0;
    double dbacc = 0.0;
    for (int64_t b = 0; b < c->batch; ++b) {
      const int64_t idx = b * dim + d;
      const float* xr = c->x + idx * L;
      const float* ir = c->init ? c->init + idx * P : NULL;
      for (int64_t t = 0; t < L; ++t) c->dx[idx * L + t] = 0.0;
      if (c->dinit)
        for (int64_t j = 0; j < P; ++j) c->dinit[idx * P + j] = 0.0;
      for (int64_t t = 0; t < L; ++t) {
        double pre = c->bias ? (double)c->bias[d] : 0.0;
        for (int64_t k = 0; k < W; ++k) pre += (double)c->w[d * W + k] * conv_in(xr, ir, P, t - P + k);
        const double g = (double)c->dout[idx * L + t] * act_grad(pre, c->silu);
        dbacc += g;
        for (int64_t k = 0; k < W; ++k) {
          const int64_t s = t - P + k;
          dwacc[k] += g * conv_in(xr, ir, P, s);
          if (s >= 0)
            c->dx[idx * L + s] += g * (double)c->w[d * W + k];
          else if (c->dinit)
            c->dinit[idx * P + P + s] += g * (double)c->w[d * W + k];
        }
      }
    }
    for (int64_t k = 0; k < W; ++k) c->dw[d * W + k] = dwacc[k];
    if (c->dbias) c->dbias[d] = dbacc;
  }
}

/* Gradient of oracle_conv1d_fwd w.r.t. x, w, bias and init (dbias, dinit may be NULL).
 * dw (d,W) and dbias (d) are summed over batch and time. */
int oracle_conv1d_bwd(const float* x, const float* w, const float* bias, const float* init,
                      const float* dout, double* dx, double* dw, double* dbias, double* dinit,
                      int64_t batch, int64_t dim, int64_t seqlen, int64_t width, int silu) {
  if (width < 1 || width > 64) return 1;
  conv_ctx c = {x, w, bias, init, dout, NULL, NULL, dx, dw, dbias, dinit,
                batch, dim, seqlen, width, silu};
  parallel_for(dim, conv_bwd_channels, &c);
  return 0;
}

/* ---- decode steps ---------------------------------------------------------------------- */

/* selective_state_update.py:5-57, Mamba-1 layout with optional heads flattened by the caller:
 * state (b,d,n) updated in place (float64 copy passed in), x/dt/z (b,d), A (d,n),
 * B/C (b,g,n) with d/(dim/g) picking the group (repeat_interleave, :120-121), D/dt_bias (d). */
void oracle_state_update(double* state, const float* x, const float* dt, const float* A,
                         const float* B, const float* C, const float* D, const float* z,
                         const float* dt_bias, double* out, int64_t batch, int64_t dim,
                         int64_t dstate, int64_t ngroups, int softplus) {
  const int64_t N = dstate;
  for (int64_t b = 0; b < batch; ++b) {
    for (int64_t d = 0; d < dim; ++d) {
      const int64_t idx = b * dim + d;
      const int64_t g = d / (dim / ngroups);
      double dtv = (double)dt[idx] + (dt_bias ? (double)dt_bias[d] : 0.0);
      if (softplus) dtv = softplus_d(dtv);
      double y = 0.0;
      for (int64_t n = 0; n < N; ++n) {
        const double a = exp(dtv * (double)A[d * N + n]);
        const double s = state[idx * N + n] * a +
                         dtv * (double)x[idx] * (double)B[(b * ngroups + g) * N + n];
        state[idx * N + n] = s;
        y += s * (double)C[(b * ngroups + g) * N + n];
      }
      if (D) y += (double)x[idx] * (double)D[d];
      if (z) y *= (double)z[idx] * sigmoid_d((double)z[idx]);
      out[idx] = y;
    }
  }
}

/* causal_conv1d.py:56-85: conv_state (b,d,S) with S >= W-1 is rolled in place by seqlen
 * steps; out (b,d,seqlen). */
void oracle_conv1d_update(const float* x, double* conv_state, const float* w, const float* bias,
                          double* out, int64_t batch, int64_t dim, int64_t seqlen,
                          int64_t state_len, int64_t width, int silu) {
  const int64_t S = state_len, L = seqlen, W = width;
  double* full = (double*)malloc(sizeof(double) * (size_t)(S + L));
  for (int64_t idx = 0; idx < batch * dim; ++idx) {
    const int64_t d = idx % dim;
    for (int64_t j = 0; j < S; ++j) full[j] = conv_state[idx * S + j];
    for (int64_t t = 0; t < L; ++t) full[S + t] = (double)x[idx * L + t];
    for (int64_t t = 0; t < L; ++t) {
      double acc = bias ? (double)bias[d] : 0.0;
      for (int64_t k = 0; k < W; ++k) acc += (double)w[d * W + k] * full[S + t - (W - 1) + k];
      out[idx * L + t] = act_fwd(acc, silu);
    }
    for (int64_t j = 0; j < S; ++j) conv_state[idx * S + j] = full[L + j];
  }
  free(full);
}


/* ---- Mamba-2 SSD scan (forward) ----------------------------------------------------------
 * The reference has no SSD implementation (README.md:94 lists it as a roadmap item). This is
 * the recurrence of upstream mamba_ssm's mamba_chunk_scan_combined stated step by step, which
 * is the reference's Mamba-1 recurrence (csrc/selective_scan.cpp:120-145) with channels =
 * nheads * headdim, A[h] shared by all dstate entries and dt[b, t, h] shared by the head's
 * headdim channels:
 *   dt_t = clamp(softplus?(dt + dt_bias[h]), dt_min, dt_max)
 *   s[p][n] = exp(dt_t A[h]) s[p][n] + dt_t x[p] B[n];  y[p] = sum_n s[p][n] C[n] + D x[p];
 *   out = y * silu(z).
 * Layouts (dense): x, z, out (b, l, h, p); dt (b, l, h); B, C (b, l, g, n); D (h) or (h, p)
 * (D_per_dim); initial / final states (b, h, p, n); seq_idx (b, l) int32 or NULL. Head h reads
 * group h / (h_total / g). With seq_idx (packed sequences) the state restarts from zero wherever
 * the sequence id changes; the initial state belongs to sequence 0, as in upstream's
 * _state_passing_fwd. */
typedef struct {
  const float *x, *dt, *A, *B, *C, *D, *z, *dt_bias, *init;
  const int32_t* seq_idx;
  double *out, *final_states;
  int64_t batch, seqlen, nheads, headdim, ngroups, dstate;
  int softplus, D_per_dim;
  double dt_min, dt_max;
} ssd_ctx;

static void ssd_rows(int64_t lo, int64_t hi, void* vctx) {
  const ssd_ctx* c = (const ssd_ctx*)vctx;
  const int64_t L = c->seqlen, H = c->nheads, P = c->headdim, G = c->ngroups, N = c->dstate;
  double* s = (double*)malloc(sizeof(double) * (size_t)(P * N));
  for (int64_t r = lo; r < hi; ++r) { /* r = b * H + h */
    const int64_t b = r / H, h = r % H, g = h / (H / G);
    for (int64_t i = 0; i < P * N; ++i) s[i] = c->init ? (double)c->init[r * P * N + i] : 0.0;
    const double A = (double)c->A[h];
    int32_t seq_prev = 0; /* the initial state belongs to sequence 0 */
    for (int64_t t = 0; t < L; ++t) {
      if (c->seq_idx) { /* packed sequences: the state restarts where the sequence id changes */
        const int32_t sq = c->seq_idx[b * L + t];
        if (sq != seq_prev)
          for (int64_t i = 0; i < P * N; ++i) s[i] = 0.0;
        seq_prev = sq;
      }
      double dt = (double)c->dt[(b * L + t) * H + h] + (c->dt_bias ? (double)c->dt_bias[h] : 0.0);
      if (c->softplus) dt = softplus_d(dt);
      dt = fmin(fmax(dt, c->dt_min), c->dt_max);
      const double decay = exp(dt * A);
      const float* Bt = c->B + ((b * L + t) * G + g) * N;
      const float* Ct = c->C + ((b * L + t) * G + g) * N;
      const int64_t row = ((b * L + t) * H + h) * P;
      for (int64_t p = 0; p < P; ++p) {
        const double xv = (double)c->x[row + p];
        double y = 0.0;
        for (int64_t n = 0; n < N; ++n) {
          double* sp = &s[p * N + n];
          *sp = decay * *sp + dt * xv * (double)Bt[n];
          y += *sp * (double)Ct[n];
        }
        if (c->D) y += xv * (double)(c->D_per_dim ? c->D[h * P + p] : c->D[h]);
        if (c->z) {
          const double zv = (double)c->z[row + p];
          y *= zv * sigmoid_d(zv);
        }
        c->out[row + p] = y;
      }
    }
    if (c->final_states)
      for (int64_t i = 0; i < P * N; ++i) c->final_states[r * P * N + i] = s[i];
  }
  free(s);
}

int oracle_ssd_fwd(const float* x, const float* dt, const float* A, const float* B, const float* C,
                   const float* D, const float* z, const float* dt_bias, const float* init,
                   const int32_t* seq_idx, double* out, double* final_states, int64_t batch, int64_t seqlen,
                   int64_t nheads, int64_t headdim, int64_t ngroups, int64_t dstate, int softplus,
                   double dt_min, double dt_max, int D_per_dim) {
  if (!x || !dt || !A || !B || !C || !out) return 1;
  if (batch < 0 || seqlen < 0 || nheads < 0 || headdim <= 0 || ngroups <= 0 || dstate <= 0) return 2;
  if (nheads % ngroups != 0) return 2;
  ssd_ctx c = {x, dt, A, B, C, D, z, dt_bias, init, seq_idx, out, final_states, batch, seqlen, nheads,
               headdim, ngroups, dstate, softplus, D_per_dim, dt_min, dt_max};
  parallel_for(batch * nheads, ssd_rows, &c);
  return 0;
}
