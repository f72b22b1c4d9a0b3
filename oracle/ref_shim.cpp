// ref_shim.cpp -- a plain C entry point around the reference's own CPU kernel, so the
// unmodified reference C++ code (csrc/selective_scan.cpp of SandyTheAdventurer/mamba-cpu)
// can be loaded through ctypes without nanobind (which is not installed here).
//
// TEST INFRASTRUCTURE: compiled by oracle/Makefile into oracle/_ref/ together with the
// reference's selective_scan.cpp, read from where it lies. Used to pin the float64 oracle,
// to generate golden fixtures, and as the timed CPU baseline. Never part of the product.
//
// Each function mirrors one nanobind binding of csrc/bindings.cpp and forwards to the
// reference's entry points declared in csrc/selective_scan.h:
//   ref_cpu_isa / ref_set_cpu_isa   <- bindings.cpp:20-21 (selective_scan.h:11-12)
//   ref_selective_scan_fwd_f32      <- bindings.cpp:23-45 (selective_scan.h:21-40)
//   ref_selective_scan_bwd_f32      <- bindings.cpp:47-84 (selective_scan.h:51-65)
#include <cstdint>
#include <string>

#include "selective_scan.h"

extern "C" {

const char* ref_cpu_isa() { return mamba_cpu::cpu_isa(); }

int ref_set_cpu_isa(const char* name) { return mamba_cpu::set_cpu_isa(std::string(name)) ? 1 : 0; }

void ref_selective_scan_fwd_f32(const float* u, const float* delta, const float* A, const float* B,
                                const float* C, const float* D, const float* z,
                                const float* delta_bias, float* out, float* last_state,
                                int64_t batch, int64_t dim, int64_t seqlen, int64_t dstate,
                                int64_t ngroups, int delta_softplus, int num_threads) {
  mamba_cpu::SelectiveScanParams p;
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
  p.batch = batch;
  p.dim = dim;
  p.seqlen = seqlen;
  p.dstate = dstate;
  p.ngroups = ngroups;
  p.delta_softplus = delta_softplus != 0;
  mamba_cpu::selective_scan_fwd_f32(p, num_threads);
}

void ref_selective_scan_bwd_f32(const float* u, const float* delta, const float* A, const float* B,
                                const float* C, const float* D, const float* z,
                                const float* delta_bias, const float* dout,
                                const float* dlast_state, float* du, float* ddelta, float* dA_part,
                                float* dB, float* dC, float* dD_part, float* dz,
                                float* ddelta_bias_part, int64_t batch, int64_t dim,
                                int64_t seqlen, int64_t dstate, int64_t ngroups,
                                int delta_softplus, int num_threads) {
  mamba_cpu::SelectiveScanBwdParams p;
  p.fwd.u = u;
  p.fwd.delta = delta;
  p.fwd.A = A;
  p.fwd.B = B;
  p.fwd.C = C;
  p.fwd.D = D;
  p.fwd.z = z;
  p.fwd.delta_bias = delta_bias;
  p.fwd.out = nullptr;
  p.fwd.last_state = nullptr;
  p.fwd.batch = batch;
  p.fwd.dim = dim;
  p.fwd.seqlen = seqlen;
  p.fwd.dstate = dstate;
  p.fwd.ngroups = ngroups;
  p.fwd.delta_softplus = delta_softplus != 0;
  p.dout = dout;
  p.dlast_state = dlast_state;
  p.du = du;
  p.ddelta = ddelta;
  p.dA_part = dA_part;
  p.dB = dB;
  p.dC = dC;
  p.dD_part = dD_part;
  p.dz = dz;
  p.ddelta_bias_part = ddelta_bias_part;
  mamba_cpu::selective_scan_bwd_f32(p, num_threads);
}

}  // extern "C"
