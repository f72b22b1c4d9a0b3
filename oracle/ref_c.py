"""The reference's own CPU kernel behind its original Python-level interface. TEST INFRASTRUCTURE.

``oracle/_ref/libmamba_cpu_ref.so`` is mamba-cpu's ``csrc/selective_scan.cpp`` compiled unmodified
(see ``oracle/Makefile``) plus a plain ``extern "C"`` shim (``ref_shim.cpp``). This module exposes
the functions of the reference's nanobind module ``mamba_cpu._C`` (``csrc/bindings.cpp:18-85``)
with the same names and arguments -- uintptr data pointers, 0 for None -- so it can

* stand in for ``mamba_cpu._C`` when the unmodified reference package is imported in the build
  container (``tests/golden/make_golden.py`` does that to produce the committed fixtures), and
* be timed as the reference CPU baseline (``bench.py``), with the reference's own threading.
"""

import ctypes

from . import LIB_REF, ref_available

_lib = None
_P = ctypes.c_void_p
_I = ctypes.c_int64


def _load():
    global _lib
    if _lib is None:
        if not ref_available():
            raise RuntimeError(f"reference kernel not built: {LIB_REF} (run `make -C oracle ref`)")
        lib = ctypes.CDLL(LIB_REF)
        lib.ref_cpu_isa.restype = ctypes.c_char_p
        lib.ref_set_cpu_isa.argtypes = [ctypes.c_char_p]
        lib.ref_set_cpu_isa.restype = ctypes.c_int
        lib.ref_selective_scan_fwd_f32.argtypes = [_P] * 10 + [_I] * 5 + [ctypes.c_int, ctypes.c_int]
        lib.ref_selective_scan_fwd_f32.restype = None
        lib.ref_selective_scan_bwd_f32.argtypes = [_P] * 18 + [_I] * 5 + [ctypes.c_int, ctypes.c_int]
        lib.ref_selective_scan_bwd_f32.restype = None
        _lib = lib
    return _lib


def _p(x):
    return None if not x else ctypes.c_void_p(int(x))


# --- the reference's _C interface (bindings.cpp:20-84) ------------------------------------

def cpu_isa() -> str:
    return _load().ref_cpu_isa().decode()


def set_cpu_isa(name: str) -> bool:
    return bool(_load().ref_set_cpu_isa(name.encode()))


def selective_scan_fwd_f32(u, delta, A, B, C, D, z, delta_bias, out, last_state, batch, dim,
                           seqlen, dstate, ngroups, delta_softplus, num_threads):
    _load().ref_selective_scan_fwd_f32(
        _p(u), _p(delta), _p(A), _p(B), _p(C), _p(D), _p(z), _p(delta_bias), _p(out),
        _p(last_state), batch, dim, seqlen, dstate, ngroups, int(bool(delta_softplus)),
        int(num_threads))


def selective_scan_bwd_f32(u, delta, A, B, C, D, z, delta_bias, dout, dlast_state, du, ddelta,
                           dA_part, dB, dC, dD_part, dz, ddelta_bias_part, batch, dim, seqlen,
                           dstate, ngroups, delta_softplus, num_threads):
    _load().ref_selective_scan_bwd_f32(
        _p(u), _p(delta), _p(A), _p(B), _p(C), _p(D), _p(z), _p(delta_bias), _p(dout),
        _p(dlast_state), _p(du), _p(ddelta), _p(dA_part), _p(dB), _p(dC), _p(dD_part), _p(dz),
        _p(ddelta_bias_part), batch, dim, seqlen, dstate, ngroups, int(bool(delta_softplus)),
        int(num_threads))


def as_module():
    """A module object with the reference ``_C`` surface, for ``sys.modules['mamba_cpu._C']``."""
    import types

    m = types.ModuleType("mamba_cpu._C")
    m.__doc__ = "mamba_cpu native kernels (reference C++ via a ctypes shim)"
    for name in ("cpu_isa", "set_cpu_isa", "selective_scan_fwd_f32", "selective_scan_bwd_f32"):
        setattr(m, name, globals()[name])
    return m
