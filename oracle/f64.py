"""ctypes wrapper of the float64 C restatement (``oracle.c``). TEST INFRASTRUCTURE ONLY.

Every function takes numpy arrays (any float dtype; they are converted to contiguous float32,
exactly the values the GPU kernels see) and returns float64 numpy arrays. B and C are in the
upstream (batch, ngroups, dstate, seqlen) layout; 3-D (batch, dstate, seqlen) is taken as
ngroups = 1, as the reference's ``_as_kernel_bc`` does (selective_scan_interface.py:131-135).
"""

import ctypes

import numpy as np

from . import ensure_f64

_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int64


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(ensure_f64())
        lib.oracle_scan_fwd.argtypes = [_P] * 10 + [_I] * 5 + [ctypes.c_int]
        lib.oracle_scan_fwd.restype = ctypes.c_int
        lib.oracle_scan_bwd.argtypes = [_P] * 18 + [_I] * 5 + [ctypes.c_int]
        lib.oracle_scan_bwd.restype = ctypes.c_int
        lib.oracle_scan_fwd_init.argtypes = [_P] * 11 + [_I] * 5 + [ctypes.c_int]
        lib.oracle_scan_fwd_init.restype = ctypes.c_int
        lib.oracle_scan_bwd_init.argtypes = [_P] * 20 + [_I] * 5 + [ctypes.c_int]
        lib.oracle_scan_bwd_init.restype = ctypes.c_int
        lib.oracle_conv1d_fwd.argtypes = [_P] * 6 + [_I] * 4 + [ctypes.c_int]
        lib.oracle_conv1d_fwd.restype = ctypes.c_int
        lib.oracle_conv1d_bwd.argtypes = [_P] * 9 + [_I] * 4 + [ctypes.c_int]
        lib.oracle_conv1d_bwd.restype = ctypes.c_int
        lib.oracle_state_update.argtypes = [_P] * 10 + [_I] * 4 + [ctypes.c_int]
        lib.oracle_state_update.restype = None
        lib.oracle_conv1d_update.argtypes = [_P] * 5 + [_I] * 5 + [ctypes.c_int]
        lib.oracle_conv1d_update.restype = None
        lib.oracle_ssd_fwd.argtypes = [_P] * 12 + [_I] * 6 + [ctypes.c_int, ctypes.c_double, ctypes.c_double,
                                                                ctypes.c_int]
        lib.oracle_ssd_fwd.restype = ctypes.c_int
        lib.oracle_set_num_threads.argtypes = [ctypes.c_int]
        lib.oracle_num_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def set_num_threads(n: int) -> None:
    _load().oracle_set_num_threads(int(n))


def num_threads() -> int:
    return _load().oracle_num_threads()


def _f32(x):
    if x is None:
        return None
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().float().cpu().numpy()
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _bc(X):
    X = _f32(X)
    return X[:, None] if X.ndim == 3 else X


def scan_fwd(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False, initial_state=None):
    """Returns (out, last_state) in float64. initial_state (batch, dim, dstate): the state before
    the first step (zeros when None)."""
    u, delta, A, D, z, delta_bias, h0 = map(_f32, (u, delta, A, D, z, delta_bias, initial_state))
    B, C = _bc(B), _bc(C)
    batch, dim, seqlen = u.shape
    ngroups, dstate = B.shape[1], B.shape[2]
    out = np.empty((batch, dim, seqlen), np.float64)
    last = np.empty((batch, dim, dstate), np.float64)
    rc = _load().oracle_scan_fwd_init(
        _ptr(u), _ptr(delta), _ptr(A), _ptr(B), _ptr(C), _ptr(D), _ptr(z), _ptr(delta_bias), _ptr(h0),
        _ptr(out), _ptr(last), batch, dim, seqlen, dstate, ngroups, int(bool(delta_softplus)))
    if rc:
        raise ValueError(f"oracle_scan_fwd rejected its arguments (status {rc})")
    return out, last


def scan_bwd(u, delta, A, B, C, D, z, delta_bias, delta_softplus, dout, dlast_state=None, initial_state=None):
    """Returns a dict with du, ddelta, dA, dB, dC, dD, dz (None without z), ddelta_bias and
    dinitial_state (the gradient with respect to initial_state, (batch, dim, dstate)).

    dA/dD/ddelta_bias are summed over batch (selective_scan_interface.py:87); dB/dC have B's
    (batch, ngroups, dstate, seqlen) shape (3-D B gives a 4-D result with ngroups = 1)."""
    u, delta, A, D, z, delta_bias, dout, dlast_state, h0 = map(
        _f32, (u, delta, A, D, z, delta_bias, dout, dlast_state, initial_state))
    B, C = _bc(B), _bc(C)
    batch, dim, seqlen = u.shape
    ngroups, dstate = B.shape[1], B.shape[2]
    du = np.empty_like(u, dtype=np.float64)
    ddelta = np.empty_like(u, dtype=np.float64)
    dz = np.empty_like(u, dtype=np.float64) if z is not None else None
    dA = np.empty((dim, dstate), np.float64)
    dB = np.empty(B.shape, np.float64)
    dC = np.empty(C.shape, np.float64)
    dD = np.empty((dim,), np.float64)
    db = np.empty((dim,), np.float64)
    dh0 = np.empty((batch, dim, dstate), np.float64)
    rc = _load().oracle_scan_bwd_init(
        _ptr(u), _ptr(delta), _ptr(A), _ptr(B), _ptr(C), _ptr(D), _ptr(z), _ptr(delta_bias), _ptr(h0),
        _ptr(dout), _ptr(dlast_state), _ptr(du), _ptr(ddelta), _ptr(dA), _ptr(dB), _ptr(dC),
        _ptr(dD), _ptr(dz), _ptr(db), _ptr(dh0), batch, dim, seqlen, dstate, ngroups,
        int(bool(delta_softplus)))
    if rc:
        raise ValueError(f"oracle_scan_bwd rejected its arguments (status {rc})")
    return dict(du=du, ddelta=ddelta, dA=dA, dB=dB, dC=dC, dD=dD, dz=dz, ddelta_bias=db, dinitial_state=dh0)


def conv1d_fwd(x, weight, bias=None, initial_states=None, activation=None, return_final_states=False):
    x, w, bias, init = map(_f32, (x, weight, bias, initial_states))
    batch, dim, seqlen = x.shape
    width = w.shape[1]
    out = np.empty((batch, dim, seqlen), np.float64)
    fin = np.empty((batch, dim, width - 1), np.float64) if return_final_states else None
    rc = _load().oracle_conv1d_fwd(_ptr(x), _ptr(w), _ptr(bias), _ptr(init), _ptr(out), _ptr(fin),
                                   batch, dim, seqlen, width, int(activation in ("silu", "swish")))
    if rc:
        raise ValueError(f"oracle_conv1d_fwd rejected its arguments (status {rc})")
    return (out, fin) if return_final_states else out


def conv1d_bwd(x, weight, bias, initial_states, activation, dout):
    """Returns dict(dx, dweight, dbias, dinitial_states) in float64."""
    x, w, bias, init, dout = map(_f32, (x, weight, bias, initial_states, dout))
    batch, dim, seqlen = x.shape
    width = w.shape[1]
    dx = np.empty_like(x, dtype=np.float64)
    dw = np.empty_like(w, dtype=np.float64)
    db = np.empty((dim,), np.float64) if bias is not None else None
    dinit = np.empty((batch, dim, width - 1), np.float64) if init is not None else None
    rc = _load().oracle_conv1d_bwd(_ptr(x), _ptr(w), _ptr(bias), _ptr(init), _ptr(dout), _ptr(dx),
                                   _ptr(dw), _ptr(db), _ptr(dinit), batch, dim, seqlen, width,
                                   int(activation in ("silu", "swish")))
    if rc:
        raise ValueError(f"oracle_conv1d_bwd rejected its arguments (status {rc})")
    return dict(dx=dx, dweight=dw, dbias=db, dinitial_states=dinit)


def state_update(state, x, dt, A, B, C, D=None, z=None, dt_bias=None, dt_softplus=False):
    """Mamba-1 layout decode step. Returns (out, new_state) in float64; `state` is not modified."""
    st = np.array(_f32(state), dtype=np.float64, copy=True)
    x, dt, A, B, C, D, z, dt_bias = map(_f32, (x, dt, A, B, C, D, z, dt_bias))
    if B.ndim == 2:
        B, C = B[:, None], C[:, None]
    batch, dim = x.shape
    ngroups, dstate = B.shape[1], B.shape[2]
    out = np.empty((batch, dim), np.float64)
    _load().oracle_state_update(_ptr(st), _ptr(x), _ptr(dt), _ptr(A), _ptr(B), _ptr(C), _ptr(D),
                                _ptr(z), _ptr(dt_bias), _ptr(out), batch, dim, dstate, ngroups,
                                int(bool(dt_softplus)))
    return out, st


def conv1d_update(x, conv_state, weight, bias=None, activation=None):
    """Returns (out, new_conv_state) in float64; x is (b,d) or (b,d,l)."""
    single = np.ndim(x) == 2
    x = _f32(x)
    if single:
        x = x[..., None]
    st = np.array(_f32(conv_state), dtype=np.float64, copy=True)
    w, bias = _f32(weight), _f32(bias)
    batch, dim, seqlen = x.shape
    out = np.empty((batch, dim, seqlen), np.float64)
    _load().oracle_conv1d_update(_ptr(np.ascontiguousarray(x)), _ptr(st), _ptr(w), _ptr(bias),
                                 _ptr(out), batch, dim, seqlen, st.shape[-1], w.shape[1],
                                 int(activation in ("silu", "swish")))
    return (out[..., 0] if single else out), st


def ssd_fwd(x, dt, A, B, C, D=None, z=None, dt_bias=None, initial_states=None, dt_softplus=False,
            dt_limit=(0.0, float("inf")), seq_idx=None):
    """Mamba-2 SSD scan, step by step in float64. x, z (b, l, h, p); dt (b, l, h); A, dt_bias (h);
    B, C (b, l, g, n); D (h) or (h, p); initial_states (b, h, p, n); seq_idx (b, l) packed sequence
    ids (the state restarts where the id changes). Returns (out, final_states)."""
    x, dt, A, B, C, D, z, dt_bias, init = map(_f32, (x, dt, A, B, C, D, z, dt_bias, initial_states))
    if seq_idx is not None:
        if hasattr(seq_idx, "detach"):
            seq_idx = seq_idx.detach().cpu().numpy()
        seq_idx = np.ascontiguousarray(np.asarray(seq_idx, dtype=np.int32))
    batch, seqlen, nheads, headdim = x.shape
    ngroups, dstate = B.shape[2], B.shape[3]
    out = np.empty(x.shape, np.float64)
    fin = np.empty((batch, nheads, headdim, dstate), np.float64)
    rc = _load().oracle_ssd_fwd(
        _ptr(x), _ptr(dt), _ptr(A), _ptr(B), _ptr(C), _ptr(D), _ptr(z), _ptr(dt_bias), _ptr(init), _ptr(seq_idx),
        _ptr(out), _ptr(fin), batch, seqlen, nheads, headdim, ngroups, dstate, int(bool(dt_softplus)),
        float(dt_limit[0]), float(dt_limit[1]), int(D is not None and D.ndim == 2))
    if rc:
        raise ValueError(f"oracle_ssd_fwd rejected its arguments (status {rc})")
    return out, fin
