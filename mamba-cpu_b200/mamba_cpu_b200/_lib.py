"""ctypes binding of libmamba_b200.so (the C ABI declared in include/mamba_b200.h).

This is the Python side of the drop-in boundary: it plays the role of the reference's nanobind
module ``mamba_cpu._C`` (csrc/bindings.cpp) -- tensors cross as raw data pointers, with ``None``
as NULL -- but targets the CUDA library and passes the current CUDA stream instead of a thread
count. ctypes releases the GIL around every call, like ``nb::gil_scoped_release`` does there.

There is no fallback: if the shared library is missing or cannot be loaded, importing the
package raises, so a CUDA tensor can never silently take another path.
"""

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("MAMBA_B200_LIB", os.path.join(_HERE, "_lib", "libmamba_b200.so"))

F32, BF16, F16 = 0, 1, 2
MAX_DSTATE = 16
DECODE_MAX_DSTATE = 256
CHUNK = 64
CONV_MAX_WIDTH = 8

_DTYPE_CODE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

OK = 0
_STATUS_EXC = {
    1: ValueError,  # NULL pointer
    2: ValueError,  # bad shape
    3: TypeError,  # bad dtype
    4: ValueError,  # bad layout
    5: NotImplementedError,
    6: RuntimeError,  # workspace
    7: RuntimeError,  # CUDA
    8: ValueError,  # exceeds the no-allocation entry point's static scratch
}

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32


class ScanFwdParams(ctypes.Structure):
    _fields_ = [
        ("u", _vp), ("delta", _vp), ("A", _vp), ("B", _vp), ("C", _vp), ("D", _vp), ("z", _vp),
        ("delta_bias", _vp), ("out", _vp), ("last_state", _vp), ("chunk_states", _vp), ("initial_state", _vp),
        ("batch", _i64), ("dim", _i64), ("seqlen", _i64), ("dstate", _i64), ("ngroups", _i64),
        ("B_batch_stride", _i64), ("B_group_stride", _i64), ("B_dstate_stride", _i64),
        ("B_seqlen_stride", _i64),
        ("C_batch_stride", _i64), ("C_group_stride", _i64), ("C_dstate_stride", _i64),
        ("C_seqlen_stride", _i64),
        ("io_dtype", _i32), ("bc_dtype", _i32), ("delta_softplus", _i32), ("reserved", _i32),
        ("u_batch_stride", _i64), ("u_dim_stride", _i64), ("delta_batch_stride", _i64),
        ("delta_dim_stride", _i64), ("z_batch_stride", _i64), ("z_dim_stride", _i64),
    ]


class ScanBwdParams(ctypes.Structure):
    _fields_ = [
        ("fwd", ScanFwdParams),
        ("dout", _vp), ("dlast_state", _vp), ("du", _vp), ("ddelta", _vp), ("dz", _vp), ("dA", _vp),
        ("dB", _vp), ("dC", _vp), ("dD", _vp), ("ddelta_bias", _vp), ("dinitial_state", _vp),
        ("dbc_dtype", _i32), ("reserved", _i32),
    ]


class Conv1dParams(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("weight", _vp), ("bias", _vp), ("initial_states", _vp), ("out", _vp),
        ("final_states", _vp),
        ("batch", _i64), ("dim", _i64), ("seqlen", _i64), ("width", _i64),
        ("x_dtype", _i32), ("activation", _i32),
    ]


class StateUpdateParams(ctypes.Structure):
    _fields_ = [
        ("state", _vp), ("x", _vp), ("dt", _vp), ("A", _vp), ("B", _vp), ("C", _vp), ("D", _vp),
        ("z", _vp), ("dt_bias", _vp), ("out", _vp),
        ("batch", _i64), ("dim", _i64), ("dstate", _i64), ("ngroups", _i64),
        ("io_dtype", _i32), ("bc_dtype", _i32), ("state_dtype", _i32), ("dt_softplus", _i32),
    ]


class Conv1dUpdateParams(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("conv_state", _vp), ("weight", _vp), ("bias", _vp), ("out", _vp),
        ("batch", _i64), ("dim", _i64), ("seqlen", _i64), ("state_len", _i64), ("width", _i64),
        ("x_dtype", _i32), ("activation", _i32),
    ]


class SsdParams(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("dt", _vp), ("A", _vp), ("B", _vp), ("C", _vp), ("D", _vp), ("z", _vp),
        ("dt_bias", _vp), ("initial_states", _vp), ("out", _vp), ("final_states", _vp),
        ("batch", _i64), ("seqlen", _i64), ("nheads", _i64), ("headdim", _i64), ("ngroups", _i64),
        ("dstate", _i64),
        ("x_batch_stride", _i64), ("x_seqlen_stride", _i64), ("x_head_stride", _i64),
        ("z_batch_stride", _i64), ("z_seqlen_stride", _i64), ("z_head_stride", _i64),
        ("B_batch_stride", _i64), ("B_seqlen_stride", _i64), ("B_group_stride", _i64),
        ("C_batch_stride", _i64), ("C_seqlen_stride", _i64), ("C_group_stride", _i64),
        ("dt_batch_stride", _i64), ("dt_seqlen_stride", _i64),
        ("seq_idx", _vp), ("seq_idx_batch_stride", _i64), ("seq_idx_seqlen_stride", _i64),
        ("dt_min", ctypes.c_float), ("dt_max", ctypes.c_float),
        ("x_dtype", _i32), ("dt_softplus", _i32), ("D_per_dim", _i32), ("reserved", _i32),
    ]


# Every entry point of include/mamba_b200.h with its ctypes signature.
SIGNATURES = {
    "mb200_selective_scan_fwd": ([ctypes.POINTER(ScanFwdParams), _vp], ctypes.c_int),
    "mb200_selective_scan_fwd_workspace_size": ([ctypes.POINTER(ScanFwdParams)], ctypes.c_size_t),
    "mb200_selective_scan_fwd_ws": ([ctypes.POINTER(ScanFwdParams), _vp, ctypes.c_size_t, _vp], ctypes.c_int),
    "mb200_set_sequence_pieces": ([ctypes.c_int], None),
    "mb200_sequence_pieces": ([_i64, ctypes.c_int, ctypes.c_int], ctypes.c_int),
    "mb200_selective_scan_bwd_workspace_size": ([ctypes.POINTER(ScanBwdParams)], ctypes.c_size_t),
    "mb200_selective_scan_bwd": ([ctypes.POINTER(ScanBwdParams), _vp, ctypes.c_size_t, _vp], ctypes.c_int),
    "mb200_selective_scan_bwd_noalloc": ([ctypes.POINTER(ScanBwdParams), _vp], ctypes.c_int),
    "mb200_selective_scan_fwd_f32": ([_vp] * 10 + [_i64] * 5 + [ctypes.c_int, _vp], ctypes.c_int),
    "mb200_selective_scan_bwd_f32": ([_vp] * 18 + [_i64] * 5 + [ctypes.c_int, _vp], ctypes.c_int),
    "mb200_causal_conv1d_fwd": ([ctypes.POINTER(Conv1dParams), _vp], ctypes.c_int),
    "mb200_causal_conv1d_bwd_workspace_size": ([ctypes.POINTER(Conv1dParams)], ctypes.c_size_t),
    "mb200_causal_conv1d_bwd": ([ctypes.POINTER(Conv1dParams), _vp, _vp, _vp, _vp, _vp, _vp,
                                 ctypes.c_size_t, _vp], ctypes.c_int),
    "mb200_selective_state_update": ([ctypes.POINTER(StateUpdateParams), _vp], ctypes.c_int),
    "mb200_causal_conv1d_update": ([ctypes.POINTER(Conv1dUpdateParams), _vp], ctypes.c_int),
    "mb200_ssd_chunk_scan_fwd": ([ctypes.POINTER(SsdParams), _vp], ctypes.c_int),
    "mb200_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "mb200_version": ([], ctypes.c_int),
    "mb200_last_launch_count": ([], ctypes.c_int),
    "mb200_device_fault": ([ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "mb200_peer_alloc": ([ctypes.c_size_t, ctypes.POINTER(_vp)], ctypes.c_int),
    "mb200_peer_free": ([_vp], ctypes.c_int),
    "mb200_ipc_handle": ([_vp, ctypes.POINTER(ctypes.c_ubyte)], ctypes.c_int),
    "mb200_ipc_open": ([ctypes.POINTER(ctypes.c_ubyte), ctypes.POINTER(_vp)], ctypes.c_int),
    "mb200_ipc_close": ([_vp], ctypes.c_int),
    "mb200_peer_sum_f32": ([_vp, _i64, _vp, _i64, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _i64, _vp],
                           ctypes.c_int),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libmamba_b200.so not found at {LIB_PATH}; build it with `make -C mamba-cpu_b200` "
            "(or __graft_entry__.build()). There is no non-CUDA fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


lib = _load()


def set_sequence_pieces(pieces: int) -> None:
    """Force the number of sequence pieces per row of the scan kernels (0: automatic, the default).
    The automatic choice splits rows only when whole rows leave most of the GPU idle."""
    lib.mb200_set_sequence_pieces(int(pieces))


def status_string(status: int) -> str:
    return lib.mb200_status_string(status).decode()


def check(status: int, what: str) -> None:
    if status != OK:
        exc = _STATUS_EXC.get(status, RuntimeError)
        raise exc(f"{what}: {status_string(status)} (status {status})")


def device_fault() -> int:
    """Read and clear the kernels' device-side fault word (0 = none). Synchronises the device."""
    v = ctypes.c_int(0)
    check(lib.mb200_device_fault(ctypes.byref(v)), "mb200_device_fault")
    return v.value


def last_launch_count() -> int:
    return lib.mb200_last_launch_count()


def ptr(t):
    return None if t is None else t.data_ptr()


def dtype_code(dtype) -> int:
    return _DTYPE_CODE[dtype]


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream
