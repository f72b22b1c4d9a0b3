"""Mamba-2 SSD chunk scan (forward) on B200 tensor cores.

The reference lists the Mamba-2 SSD scan as a roadmap item (mamba-cpu README.md:94) and has no
implementation of it. ``mamba_chunk_scan_combined`` here takes the arguments of upstream
mamba_ssm's function of that name (mamba_ssm/ops/triton/ssd_combined.py, mamba_ssm 2.x) and
computes the same recurrence: per (batch, head) a headdim x dstate state with one scalar decay
per step,

    dt_t = clamp(softplus?(dt[b, t, h] + dt_bias[h]), *dt_limit)
    h_t  = exp(dt_t A[h]) h_{t-1} + dt_t x_t B_t^T,   y_t = h_t C_t + D x_t,   out = y * silu(z).

This is the Mamba-1 selective scan of ``selective_scan_fn`` with channels = nheads * headdim, A
broadcast over dstate and delta broadcast over headdim, which is how the tests pin it to the
reference's own kernel. The work runs in one sm_100a kernel (``mb200_ssd_chunk_scan_fwd`` in
libmamba_b200.so): 64-step chunks as tcgen05 matrix products, the state carried in float32.
"""

import math
from typing import Optional, Tuple

import torch

from .. import _lib


def _rows16(t: torch.Tensor) -> torch.Tensor:
    """The tensor itself when its last dimension is contiguous and every other stride and the
    base address are 16-byte multiples (what the kernel's 16-byte row pieces need); else a
    contiguous copy."""
    es = t.element_size()
    ok = t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and all((s * es) % 16 == 0 for s in t.stride()[:-1])
    return t if ok else t.contiguous()


@torch.library.custom_op("mamba_b200::ssd_chunk_scan_fwd", mutates_args=(), device_types="cuda")
def _ssd_chunk_scan_fwd(
    x: torch.Tensor,
    dt: torch.Tensor,
    A: torch.Tensor,
    B: torch.Tensor,
    C: torch.Tensor,
    D: Optional[torch.Tensor],
    z: Optional[torch.Tensor],
    dt_bias: Optional[torch.Tensor],
    initial_states: Optional[torch.Tensor],
    seq_idx: Optional[torch.Tensor],
    dt_softplus: bool,
    dt_min: float,
    dt_max: float,
    want_final: bool,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """x, z (b, l, h, p) bf16 with 16-byte rows; dt (b, l, h) f32 (h contiguous); A, dt_bias (h)
    f32; B, C (b, l, g, n) bf16 with 16-byte rows; D (h) or (h, p) f32; initial_states (b, h, p, n)
    f32; seq_idx (b, l) int32 or None. Returns out (b, l, h, p) and final_states (b, h, p, n)
    (empty unless want_final)."""
    b, l, h, p = x.shape
    g, n = B.shape[2], B.shape[3]
    out = torch.empty((b, l, h, p), dtype=x.dtype, device=x.device)
    final = torch.empty((b, h, p, n) if want_final else (0,), dtype=torch.float32, device=x.device)
    prm = _lib.SsdParams()
    prm.x, prm.dt, prm.A, prm.B, prm.C = _lib.ptr(x), _lib.ptr(dt), _lib.ptr(A), _lib.ptr(B), _lib.ptr(C)
    prm.D, prm.z, prm.dt_bias = _lib.ptr(D), _lib.ptr(z), _lib.ptr(dt_bias)
    prm.initial_states, prm.out = _lib.ptr(initial_states), _lib.ptr(out)
    prm.final_states = _lib.ptr(final) if want_final else None
    prm.batch, prm.seqlen, prm.nheads, prm.headdim, prm.ngroups, prm.dstate = b, l, h, p, g, n
    prm.x_batch_stride, prm.x_seqlen_stride, prm.x_head_stride = x.stride(0), x.stride(1), x.stride(2)
    if z is not None:
        prm.z_batch_stride, prm.z_seqlen_stride, prm.z_head_stride = z.stride(0), z.stride(1), z.stride(2)
    prm.B_batch_stride, prm.B_seqlen_stride, prm.B_group_stride = B.stride(0), B.stride(1), B.stride(2)
    prm.C_batch_stride, prm.C_seqlen_stride, prm.C_group_stride = C.stride(0), C.stride(1), C.stride(2)
    prm.dt_batch_stride, prm.dt_seqlen_stride = dt.stride(0), dt.stride(1)
    if seq_idx is not None:
        prm.seq_idx = _lib.ptr(seq_idx)
        prm.seq_idx_batch_stride, prm.seq_idx_seqlen_stride = seq_idx.stride(0), seq_idx.stride(1)
    prm.dt_min, prm.dt_max = float(dt_min), float(dt_max)
    prm.x_dtype = _lib.dtype_code(x.dtype)
    prm.dt_softplus = int(bool(dt_softplus))
    prm.D_per_dim = int(D is not None and D.dim() == 2)
    with torch.cuda.device(x.device):
        st = _lib.lib.mb200_ssd_chunk_scan_fwd(prm, _lib.stream_of(x))
    _lib.check(st, "mamba_b200::ssd_chunk_scan_fwd")
    return out, final


@_ssd_chunk_scan_fwd.register_fake
def _(x, dt, A, B, C, D, z, dt_bias, initial_states, seq_idx, dt_softplus, dt_min, dt_max, want_final):
    b, l, h, p = x.shape
    n = B.shape[3]
    return (x.new_empty((b, l, h, p)),
            x.new_empty((b, h, p, n) if want_final else (0,), dtype=torch.float32))


def _no_backward(ctx, grad_out, grad_final):
    raise NotImplementedError(
        "mamba_chunk_scan_combined: this build has the forward (prefill / inference) only; "
        "the backward of the Mamba-2 SSD scan is not built")


_ssd_chunk_scan_fwd.register_autograd(_no_backward)


def mamba_chunk_scan_combined(
    x,
    dt,
    A,
    B,
    C,
    chunk_size,
    D=None,
    z=None,
    dt_bias=None,
    initial_states=None,
    seq_idx=None,
    cu_seqlens=None,
    dt_softplus=False,
    dt_limit=(0.0, float("inf")),
    return_final_states=False,
    return_varlen_states=False,
):
    """Mamba-2 SSD scan over a whole sequence (forward).

    Shapes: x and z (batch, seqlen, nheads, headdim); dt (batch, seqlen, nheads); A and dt_bias
    (nheads,); B and C (batch, seqlen, ngroups, dstate), heads split evenly over the groups;
    D (nheads,) or (nheads, headdim); initial_states (batch, nheads, headdim, dstate).
    Returns out (batch, seqlen, nheads, headdim) in x's dtype, and with
    ``return_final_states=True`` also the float32 state after the last step,
    (batch, nheads, headdim, dstate).

    dt is clamped to ``dt_limit`` after the bias and the optional softplus (threshold 20), as
    upstream does; the default (0, inf) only removes negative steps. ``chunk_size`` is checked
    and otherwise does not change the result beyond rounding: the kernel always works in chunks
    of 64 steps. This build takes bf16 or fp16 x / z (B and C are used in x's dtype; the products
    run in that 16-bit type with float32 accumulation), dstate a multiple of 8
    up to 128 and headdim a multiple of 32 up to 256.

    ``seq_idx`` (batch, seqlen), non-decreasing along seqlen, packs several sequences into one
    row: no step sees another sequence's steps and the state restarts from zero where the id
    changes; ``initial_states`` belong to sequence 0 and ``final_states`` are the last
    sequence's, as upstream. ``cu_seqlens`` / ``return_varlen_states`` (per-sequence final
    states) are not supported, and neither is the backward.
    """
    if not x.is_cuda:
        raise ValueError("mamba_chunk_scan_combined (mamba_cpu_b200) expects CUDA tensors")
    if cu_seqlens is not None or return_varlen_states:
        raise NotImplementedError("cu_seqlens / return_varlen_states are not supported")
    if not isinstance(chunk_size, int) or chunk_size <= 0:
        raise ValueError(f"chunk_size must be a positive int, got {chunk_size!r}")
    if x.dim() != 4:
        raise ValueError(f"x must be (batch, seqlen, nheads, headdim), got {tuple(x.shape)}")
    b, l, h, p = x.shape
    if dt.shape != (b, l, h):
        raise ValueError(f"dt must be {(b, l, h)}, got {tuple(dt.shape)}")
    if A.shape != (h,):
        raise ValueError(f"A must be ({h},), got {tuple(A.shape)}")
    if B.dim() != 4 or B.shape[:2] != (b, l) or C.shape != B.shape:
        raise ValueError(f"B and C must be (batch, seqlen, ngroups, dstate) alike, got {tuple(B.shape)}, "
                         f"{tuple(C.shape)}")
    g, n = B.shape[2], B.shape[3]
    if h % g != 0:
        raise ValueError(f"nheads ({h}) must be a multiple of ngroups ({g})")
    if D is not None and D.shape not in ((h,), (h, p)):
        raise ValueError(f"D must be ({h},) or ({h}, {p}), got {tuple(D.shape)}")
    if z is not None and z.shape != x.shape:
        raise ValueError(f"z must have x's shape {tuple(x.shape)}, got {tuple(z.shape)}")
    if initial_states is not None and initial_states.shape != (b, h, p, n):
        raise ValueError(f"initial_states must be {(b, h, p, n)}, got {tuple(initial_states.shape)}")
    if seq_idx is not None and tuple(seq_idx.shape) != (b, l):
        raise ValueError(f"seq_idx must be {(b, l)}, got {tuple(seq_idx.shape)}")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise NotImplementedError(f"mamba_chunk_scan_combined: x dtype {x.dtype} (this build takes bfloat16 or "
                                  "float16)")
    if n % 8 != 0 or n > 128 or p % 32 != 0 or p > 256:
        raise NotImplementedError(f"mamba_chunk_scan_combined: dstate {n} / headdim {p} outside this build "
                                  "(dstate a multiple of 8 up to 128, headdim a multiple of 32 up to 256)")
    dt_min, dt_max = float(dt_limit[0]), float(dt_limit[1])
    f32 = torch.float32
    x_k = _rows16(x)
    z_k = None if z is None else _rows16(z.to(x.dtype))
    B_k = _rows16(B.to(x.dtype))
    C_k = _rows16(C.to(x.dtype))
    dt_k = dt.to(f32)
    if dt_k.stride(2) != 1:
        dt_k = dt_k.contiguous()
    A_k = A.to(f32).contiguous()
    D_k = None if D is None else D.to(f32).contiguous()
    bias_k = None if dt_bias is None else dt_bias.to(f32).contiguous()
    init_k = None if initial_states is None else initial_states.to(f32).contiguous()
    seq_k = None if seq_idx is None else seq_idx.to(torch.int32)
    out, final = _ssd_chunk_scan_fwd(x_k, dt_k, A_k, B_k, C_k, D_k, z_k, bias_k, init_k, seq_k, bool(dt_softplus),
                                     dt_min, dt_max if not math.isnan(dt_max) else float("inf"),
                                     bool(return_final_states))
    return (out, final) if return_final_states else out
