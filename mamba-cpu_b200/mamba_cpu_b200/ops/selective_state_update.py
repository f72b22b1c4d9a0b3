"""Single decode step of the selective scan on B200.

Same signature, layouts and in-place semantics as mamba-cpu's
src/mamba_cpu/ops/selective_state_update.py:5-57 (Mamba-1 layout, and the Mamba-2 multi-head
layout, which is the Mamba-1 one with dim = nheads * headdim after flattening, :101-111). The
reference runs this in plain PyTorch; here it is one kernel (libmamba_b200.so) behind the op
``mamba_b200::selective_state_update``.
"""

from typing import Optional

import torch

from .. import _lib

_IO = (torch.float32, torch.bfloat16, torch.float16)


@torch.library.custom_op("mamba_b200::selective_state_update", mutates_args=("state",), device_types="cuda")
def _selective_state_update(
    state: torch.Tensor,
    x: torch.Tensor,
    dt: torch.Tensor,
    A: torch.Tensor,
    B: torch.Tensor,
    C: torch.Tensor,
    D: Optional[torch.Tensor],
    z: Optional[torch.Tensor],
    dt_bias: Optional[torch.Tensor],
    dt_softplus: bool,
) -> torch.Tensor:
    """Flattened layout: state (b, d, n); x, dt, z (b, d); A (d, n); B, C (b, g, n); D, dt_bias (d)."""
    out = torch.empty_like(x)
    p = _lib.StateUpdateParams()
    p.state, p.x, p.dt, p.A, p.B, p.C = (_lib.ptr(state), _lib.ptr(x), _lib.ptr(dt), _lib.ptr(A),
                                         _lib.ptr(B), _lib.ptr(C))
    p.D, p.z, p.dt_bias, p.out = _lib.ptr(D), _lib.ptr(z), _lib.ptr(dt_bias), _lib.ptr(out)
    p.batch, p.dim = x.shape
    p.dstate = state.shape[-1]
    p.ngroups = B.shape[1]
    p.io_dtype = _lib.dtype_code(x.dtype)
    p.bc_dtype = _lib.dtype_code(B.dtype)
    p.state_dtype = _lib.dtype_code(state.dtype)
    p.dt_softplus = int(bool(dt_softplus))
    with torch.cuda.device(x.device):
        st = _lib.lib.mb200_selective_state_update(p, _lib.stream_of(x))
    _lib.check(st, "mamba_b200::selective_state_update")
    return out


@_selective_state_update.register_fake
def _(state, x, dt, A, B, C, D, z, dt_bias, dt_softplus):
    return torch.empty_like(x)


def selective_state_update(
    state, x, dt, A, B, C, D=None, z=None, dt_bias=None, dt_softplus=False, state_batch_indices=None
):
    """Single decode step of the selective scan. Updates state in place.

    Mamba-1 shapes:
        state: (batch, dim, dstate)
        x, dt, z: (batch, dim)
        A: (dim, dstate)
        B, C: (batch, dstate)
        D, dt_bias: (dim,)
    Mamba-2 (multi-head) shapes:
        state: (batch, nheads, headdim, dstate)
        x, dt, z: (batch, nheads, headdim)
        A: (nheads, headdim, dstate)
        B, C: (batch, ngroups, dstate)
        D, dt_bias: (nheads, headdim)
    Returns out shaped like x.
    """
    if state_batch_indices is not None:
        raise NotImplementedError("state_batch_indices is not supported yet")
    if x.device.type != "cuda":
        raise ValueError(f"mamba_cpu_b200 runs on CUDA tensors, got device {x.device}")
    has_heads = state.dim() > 3
    batch, dstate = state.shape[0], state.shape[-1]
    if dstate > _lib.DECODE_MAX_DSTATE:
        raise NotImplementedError(f"dstate > {_lib.DECODE_MAX_DSTATE} is not supported by the B200 kernels")
    lead = tuple(state.shape[1:-1])
    dim = 1
    for s in lead:
        dim *= s
    io = x.dtype if x.dtype in _IO else torch.float32
    Bg = B if has_heads else B.unsqueeze(1)
    Cg = C if has_heads else C.unsqueeze(1)
    if Bg.dtype not in (torch.float32, io) or Cg.dtype != Bg.dtype:
        Bg, Cg = Bg.float(), Cg.float()
    if dim % Bg.shape[1] != 0:
        raise ValueError(f"heads ({dim}) must be divisible by ngroups ({Bg.shape[1]})")

    def flat(t, dtype=io):
        return None if t is None else t.to(dtype).reshape(batch, dim).contiguous()

    def per_channel(t):
        return None if t is None else t.float().expand(*lead).reshape(dim).contiguous()

    st = state if (state.dtype in (torch.float32, io) and state.is_contiguous()) else state.to(torch.float32).contiguous()
    st_flat = st.view(batch, dim, dstate)
    out = torch.ops.mamba_b200.selective_state_update(
        st_flat, flat(x), flat(dt), A.float().expand(*lead, dstate).reshape(dim, dstate).contiguous(),
        Bg.contiguous(), Cg.contiguous(), per_channel(D), flat(z), per_channel(dt_bias), bool(dt_softplus))
    if st is not state:
        state.copy_(st)
    return out.view(batch, *lead).to(x.dtype)
