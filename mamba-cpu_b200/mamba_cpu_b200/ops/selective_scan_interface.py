"""Selective scan: torch.library custom ops on the CUDA dispatch key, autograd, public API.

Mirrors mamba-cpu's src/mamba_cpu/ops/selective_scan_interface.py:
  * ``mamba_b200::selective_scan_fwd`` / ``::selective_scan_bwd`` replace the CPU-only ops
    ``mamba_cpu::selective_scan_fwd`` / ``::selective_scan_bwd`` (:16-97), registered with
    ``register_fake`` and ``register_autograd`` the same way (:43-45, 90-97, 100-124);
  * ``selective_scan_fn`` keeps the exact signature, argument meaning, return types and error
    behaviour of the reference's public function (:138-177), with CUDA tensors where the reference
    takes CPU tensors.

Differences that are deliberate (the B200 kernels need no conversions the CPU kernel needed):
  * B / C stay in the upstream (batch, ngroups, dstate, seqlen) layout -- any batch/group/state
    strides, seqlen stride 1 -- instead of being transposed to (b, g, l, n) (:131-135);
  * float32, bfloat16 and float16 inputs are consumed as they are (fp32 state and accumulation);
    the reference casts everything to float32 first (:127-128);
  * the forward also returns the state after every 64 timesteps (``chunk_states``), which the
    backward uses as restart points instead of recomputing the forward from t = 0;
  * dA / dD / ddelta_bias come back summed over batch (the reference sums per-batch partials in
    Python, :87).
"""

from typing import Optional

import torch

from .. import _lib
from .. import parallel as _parallel


def _nchunks(seqlen: int) -> int:
    return (seqlen + _lib.CHUNK - 1) // _lib.CHUNK


def _fwd_params(u, delta, A, B, C, D, z, delta_bias, delta_softplus):
    batch, dim, seqlen = u.shape
    ngroups, dstate = B.shape[1], B.shape[2]
    p = _lib.ScanFwdParams()
    p.u, p.delta, p.A, p.B, p.C = _lib.ptr(u), _lib.ptr(delta), _lib.ptr(A), _lib.ptr(B), _lib.ptr(C)
    p.D, p.z, p.delta_bias = _lib.ptr(D), _lib.ptr(z), _lib.ptr(delta_bias)
    p.batch, p.dim, p.seqlen, p.dstate, p.ngroups = batch, dim, seqlen, dstate, ngroups
    (p.B_batch_stride, p.B_group_stride, p.B_dstate_stride, p.B_seqlen_stride) = B.stride()
    (p.C_batch_stride, p.C_group_stride, p.C_dstate_stride, p.C_seqlen_stride) = C.stride()
    # u / delta / z may be views with their own batch and dim strides (seqlen-contiguous rows)
    p.u_batch_stride, p.u_dim_stride = u.stride(0), u.stride(1)
    p.delta_batch_stride, p.delta_dim_stride = delta.stride(0), delta.stride(1)
    if z is not None:
        p.z_batch_stride, p.z_dim_stride = z.stride(0), z.stride(1)
    p.io_dtype = _lib.dtype_code(u.dtype)
    p.bc_dtype = _lib.dtype_code(B.dtype)
    p.delta_softplus = int(bool(delta_softplus))
    return p


def _dense(t):
    """A contiguous tensor of t's shape and dtype (the kernels write dense rows; empty_like would
    copy the strides of a view)."""
    return torch.empty_like(t, memory_format=torch.contiguous_format)


def _seqlen_rows(t):
    """(batch, dim, seqlen) rows the kernels can read in place: unit stride along seqlen."""
    return t.shape[-1] <= 1 or t.stride(-1) == 1


def _check_op_inputs(name, u, delta, A, B, C, D, z, delta_bias):
    if u.dim() != 3 or B.dim() != 4 or C.dim() != 4:
        raise ValueError(f"{name}: u must be (batch, dim, seqlen), B/C (batch, ngroups, dstate, seqlen)")
    if u.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise TypeError(f"{name}: u must be float32, bfloat16 or float16")
    for t, nm in ((delta, "delta"), (z, "z")):
        if t is not None and (t.dtype != u.dtype or t.shape != u.shape):
            raise ValueError(f"{name}: {nm} must have u's shape and dtype")
    for t, nm in ((u, "u"), (delta, "delta"), (z, "z")):
        if t is not None and not _seqlen_rows(t):
            raise ValueError(f"{name}: {nm} must be contiguous along seqlen (any batch / dim strides)")
    for t, nm in ((A, "A"), (D, "D"), (delta_bias, "delta_bias")):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()):
            raise ValueError(f"{name}: {nm} must be contiguous float32")
    for t, nm in ((B, "B"), (C, "C")):
        if t.dtype not in (torch.float32, u.dtype):
            raise TypeError(f"{name}: {nm} must be float32 or u's dtype")
    if B.dtype != C.dtype:
        raise TypeError(f"{name}: B and C must share a dtype")


@torch.library.custom_op("mamba_b200::selective_scan_fwd", mutates_args=(), device_types="cuda")
def _selective_scan_fwd(
    u: torch.Tensor,
    delta: torch.Tensor,
    A: torch.Tensor,
    B: torch.Tensor,
    C: torch.Tensor,
    D: Optional[torch.Tensor],
    z: Optional[torch.Tensor],
    delta_bias: Optional[torch.Tensor],
    delta_softplus: bool,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (out in u's dtype, last_state float32 (b, d, n), chunk_states float32 (b, d, c, n))."""
    return _run_fwd("mamba_b200::selective_scan_fwd", u, delta, A, B, C, D, z, delta_bias, delta_softplus, None)


def _check_state(name, what, t, batch, dim, dstate):
    if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.shape != (batch, dim, dstate)):
        raise ValueError(f"{name}: {what} must be contiguous float32 (batch, dim, dstate)")


def _run_fwd(name, u, delta, A, B, C, D, z, delta_bias, delta_softplus, initial_state):
    _check_op_inputs(name, u, delta, A, B, C, D, z, delta_bias)
    batch, dim, seqlen = u.shape
    dstate = B.shape[2]
    _check_state(name, "initial_state", initial_state, batch, dim, dstate)
    out = _dense(u)
    last_state = u.new_empty(batch, dim, dstate, dtype=torch.float32)
    chunk_states = u.new_empty(batch, dim, _nchunks(seqlen), dstate, dtype=torch.float32)
    p = _fwd_params(u, delta, A, B, C, D, z, delta_bias, delta_softplus)
    p.out, p.last_state, p.chunk_states = _lib.ptr(out), _lib.ptr(last_state), _lib.ptr(chunk_states)
    p.initial_state = _lib.ptr(initial_state)
    with torch.cuda.device(u.device):
        # workspace: the sequence-piece summaries, when rows are split over CTAs (small grids)
        nbytes = _lib.lib.mb200_selective_scan_fwd_workspace_size(p)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=u.device) if nbytes else None
        st = _lib.lib.mb200_selective_scan_fwd_ws(p, _lib.ptr(ws), nbytes, _lib.stream_of(u))
    _lib.check(st, name)
    return out, last_state, chunk_states


@_selective_scan_fwd.register_fake
def _(u, delta, A, B, C, D, z, delta_bias, delta_softplus):
    batch, dim, seqlen = u.shape
    dstate = B.shape[2]
    return (
        _dense(u),
        u.new_empty(batch, dim, dstate, dtype=torch.float32),
        u.new_empty(batch, dim, _nchunks(seqlen), dstate, dtype=torch.float32),
    )


@torch.library.custom_op("mamba_b200::selective_scan_bwd", mutates_args=(), device_types="cuda")
def _selective_scan_bwd(
    u: torch.Tensor,
    delta: torch.Tensor,
    A: torch.Tensor,
    B: torch.Tensor,
    C: torch.Tensor,
    D: Optional[torch.Tensor],
    z: Optional[torch.Tensor],
    delta_bias: Optional[torch.Tensor],
    delta_softplus: bool,
    dout: torch.Tensor,
    dlast_state: Optional[torch.Tensor],
    chunk_states: Optional[torch.Tensor],
) -> tuple[
    torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
    torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
]:
    """Returns (du, ddelta, dA, dB, dC, dD, dz, ddelta_bias).

    du/ddelta/dz are in u's dtype, dB/dC float32 in B's shape (contiguous), dA/dD/ddelta_bias
    float32 summed over batch. dz is empty when z is None; dD and ddelta_bias are always
    computed, as in the reference (selective_scan_interface.py:65-66)."""
    return _run_bwd("mamba_b200::selective_scan_bwd", u, delta, A, B, C, D, z, delta_bias, delta_softplus, dout,
                    dlast_state, chunk_states, None)[:8]


def _run_bwd(name, u, delta, A, B, C, D, z, delta_bias, delta_softplus, dout, dlast_state, chunk_states,
             initial_state):
    _check_op_inputs(name, u, delta, A, B, C, D, z, delta_bias)
    if dout.shape != u.shape or dout.dtype != u.dtype or not dout.is_contiguous():
        raise ValueError(f"{name}: dout must be contiguous with u's shape and dtype")
    batch, dim, seqlen = u.shape
    dstate = B.shape[2]
    if dlast_state is not None and (dlast_state.dtype != torch.float32 or not dlast_state.is_contiguous()
                                    or dlast_state.shape != (batch, dim, dstate)):
        raise ValueError(f"{name}: dlast_state must be contiguous float32 (b, d, n)")
    if chunk_states is not None and (chunk_states.dtype != torch.float32 or not chunk_states.is_contiguous()
                                     or chunk_states.shape != (batch, dim, _nchunks(seqlen), dstate)):
        raise ValueError(f"{name}: chunk_states must come from selective_scan_fwd")
    du = _dense(u)
    ddelta = _dense(delta)
    dA = torch.empty_like(A)
    dB = torch.empty(B.shape, dtype=torch.float32, device=u.device)
    dC = torch.empty(C.shape, dtype=torch.float32, device=u.device)
    dD = u.new_empty(dim, dtype=torch.float32)
    dz = _dense(z) if z is not None else u.new_empty(0)
    ddelta_bias = u.new_empty(dim, dtype=torch.float32)
    _check_state(name, "initial_state", initial_state, batch, dim, dstate)
    dinit = u.new_empty(batch, dim, dstate, dtype=torch.float32) if initial_state is not None else u.new_empty(0)
    p = _lib.ScanBwdParams()
    p.fwd = _fwd_params(u, delta, A, B, C, D, z, delta_bias, delta_softplus)
    p.fwd.chunk_states = _lib.ptr(chunk_states)
    p.fwd.initial_state = _lib.ptr(initial_state)
    p.dinitial_state = _lib.ptr(dinit) if initial_state is not None else None
    p.dout, p.dlast_state = _lib.ptr(dout), _lib.ptr(dlast_state)
    p.du, p.ddelta, p.dz = _lib.ptr(du), _lib.ptr(ddelta), (_lib.ptr(dz) if z is not None else None)
    p.dA, p.dB, p.dC, p.dD, p.ddelta_bias = (_lib.ptr(dA), _lib.ptr(dB), _lib.ptr(dC), _lib.ptr(dD),
                                              _lib.ptr(ddelta_bias))
    p.dbc_dtype = _lib.F32
    nbytes = _lib.lib.mb200_selective_scan_bwd_workspace_size(p)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=u.device)
    with torch.cuda.device(u.device):
        st = _lib.lib.mb200_selective_scan_bwd(p, _lib.ptr(ws), nbytes, _lib.stream_of(u))
    _lib.check(st, name)
    return du, ddelta, dA, dB, dC, dD, dz, ddelta_bias, dinit


@_selective_scan_bwd.register_fake
def _(u, delta, A, B, C, D, z, delta_bias, delta_softplus, dout, dlast_state, chunk_states):
    dim = u.shape[1]
    return (
        _dense(u), _dense(delta), torch.empty_like(A),
        u.new_empty(B.shape, dtype=torch.float32), u.new_empty(C.shape, dtype=torch.float32),
        u.new_empty(dim, dtype=torch.float32),
        _dense(z) if z is not None else u.new_empty(0),
        u.new_empty(dim, dtype=torch.float32),
    )


def _setup_context(ctx, inputs, output):
    u, delta, A, B, C, D, z, delta_bias, delta_softplus = inputs
    _, _, chunk_states = output
    ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, chunk_states)
    ctx.delta_softplus = delta_softplus
    # Channel sharding (mamba_cpu_b200.parallel): dB/dC are sums over ALL channels, so the
    # shards' partial sums are all-reduced before they leave the backward.
    ctx.shard_group = _parallel.current_group()


def _backward(ctx, grad_out, grad_last_state, grad_chunk_states):
    u, delta, A, B, C, D, z, delta_bias, chunk_states = ctx.saved_tensors
    dout = _dense(u).zero_() if grad_out is None else grad_out.to(u.dtype).contiguous()
    dlast = None if grad_last_state is None else grad_last_state.float().contiguous()
    du, ddelta, dA, dB, dC, dD, dz, ddelta_bias = torch.ops.mamba_b200.selective_scan_bwd(
        u, delta, A, B, C, D, z, delta_bias, ctx.delta_softplus, dout, dlast, chunk_states
    )
    if ctx.shard_group is not None:
        dB, dC = _parallel.all_reduce_bc(dB, dC, ctx.shard_group)
    return (
        du, ddelta, dA, dB.to(B.dtype), dC.to(C.dtype),
        dD if D is not None else None,
        dz if z is not None else None,
        ddelta_bias if delta_bias is not None else None,
        None,
    )


torch.library.register_autograd(
    "mamba_b200::selective_scan_fwd", _backward, setup_context=_setup_context
)


# ---- variants with an initial state (a sequence scanned in pieces, e.g. across GPUs) ----------
# No reference counterpart: the reference always starts from a zero state. The kernels are the
# same; the state before the first step comes from `initial_state` (batch, dim, dstate) fp32,
# and the backward also returns the gradient with respect to it.


@torch.library.custom_op("mamba_b200::selective_scan_fwd_init", mutates_args=(), device_types="cuda")
def _selective_scan_fwd_init(
    u: torch.Tensor,
    delta: torch.Tensor,
    A: torch.Tensor,
    B: torch.Tensor,
    C: torch.Tensor,
    D: Optional[torch.Tensor],
    z: Optional[torch.Tensor],
    delta_bias: Optional[torch.Tensor],
    delta_softplus: bool,
    initial_state: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """selective_scan_fwd starting from initial_state instead of zeros."""
    return _run_fwd("mamba_b200::selective_scan_fwd_init", u, delta, A, B, C, D, z, delta_bias, delta_softplus,
                    initial_state)


@_selective_scan_fwd_init.register_fake
def _(u, delta, A, B, C, D, z, delta_bias, delta_softplus, initial_state):
    batch, dim, seqlen = u.shape
    dstate = B.shape[2]
    return (
        _dense(u),
        u.new_empty(batch, dim, dstate, dtype=torch.float32),
        u.new_empty(batch, dim, _nchunks(seqlen), dstate, dtype=torch.float32),
    )


@torch.library.custom_op("mamba_b200::selective_scan_bwd_init", mutates_args=(), device_types="cuda")
def _selective_scan_bwd_init(
    u: torch.Tensor,
    delta: torch.Tensor,
    A: torch.Tensor,
    B: torch.Tensor,
    C: torch.Tensor,
    D: Optional[torch.Tensor],
    z: Optional[torch.Tensor],
    delta_bias: Optional[torch.Tensor],
    delta_softplus: bool,
    dout: torch.Tensor,
    dlast_state: Optional[torch.Tensor],
    chunk_states: Optional[torch.Tensor],
    initial_state: torch.Tensor,
) -> tuple[
    torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
    torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
]:
    """selective_scan_bwd of selective_scan_fwd_init: the eight gradients plus dinitial_state."""
    return _run_bwd("mamba_b200::selective_scan_bwd_init", u, delta, A, B, C, D, z, delta_bias, delta_softplus,
                    dout, dlast_state, chunk_states, initial_state)


@_selective_scan_bwd_init.register_fake
def _(u, delta, A, B, C, D, z, delta_bias, delta_softplus, dout, dlast_state, chunk_states, initial_state):
    dim = u.shape[1]
    return (
        _dense(u), _dense(delta), torch.empty_like(A),
        u.new_empty(B.shape, dtype=torch.float32), u.new_empty(C.shape, dtype=torch.float32),
        u.new_empty(dim, dtype=torch.float32),
        _dense(z) if z is not None else u.new_empty(0),
        u.new_empty(dim, dtype=torch.float32),
        torch.empty_like(initial_state),
    )


def _setup_context_init(ctx, inputs, output):
    u, delta, A, B, C, D, z, delta_bias, delta_softplus, initial_state = inputs
    _, _, chunk_states = output
    ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, chunk_states, initial_state)
    ctx.delta_softplus = delta_softplus


def _backward_init(ctx, grad_out, grad_last_state, grad_chunk_states):
    u, delta, A, B, C, D, z, delta_bias, chunk_states, initial_state = ctx.saved_tensors
    dout = _dense(u).zero_() if grad_out is None else grad_out.to(u.dtype).contiguous()
    dlast = None if grad_last_state is None else grad_last_state.float().contiguous()
    du, ddelta, dA, dB, dC, dD, dz, ddelta_bias, dinit = torch.ops.mamba_b200.selective_scan_bwd_init(
        u, delta, A, B, C, D, z, delta_bias, ctx.delta_softplus, dout, dlast, chunk_states, initial_state
    )
    return (
        du, ddelta, dA, dB.to(B.dtype), dC.to(C.dtype),
        dD if D is not None else None,
        dz if z is not None else None,
        ddelta_bias if delta_bias is not None else None,
        None,
        dinit,
    )


torch.library.register_autograd(
    "mamba_b200::selective_scan_fwd_init", _backward_init, setup_context=_setup_context_init
)


_IO_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


def _as_rows(X: torch.Tensor, io_dtype) -> torch.Tensor:
    # u / delta / z: a view whose rows are seqlen-contiguous and 16-byte aligned is read in place
    # (no copy of e.g. a transposed projection output or a chunk of in_proj's output); anything
    # else is made contiguous.
    X = X.to(io_dtype)
    es = X.element_size()
    if (_seqlen_rows(X) and X.data_ptr() % 16 == 0 and (X.stride(0) * es) % 16 == 0
            and (X.stride(1) * es) % 16 == 0):
        return X
    return X.contiguous()


def _as_kernel_bc(X: torch.Tensor, io_dtype) -> torch.Tensor:
    # (b, n, l) or (b, g, n, l) -> (b, g, n, l) view. Seqlen-contiguous B / C are staged by the
    # bulk-copy engine; other layouts (x_proj's slices in mamba_inner_fn have seqlen stride
    # dt_rank + 2 * dstate) are read by per-lane loads in the kernels. For float32 that is faster
    # than a copy (HF layout at config-2 size, fwd + bwd through autograd: 0.649 ms in place vs
    # 0.725 ms copied); for 2-byte types the copy is faster (0.561 vs 0.663 ms), so those are copied.
    if X.dim() == 3:
        X = X.unsqueeze(1)
    if X.dtype not in (torch.float32, io_dtype):
        X = X.float()
    if X.shape[-1] > 1 and X.stride(-1) != 1 and X.dtype != torch.float32:
        X = X.contiguous()
    return X


def selective_scan_fn(
    u,
    delta,
    A,
    B,
    C,
    D=None,
    z=None,
    delta_bias=None,
    delta_softplus=False,
    return_last_state=False,
):
    """Drop-in for mamba_ssm.ops.selective_scan_interface.selective_scan_fn on B200 GPUs.

    u, delta, z: (batch, dim, seqlen)
    A: (dim, dstate), real-valued, dstate <= 16
    B, C: (batch, dstate, seqlen) or (batch, ngroups, dstate, seqlen)
    D, delta_bias: (dim,)
    Returns out: (batch, dim, seqlen) in u's dtype [, last_state: (batch, dim, dstate) float32]
    """
    if u.device.type != "cuda":
        raise ValueError(f"mamba_cpu_b200 runs on CUDA tensors, got device {u.device}")
    if A.is_complex():
        raise NotImplementedError("complex A is not supported yet")
    if B.dim() < 3 or C.dim() < 3:
        raise NotImplementedError("input-independent (2D) B/C is not supported yet")
    dim = u.shape[1]
    for name, X in (("B", B), ("C", C)):
        ngroups = 1 if X.dim() == 3 else X.shape[1]
        if dim % ngroups != 0:
            raise ValueError(f"dim ({dim}) must be divisible by {name}'s ngroups ({ngroups})")
    if B.dim() != C.dim() or (B.dim() == 4 and B.shape[1] != C.shape[1]):
        raise NotImplementedError("B and C must have the same number of groups")
    if A.shape[-1] > _lib.MAX_DSTATE:
        raise NotImplementedError(f"dstate > {_lib.MAX_DSTATE} is not supported by the B200 kernels")

    io = u.dtype
    if io not in _IO_DTYPES or delta.dtype != io or (z is not None and z.dtype != io):
        io = torch.float32
    Bk, Ck = _as_kernel_bc(B, io), _as_kernel_bc(C, io)
    if Bk.dtype != Ck.dtype:
        Bk, Ck = Bk.float(), Ck.float()
    out, last_state, _ = torch.ops.mamba_b200.selective_scan_fwd(
        _as_rows(u, io), _as_rows(delta, io), A.float().contiguous(), Bk, Ck,
        None if D is None else D.float().contiguous(),
        None if z is None else _as_rows(z, io),
        None if delta_bias is None else delta_bias.float().contiguous(),
        bool(delta_softplus),
    )
    out = out.to(u.dtype)
    return (out, last_state) if return_last_state else out
