"""Causal depthwise conv1d (+ SiLU) and its decode step on B200.

Mirrors mamba-cpu's src/mamba_cpu/ops/causal_conv1d.py: same public signatures as the
``causal_conv1d`` package (:16-25, :56-58), same argument meaning and errors (seq_idx,
cache_seqlens and conv_state_indices raise NotImplementedError; an unknown activation raises
ValueError, :8-13). Where the reference runs torch's F.conv1d plus autograd, these run the
CUDA kernels of libmamba_b200.so through the ops ``mamba_b200::causal_conv1d_fwd`` /
``::causal_conv1d_bwd`` / ``::causal_conv1d_update``. Arithmetic is float32 for every input
dtype; outputs come back in x's dtype, as the reference returns them.
"""

from typing import Optional

import torch

from .. import _lib

_IO = (torch.float32, torch.bfloat16, torch.float16)


def _silu_flag(activation) -> bool:
    if activation is None:
        return False
    if activation in ("silu", "swish"):
        return True
    raise ValueError(f"activation must be None, 'silu' or 'swish', got {activation!r}")


def _conv_params(x, weight, bias, initial_states, silu):
    batch, dim, seqlen = x.shape
    p = _lib.Conv1dParams()
    p.x, p.weight, p.bias, p.initial_states = (_lib.ptr(x), _lib.ptr(weight), _lib.ptr(bias),
                                               _lib.ptr(initial_states))
    p.batch, p.dim, p.seqlen, p.width = batch, dim, seqlen, weight.shape[1]
    p.x_dtype = _lib.dtype_code(x.dtype)
    p.activation = int(bool(silu))
    return p


def _check(name, x, weight, bias, initial_states):
    if x.dim() != 3 or weight.dim() != 2 or weight.shape[0] != x.shape[1]:
        raise ValueError(f"{name}: x must be (batch, dim, seqlen) and weight (dim, width)")
    if x.dtype not in _IO or not x.is_contiguous():
        raise ValueError(f"{name}: x must be contiguous float32 / bfloat16 / float16")
    for t, nm in ((weight, "weight"), (bias, "bias")):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()):
            raise ValueError(f"{name}: {nm} must be contiguous float32")
    if initial_states is not None:
        want = (x.shape[0], x.shape[1], weight.shape[1] - 1)
        if initial_states.dtype != x.dtype or tuple(initial_states.shape) != want or not initial_states.is_contiguous():
            raise ValueError(f"{name}: initial_states must be contiguous {want} in x's dtype")


@torch.library.custom_op("mamba_b200::causal_conv1d_fwd", mutates_args=(), device_types="cuda")
def _causal_conv1d_fwd(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor],
    initial_states: Optional[torch.Tensor],
    silu: bool,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (out, final_states (batch, dim, width - 1)), both in x's dtype."""
    _check("mamba_b200::causal_conv1d_fwd", x, weight, bias, initial_states)
    out = torch.empty_like(x)
    final = x.new_empty(x.shape[0], x.shape[1], weight.shape[1] - 1)
    p = _conv_params(x, weight, bias, initial_states, silu)
    p.out, p.final_states = _lib.ptr(out), (_lib.ptr(final) if final.numel() else None)
    with torch.cuda.device(x.device):
        st = _lib.lib.mb200_causal_conv1d_fwd(p, _lib.stream_of(x))
    _lib.check(st, "mamba_b200::causal_conv1d_fwd")
    return out, final


@_causal_conv1d_fwd.register_fake
def _(x, weight, bias, initial_states, silu):
    return torch.empty_like(x), x.new_empty(x.shape[0], x.shape[1], weight.shape[1] - 1)


@torch.library.custom_op("mamba_b200::causal_conv1d_bwd", mutates_args=(), device_types="cuda")
def _causal_conv1d_bwd(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor],
    initial_states: Optional[torch.Tensor],
    silu: bool,
    dout: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (dx, dweight, dbias, dinitial_states); dbias / dinitial_states are empty when the
    corresponding input is None."""
    _check("mamba_b200::causal_conv1d_bwd", x, weight, bias, initial_states)
    if dout.shape != x.shape or dout.dtype != x.dtype or not dout.is_contiguous():
        raise ValueError("mamba_b200::causal_conv1d_bwd: dout must be contiguous with x's shape and dtype")
    dx = torch.empty_like(x)
    dw = torch.empty_like(weight)
    db = torch.empty_like(bias) if bias is not None else x.new_empty(0, dtype=torch.float32)
    dinit = torch.empty_like(initial_states) if initial_states is not None else x.new_empty(0)
    p = _conv_params(x, weight, bias, initial_states, silu)
    nbytes = _lib.lib.mb200_causal_conv1d_bwd_workspace_size(p)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        st = _lib.lib.mb200_causal_conv1d_bwd(
            p, _lib.ptr(dout), _lib.ptr(dx), _lib.ptr(dw), _lib.ptr(db) if bias is not None else None,
            _lib.ptr(dinit) if initial_states is not None else None, _lib.ptr(ws), nbytes,
            _lib.stream_of(x))
    _lib.check(st, "mamba_b200::causal_conv1d_bwd")
    return dx, dw, db, dinit


@_causal_conv1d_bwd.register_fake
def _(x, weight, bias, initial_states, silu, dout):
    return (torch.empty_like(x), torch.empty_like(weight),
            torch.empty_like(bias) if bias is not None else x.new_empty(0, dtype=torch.float32),
            torch.empty_like(initial_states) if initial_states is not None else x.new_empty(0))


def _setup_context(ctx, inputs, output):
    x, weight, bias, initial_states, silu = inputs
    ctx.save_for_backward(x, weight, bias, initial_states)
    ctx.silu = silu


def _backward(ctx, grad_out, grad_final):
    x, weight, bias, initial_states = ctx.saved_tensors
    dout = torch.zeros_like(x) if grad_out is None else grad_out.to(x.dtype).contiguous()
    dx, dw, db, dinit = torch.ops.mamba_b200.causal_conv1d_bwd(x, weight, bias, initial_states, ctx.silu, dout)
    if grad_final is not None and grad_final.numel():
        # final_states[j] = [initial_states | x][seqlen + j]  (causal_conv1d.py:48-53)
        # The sums are formed in fp32 and rounded to x's dtype once (grad_final is not rounded to
        # bf16 / fp16 before it is added).
        P, L = grad_final.shape[-1], x.shape[-1]
        gf = grad_final.float()
        nx = min(P, L)  # entries that come from x
        if nx:
            dx[..., L - nx:] = (dx[..., L - nx:].float() + gf[..., P - nx:]).to(dx.dtype)
        if P > L and initial_states is not None:
            dinit[..., L:] = (dinit[..., L:].float() + gf[..., : P - L]).to(dinit.dtype)
    return dx, dw, (db if bias is not None else None), (dinit if initial_states is not None else None), None


torch.library.register_autograd("mamba_b200::causal_conv1d_fwd", _backward, setup_context=_setup_context)


def causal_conv1d_fn(
    x,
    weight,
    bias=None,
    seq_idx=None,
    initial_states=None,
    return_final_states=False,
    final_states_out=None,
    activation=None,
):
    """
    x: (batch, dim, seqlen)
    weight: (dim, width)
    bias: (dim,)
    initial_states: (batch, dim, width - 1)
    final_states_out: optional (batch, dim, width - 1) buffer for the final states
    Returns out: (batch, dim, seqlen) in x's dtype [, final_states: (batch, dim, width - 1)]
    """
    if seq_idx is not None:
        raise NotImplementedError("seq_idx is not supported yet")
    silu = _silu_flag(activation)
    if x.device.type != "cuda":
        raise ValueError(f"mamba_cpu_b200 runs on CUDA tensors, got device {x.device}")
    width = weight.shape[1]
    if width > _lib.CONV_MAX_WIDTH:
        raise NotImplementedError(f"conv width > {_lib.CONV_MAX_WIDTH} is not supported by the B200 kernels")
    io = x.dtype if x.dtype in _IO else torch.float32
    init = None if initial_states is None else initial_states.to(io).contiguous()
    out, final = torch.ops.mamba_b200.causal_conv1d_fwd(
        x.to(io).contiguous(), weight.float().contiguous(),
        None if bias is None else bias.float().contiguous(), init, silu)
    out = out.to(x.dtype)
    if not return_final_states:
        return out
    final = final.to(x.dtype)
    if final_states_out is not None:
        final = final_states_out.copy_(final)
    return out, final


@torch.library.custom_op("mamba_b200::causal_conv1d_update", mutates_args=("conv_state",), device_types="cuda")
def _causal_conv1d_update(
    x: torch.Tensor, conv_state: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], silu: bool
) -> torch.Tensor:
    if x.dtype != conv_state.dtype or not x.is_contiguous() or not conv_state.is_contiguous():
        raise ValueError("mamba_b200::causal_conv1d_update: x and conv_state must be contiguous, same dtype")
    out = torch.empty_like(x)
    p = _lib.Conv1dUpdateParams()
    p.x, p.conv_state, p.weight, p.bias, p.out = (_lib.ptr(x), _lib.ptr(conv_state), _lib.ptr(weight),
                                                  _lib.ptr(bias), _lib.ptr(out))
    p.batch, p.dim, p.seqlen = x.shape
    p.state_len, p.width = conv_state.shape[-1], weight.shape[1]
    p.x_dtype = _lib.dtype_code(x.dtype)
    p.activation = int(bool(silu))
    with torch.cuda.device(x.device):
        st = _lib.lib.mb200_causal_conv1d_update(p, _lib.stream_of(x))
    _lib.check(st, "mamba_b200::causal_conv1d_update")
    return out


@_causal_conv1d_update.register_fake
def _(x, conv_state, weight, bias, silu):
    return torch.empty_like(x)


def causal_conv1d_update(
    x, conv_state, weight, bias=None, activation=None, cache_seqlens=None, conv_state_indices=None
):
    """Decode step(s). Updates conv_state in place.

    x: (batch, dim) or (batch, dim, seqlen)
    conv_state: (batch, dim, state_len), state_len >= width - 1
    weight: (dim, width)
    Returns out shaped like x.
    """
    if cache_seqlens is not None or conv_state_indices is not None:
        raise NotImplementedError("cache_seqlens and conv_state_indices are not supported yet")
    silu = _silu_flag(activation)
    if x.device.type != "cuda":
        raise ValueError(f"mamba_cpu_b200 runs on CUDA tensors, got device {x.device}")
    single_step = x.dim() == 2
    x_seq = x.unsqueeze(-1) if single_step else x
    width = weight.shape[1]
    state_len = conv_state.shape[-1]
    if state_len < width - 1:
        raise ValueError(f"conv_state length ({state_len}) must be at least width - 1 ({width - 1})")
    if width > _lib.CONV_MAX_WIDTH:
        raise NotImplementedError(f"conv width > {_lib.CONV_MAX_WIDTH} is not supported by the B200 kernels")
    io = conv_state.dtype if conv_state.dtype in _IO else torch.float32
    if conv_state.dtype == io and conv_state.is_contiguous():
        state = conv_state
    else:
        state = conv_state.to(io).contiguous()
    out = torch.ops.mamba_b200.causal_conv1d_update(
        x_seq.to(io).contiguous(), state, weight.float().contiguous(),
        None if bias is None else bias.float().contiguous(), silu)
    if state is not conv_state:
        conv_state.copy_(state)
    out = out.to(x.dtype)
    return out.squeeze(-1) if single_step else out
