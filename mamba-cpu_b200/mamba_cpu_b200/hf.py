"""Hugging Face route: run transformers' Mamba-family mixers on the B200 kernels.

Mamba-2 models (an addition: the reference patches the Mamba-1 families only) are routed the same
way through ``mamba_chunk_scan_combined`` and a composed ``mamba_split_conv1d_scan_combined``,
for inference.

mamba-cpu's ``hf.patch_transformers`` (src/mamba_cpu/hf.py:63-102) wraps module-level functions
(``mamba_selective_scan``, ...) that transformers 5.x no longer has. In transformers 5.5 each
mixer resolves its fast path when it is constructed: ``MambaMixer.__init__`` calls
``lazy_load_kernel("causal-conv1d")`` and ``lazy_load_kernel("mamba-ssm")``
(transformers/models/mamba/modeling_mamba.py), and ``lazy_load_kernel`` returns whatever module is
already registered under that name in ``transformers.integrations.hub_kernels._KERNEL_MODULE_MAPPING``.
The mixer then takes ``cuda_kernels_forward`` when all five of ``causal_conv1d_fn``,
``causal_conv1d_update``, ``selective_state_update``, ``selective_scan_fn`` and
``mamba_inner_fn`` are set and its weights are on a CUDA device; CPU models keep their
sequential PyTorch path.

:func:`patch_transformers` registers modules exposing this package's functions under those names
(and sets the globals of already-imported modeling modules, for mixers built earlier). Training
without a cache calls ``mamba_inner_fn``; here it is composed from the package's own ops (conv1d
with SiLU, the x / dt projections in PyTorch, the selective scan, the output projection), with
autograd through all of them.
"""

import importlib
import types
from typing import Optional

import torch
import torch.nn.functional as F

from .ops import (
    causal_conv1d_fn,
    causal_conv1d_update,
    mamba_chunk_scan_combined,
    selective_scan_fn,
    selective_state_update,
)

_KEYS = ("causal-conv1d", "mamba-ssm", "falcon_mamba-ssm")
_MODELS = ("mamba", "falcon_mamba", "jamba", "mamba2")
# the module globals each modeling module's fast path reads
_MODEL_GLOBALS = {
    "mamba": ("causal_conv1d_fn", "causal_conv1d_update", "selective_state_update", "selective_scan_fn",
              "mamba_inner_fn"),
    "falcon_mamba": ("causal_conv1d_fn", "causal_conv1d_update", "selective_state_update", "selective_scan_fn",
                     "falcon_mamba_inner_fn"),
    "jamba": ("causal_conv1d_fn", "causal_conv1d_update", "selective_state_update", "selective_scan_fn",
              "mamba_inner_fn"),
    "mamba2": ("causal_conv1d_fn", "causal_conv1d_update", "selective_state_update", "mamba_chunk_scan_combined",
               "mamba_split_conv1d_scan_combined"),
}
_saved: Optional[dict] = None


def _rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    """x / rms(x) over the last dim, times weight (in fp32 or wider, returned in x's dtype)."""
    ct = torch.promote_types(x.dtype, torch.float32)
    xf = x.to(ct)
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if weight is not None:
        y = y * weight.to(ct)
    return y.to(x.dtype)


def mamba_inner_fn(xz, conv1d_weight, conv1d_bias, x_proj_weight, delta_proj_weight, out_proj_weight,
                   out_proj_bias, A, B=None, C=None, D=None, delta_bias=None, B_proj_bias=None,
                   C_proj_bias=None, delta_softplus=True, checkpoint_lvl=1, b_rms_weight=None,
                   c_rms_weight=None, dt_rms_weight=None, b_c_dt_rms_eps=1e-6):
    """The Mamba-1 mixer body (mamba_ssm's ``mamba_inner_fn`` signature) on this package's ops.

    xz: (batch, 2 * d_inner, seqlen), the in_proj output; returns (batch, seqlen, d_model).
    ``checkpoint_lvl`` is accepted for signature compatibility (nothing is recomputed here beyond
    what the scan op's backward does itself). The optional RMS weights are falcon-mamba's
    normalisations, placed where mamba_ssm's ``MambaInnerFn.forward`` (mamba_ssm 2.2,
    mamba_ssm/ops/selective_scan_interface.py) places them: B and C over d_state, and delta over
    d_inner AFTER the dt projection (``dt_rms_weight`` has d_inner entries; transformers' FalconMamba
    passes its ``dt_rms`` buffer of that size). transformers' sequential FalconMamba mixer instead
    normalises the dt_rank features before ``dt_proj``, so its training fast path and its
    sequential path are different functions.
    """
    batch, _, seqlen = xz.shape
    d_state = A.shape[-1]
    dt_rank = delta_proj_weight.shape[1]
    x, z = xz.chunk(2, dim=1)
    x = causal_conv1d_fn(x, conv1d_weight.reshape(conv1d_weight.shape[0], -1), conv1d_bias, activation="silu")
    d_inner = x.shape[1]
    x_dbl = F.linear(x.transpose(1, 2).reshape(batch * seqlen, d_inner), x_proj_weight)  # (b l, r + 2n)
    # delta as (d, b l): its (b, d, l) view below is seqlen-contiguous, which the scan reads in place
    delta = delta_proj_weight @ x_dbl[:, :dt_rank].t()
    if dt_rms_weight is not None:
        delta = _rms_norm(delta.t(), dt_rms_weight, b_c_dt_rms_eps).t()  # over d_inner
    delta = delta.reshape(d_inner, batch, seqlen).transpose(0, 1)  # (b, d, l)

    def _bc(M, start, bias, rms_w):
        if M is not None:
            return M
        M = x_dbl[:, start:start + d_state]
        if bias is not None:
            M = M + bias.to(M.dtype)
        if rms_w is not None:
            M = _rms_norm(M, rms_w, b_c_dt_rms_eps)
        return M.reshape(batch, seqlen, d_state).transpose(1, 2)  # (b, n, l)

    B = _bc(B, dt_rank, B_proj_bias, b_rms_weight)
    C = _bc(C, dt_rank + d_state, C_proj_bias, c_rms_weight)
    y = selective_scan_fn(x, delta, A, B, C, D, z, delta_bias, delta_softplus)
    return F.linear(y.transpose(1, 2), out_proj_weight, out_proj_bias)


def ssd_chunk_scan(x, dt, A, B, C, chunk_size, D=None, z=None, dt_bias=None, initial_states=None, seq_idx=None,
                   cu_seqlens=None, dt_softplus=False, dt_limit=(0.0, float("inf")), return_final_states=False,
                   return_varlen_states=False):
    """``mamba_chunk_scan_combined`` for transformers' Mamba-2 mixer. The SSD kernel multiplies in
    bf16 or fp16: x, z, B and C of an fp32 model are rounded to bf16 and the output is returned in
    x's dtype (upstream's Triton kernels likewise multiply fp32 inputs in tf32)."""
    dtype = x.dtype
    work = dtype if dtype in (torch.bfloat16, torch.float16) else torch.bfloat16

    def bf(t):
        return None if t is None else (t if t.dtype == work else t.to(work))

    r = mamba_chunk_scan_combined(bf(x), dt, A, bf(B), bf(C), chunk_size, D=D, z=bf(z), dt_bias=dt_bias,
                                  initial_states=initial_states, seq_idx=seq_idx, cu_seqlens=cu_seqlens,
                                  dt_softplus=dt_softplus, dt_limit=dt_limit, return_final_states=return_final_states,
                                  return_varlen_states=return_varlen_states)
    if return_final_states:
        return r[0].to(dtype), r[1]
    return r.to(dtype)


def mamba_split_conv1d_scan_combined(zxbcdt, conv1d_weight, conv1d_bias, dt_bias, A, D, chunk_size,
                                     initial_states=None, seq_idx=None, dt_limit=(0.0, float("inf")),
                                     return_final_states=False, activation="silu", rmsnorm_weight=None,
                                     rmsnorm_eps=1e-6, outproj_weight=None, outproj_bias=None, headdim=None,
                                     ngroups=1, norm_before_gate=True):
    """The Mamba-2 mixer body (mamba_ssm's ``mamba_split_conv1d_scan_combined`` signature) on this
    package's ops: split ``zxbcdt`` (batch, seqlen, [z | x B C | dt]), causal conv1d with SiLU over
    x B C, the SSD scan, the gated RMS norm (over the whole inner dimension, as transformers'
    ``MambaRMSNormGated``) and the output projection. Forward only: the SSD backward is not built,
    so gradients through it raise ``NotImplementedError``."""
    if D is None or headdim is None:
        raise ValueError("mamba_split_conv1d_scan_combined needs D and headdim")
    nheads = A.shape[0]
    dim = nheads * headdim
    batch, seqlen, _ = zxbcdt.shape
    dstate = (zxbcdt.shape[-1] - 2 * dim - nheads) // (2 * ngroups)
    z, xbc, dt = torch.split(zxbcdt, [dim, dim + 2 * ngroups * dstate, nheads], dim=-1)
    xbc = causal_conv1d_fn(xbc.transpose(1, 2), conv1d_weight, conv1d_bias,
                           activation=activation if activation in ("silu", "swish") else None).transpose(1, 2)
    x, B, C = torch.split(xbc, [dim, ngroups * dstate, ngroups * dstate], dim=-1)
    r = ssd_chunk_scan(x.reshape(batch, seqlen, nheads, headdim), dt, A, B.reshape(batch, seqlen, ngroups, dstate),
                       C.reshape(batch, seqlen, ngroups, dstate), chunk_size, D=D,
                       z=None if rmsnorm_weight is not None else z.reshape(batch, seqlen, nheads, headdim),
                       dt_bias=dt_bias, initial_states=initial_states, seq_idx=seq_idx, dt_softplus=True,
                       dt_limit=dt_limit, return_final_states=return_final_states)
    y, last = (r[0], r[1]) if return_final_states else (r, None)
    y = y.reshape(batch, seqlen, dim)
    if rmsnorm_weight is not None:
        ct = torch.promote_types(y.dtype, torch.float32)
        yf = y.to(ct)
        if not norm_before_gate:
            yf = yf * F.silu(z.to(ct))
        yf = yf * torch.rsqrt(yf.pow(2).mean(-1, keepdim=True) + rmsnorm_eps) * rmsnorm_weight.to(ct)
        if norm_before_gate:
            yf = yf * F.silu(z.to(ct))
        y = yf.to(y.dtype)
    out = F.linear(y, outproj_weight, outproj_bias) if outproj_weight is not None else y
    return (out, last) if return_final_states else out


def _values() -> dict:
    return {
        "causal_conv1d_fn": causal_conv1d_fn,
        "causal_conv1d_update": causal_conv1d_update,
        "selective_state_update": selective_state_update,
        "selective_scan_fn": selective_scan_fn,
        "mamba_inner_fn": mamba_inner_fn,
        "falcon_mamba_inner_fn": mamba_inner_fn,
        "mamba_chunk_scan_combined": ssd_chunk_scan,
        "mamba_split_conv1d_scan_combined": mamba_split_conv1d_scan_combined,
    }


def kernel_modules() -> dict:
    """The modules registered under transformers' kernel names."""
    v = _values()
    conv = types.ModuleType("mamba_cpu_b200.hf.causal_conv1d")
    conv.causal_conv1d_fn = v["causal_conv1d_fn"]
    conv.causal_conv1d_update = v["causal_conv1d_update"]
    ssm = types.ModuleType("mamba_cpu_b200.hf.mamba_ssm")
    for name in ("selective_scan_fn", "selective_state_update", "mamba_inner_fn", "falcon_mamba_inner_fn",
                 "mamba_chunk_scan_combined", "mamba_split_conv1d_scan_combined"):
        setattr(ssm, name, v[name])
    return {"causal-conv1d": conv, "mamba-ssm": ssm, "falcon_mamba-ssm": ssm}


def patch_transformers() -> list:
    """Route transformers' Mamba / FalconMamba / Jamba / Mamba-2 mixers with CUDA weights to this package.

    Mamba-2 (``Mamba2ForCausalLM``) runs its prefill on the SSD chunk scan and its cached decoding on
    the conv / state-update kernels; it is inference only (the SSD backward is not built).

    Call before building the model (mixers resolve their kernels in ``__init__``); modeling
    modules already imported also get their globals set, so earlier mixers switch too. Returns
    the names of the modeling modules that were patched. Idempotent; undone by
    :func:`unpatch_transformers`.
    """
    global _saved
    from transformers.integrations import hub_kernels

    mapping = hub_kernels._KERNEL_MODULE_MAPPING
    if _saved is None:
        _saved = {"mapping": {k: mapping.get(k, _MISSING) for k in _KEYS}, "globals": {}}
    mapping.update(kernel_modules())
    patched = []
    values = _values()
    for model in _MODELS:
        try:
            mod = importlib.import_module(f"transformers.models.{model}.modeling_{model}")
        except ImportError:
            continue
        for name in _MODEL_GLOBALS[model]:
            _saved["globals"].setdefault((mod.__name__, name), getattr(mod, name, _MISSING))
            setattr(mod, name, values[name])
        if model in ("jamba", "mamba2"):
            # JambaMambaMixer.__init__ / Mamba2Mixer.__init__ cache the availability in a module
            # global that their forward reads (transformers/models/{jamba,mamba2}/modeling_*.py);
            # mixers built before patching would otherwise keep the sequential path.
            _saved["globals"].setdefault((mod.__name__, "is_fast_path_available"),
                                         getattr(mod, "is_fast_path_available", _MISSING))
            mod.is_fast_path_available = True
        patched.append(mod.__name__)
    return patched


def unpatch_transformers() -> None:
    """Restore transformers' kernel mapping and modeling globals to their state before patching."""
    global _saved
    if _saved is None:
        return
    from transformers.integrations import hub_kernels

    mapping = hub_kernels._KERNEL_MODULE_MAPPING
    for k, v in _saved["mapping"].items():
        if v is _MISSING:
            mapping.pop(k, None)
        else:
            mapping[k] = v
    for (modname, name), v in _saved["globals"].items():
        mod = importlib.import_module(modname)
        if v is _MISSING and name == "is_fast_path_available":
            # mixers built while patched read this global in forward: leave them the sequential path
            setattr(mod, name, False)
        elif v is _MISSING:
            if hasattr(mod, name):
                delattr(mod, name)
        else:
            setattr(mod, name, v)
    _saved = None


class _Missing:
    def __repr__(self):
        return "<missing>"


_MISSING = _Missing()
