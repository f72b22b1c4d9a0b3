"""Readable pure-PyTorch versions of the two operators, for checking results on any device.

The public names and signatures are those of mamba-cpu's ``src/mamba_cpu/reference.py``
(``selective_scan_ref`` :10-62, ``causal_conv1d_ref`` :65-75), which that package exports
(``src/mamba_cpu/__init__.py:9,18,21``) so that user code can compare a kernel against a plain
implementation. These run on whatever device their inputs live on (CPU or CUDA) in float32 and
never call the package's kernels. The scan keeps only the running state (batch, dim, dstate)
between timesteps instead of materialising (batch, dim, seqlen, dstate) tensors, so long
sequences fit in memory; it is a Python loop over time and therefore slow.
"""

import torch
import torch.nn.functional as F


def _per_channel(X: torch.Tensor, dim: int) -> torch.Tensor:
    """(batch, dstate, seqlen) or (batch, ngroups, dstate, seqlen) -> (batch, dim, dstate, seqlen):
    channel d reads group d // (dim // ngroups)."""
    if X.dim() == 3:
        X = X[:, None]
    ngroups = X.shape[1]
    return X.float().repeat_interleave(dim // ngroups, dim=1)


def selective_scan_ref(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                       return_last_state=False):
    """Selective scan h_t = exp(dt_t A) h_{t-1} + dt_t u_t B_t, y_t = <h_t, C_t> (+ D u_t),
    out = y * silu(z) when z is given, with dt = softplus(delta + delta_bias) or delta + delta_bias.

    u, delta, z: (batch, dim, seqlen); A: (dim, dstate) real; B, C: (batch, dstate, seqlen) or
    (batch, ngroups, dstate, seqlen); D, delta_bias: (dim,).
    Returns out (batch, dim, seqlen) in u's dtype [, last_state (batch, dim, dstate) float32].
    """
    out_dtype = u.dtype
    batch, dim, seqlen = u.shape
    dt = delta.float()
    if delta_bias is not None:
        dt = dt + delta_bias.float()[:, None]
    if delta_softplus:
        dt = F.softplus(dt)
    uf = u.float()
    Af = A.float()
    Bc, Cc = _per_channel(B, dim), _per_channel(C, dim)
    h = torch.zeros(batch, dim, Af.shape[-1], dtype=torch.float32, device=u.device)
    y = torch.empty(batch, dim, seqlen, dtype=torch.float32, device=u.device)
    for t in range(seqlen):
        dt_t = dt[:, :, t, None]                                   # (b, d, 1)
        h = torch.exp(dt_t * Af) * h + (dt_t * uf[:, :, t, None]) * Bc[..., t]
        y[:, :, t] = torch.einsum("bdn,bdn->bd", h, Cc[..., t])
    if D is not None:
        y = y + uf * D.float()[:, None]
    if z is not None:
        y = y * F.silu(z.float())
    out = y.to(out_dtype)
    return (out, h) if return_last_state else out


def causal_conv1d_ref(x, weight, bias=None, activation=None):
    """Causal depthwise conv1d: out[b, d, t] = sum_k weight[d, k] x[b, d, t - W + 1 + k] (+ bias[d]),
    zeros before the start, then SiLU when activation is "silu" or "swish".
    x: (batch, dim, seqlen); weight: (dim, width); bias: (dim,) or None. Computed in x's dtype."""
    width = weight.shape[1]
    out = F.conv1d(x, weight.to(x.dtype)[:, None, :], None if bias is None else bias.to(x.dtype),
                   padding=width - 1, groups=x.shape[1])[..., : x.shape[-1]]
    if activation in ("silu", "swish"):
        out = F.silu(out)
    return out
