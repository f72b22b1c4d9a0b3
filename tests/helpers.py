"""Shared helpers for the parity tests: seeded inputs (the reference test suite's distributions,
mamba-cpu tests/test_selective_scan.py:9-26) and tolerance checks against the float64 oracle."""

import numpy as np
import torch


def make_inputs(batch, dim, seqlen, dstate, ngroups, has_D, has_z, has_bias, dtype,
                seed=0, a_scale=1.0):
    g = torch.Generator().manual_seed(seed)

    def normal(*shape):
        return torch.randn(*shape, generator=g).to(dtype)

    bc = (batch, dstate, seqlen) if ngroups is None else (batch, ngroups, dstate, seqlen)
    return dict(
        u=normal(batch, dim, seqlen),
        delta=(torch.rand(batch, dim, seqlen, generator=g) * 0.5).to(dtype),
        A=-torch.rand(dim, dstate, generator=g) * a_scale - 0.5,
        B=normal(*bc),
        C=normal(*bc),
        D=torch.randn(dim, generator=g) if has_D else None,
        z=normal(batch, dim, seqlen) if has_z else None,
        delta_bias=torch.rand(dim, generator=g) * 0.1 if has_bias else None,
    )


def decay_inputs(x, seqlen=4, dstate=8):
    """Every step's dt*A equals x per channel (mamba-cpu tests/test_selective_scan.py:127-139)."""
    dim = x.shape[0]
    g = torch.Generator().manual_seed(0)
    return dict(
        u=torch.randn(1, dim, seqlen, generator=g),
        delta=torch.ones(1, dim, seqlen),
        A=x[:, None].expand(dim, dstate).contiguous(),
        B=torch.randn(1, dstate, seqlen, generator=g),
        C=torch.randn(1, dstate, seqlen, generator=g),
    )


def to_cuda(inp, requires_grad=False):
    return {k: (None if v is None else v.detach().cuda().requires_grad_(requires_grad))
            for k, v in inp.items()}


def np64(t):
    if t is None:
        return None
    if isinstance(t, torch.Tensor):
        return t.detach().float().cpu().numpy().astype(np.float64)
    return np.asarray(t, dtype=np.float64)


def assert_close(got, want, rtol, atol, name="", max_frac=0.0, norm_tol=None):
    """Elementwise |got - want| <= atol + rtol |want| on all but `max_frac` of the elements, NaN
    patterns equal, and (optionally) max|err| / max(1, max|want|) <= norm_tol."""
    g, w = np64(got), np64(want)
    assert g.shape == w.shape, f"{name}: shape {g.shape} != {w.shape}"
    gn, wn = np.isnan(g), np.isnan(w)
    assert np.array_equal(gn, wn), f"{name}: NaN pattern differs ({gn.sum()} vs {wn.sum()})"
    g, w = np.where(gn, 0.0, g), np.where(wn, 0.0, w)
    gi, wi = np.isinf(g), np.isinf(w)
    assert np.array_equal(gi, wi) and np.array_equal(g[gi], w[wi]), f"{name}: inf pattern differs"
    g, w = np.where(gi, 0.0, g), np.where(wi, 0.0, w)
    err = np.abs(g - w)
    bad = err > atol + rtol * np.abs(w)
    frac = bad.mean() if bad.size else 0.0
    worst = float(err.max()) if err.size else 0.0
    assert frac <= max_frac, (f"{name}: {bad.sum()}/{bad.size} elements outside rtol={rtol} atol={atol} "
                              f"(max err {worst:.3e}, at want={w.flat[err.argmax()]:.4e})")
    if norm_tol is not None and err.size:
        scale = max(1.0, float(np.abs(w).max()))
        assert worst / scale <= norm_tol, f"{name}: max err {worst:.3e} / scale {scale:.3e} > {norm_tol}"


def inner_fn_ref(xz, conv1d_weight, conv1d_bias, x_proj_weight, delta_proj_weight, out_proj_weight,
                 out_proj_bias, A, B=None, C=None, D=None, delta_bias=None, B_proj_bias=None,
                 C_proj_bias=None, delta_softplus=True, checkpoint_lvl=1, b_rms_weight=None,
                 c_rms_weight=None, dt_rms_weight=None, b_c_dt_rms_eps=1e-6):
    """mamba_ssm's inner function (mamba_ssm 2.2, ops/selective_scan_interface.py MambaInnerFn /
    mamba_inner_ref) in plain PyTorch: conv1d + SiLU, x_proj, dt_proj, the RMS norms of B, C (over
    d_state) and delta (over d_inner, after dt_proj), the selective scan, out_proj."""
    import torch.nn.functional as F

    from mamba_cpu_b200 import causal_conv1d_ref, selective_scan_ref

    def rms(t, w):
        ct = torch.promote_types(t.dtype, torch.float32)
        tf = t.to(ct)
        y = tf * torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + b_c_dt_rms_eps)
        return (y if w is None else y * w.to(ct)).to(t.dtype)

    r, n = delta_proj_weight.shape[1], A.shape[-1]
    x, z = xz.chunk(2, dim=1)
    x = causal_conv1d_ref(x, conv1d_weight.reshape(conv1d_weight.shape[0], -1), conv1d_bias, "silu")
    x_dbl = F.linear(x.transpose(1, 2), x_proj_weight)  # (b, l, r + 2n)
    delta = F.linear(x_dbl[..., :r], delta_proj_weight)  # (b, l, d)
    if dt_rms_weight is not None:
        delta = rms(delta, dt_rms_weight)
    if B is None:
        B = x_dbl[..., r:r + n] + (0 if B_proj_bias is None else B_proj_bias)
        B = (B if b_rms_weight is None else rms(B, b_rms_weight)).transpose(1, 2)
    if C is None:
        C = x_dbl[..., r + n:r + 2 * n] + (0 if C_proj_bias is None else C_proj_bias)
        C = (C if c_rms_weight is None else rms(C, c_rms_weight)).transpose(1, 2)
    y = selective_scan_ref(x, delta.transpose(1, 2), A, B, C, D, z, delta_bias, delta_softplus)
    return F.linear(y.transpose(1, 2), out_proj_weight, out_proj_bias)
