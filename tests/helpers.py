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
