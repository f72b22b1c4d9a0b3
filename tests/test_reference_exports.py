"""The package's own pure-PyTorch ``selective_scan_ref`` / ``causal_conv1d_ref`` (exported like the
reference's, mamba-cpu src/mamba_cpu/__init__.py:9,18,21) against the golden fixtures the
reference produced. CPU only: the functions run on any device."""

import numpy as np
import pytest
import torch

import mamba_cpu_b200 as mb
from helpers import assert_close
from test_oracle_golden import _cases


def _t(a, k):
    v = a.get(k)
    return None if v is None else torch.from_numpy(np.ascontiguousarray(v))


def test_exported_names():
    for name in ("selective_scan_ref", "causal_conv1d_ref"):
        assert name in mb.__all__ and callable(getattr(mb, name))


@pytest.mark.parametrize("meta,a", [c for c in _cases("scan", "scan") if c.values[0]["dtype"] == "f32"][:40])
def test_selective_scan_ref_matches_reference(meta, a):
    args = [_t(a, "in_" + k) for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")]
    if meta["kind"] == "decay":
        pytest.skip("the reference kernel's clamped exp differs from torch.exp at dt*A = +-3e38")
    with np.errstate(invalid="ignore"):
        out, last = mb.selective_scan_ref(*args, delta_softplus=meta["softplus"], return_last_state=True)
    assert out.dtype == args[0].dtype and last.dtype == torch.float32
    assert_close(out, a["out"], 1e-4, 1e-4, "out")
    assert_close(last, a["last_state"], 1e-4, 1e-4, "last_state")


@pytest.mark.parametrize("meta,a", _cases("conv", "conv"))
def test_causal_conv1d_ref_matches_reference(meta, a):
    if a.get("in_initial_states") is not None:
        pytest.skip("causal_conv1d_ref has no initial_states argument (as in the reference)")
    x = _t(a, "in_x")
    out = mb.causal_conv1d_ref(x, _t(a, "in_weight"), _t(a, "in_bias"), meta["activation"])
    assert out.dtype == x.dtype
    assert_close(out, a["out"], 1e-5, 1e-5, "out")


def test_selective_scan_ref_groups_and_bf16():
    g = torch.Generator().manual_seed(5)
    u = torch.randn(2, 8, 33, generator=g).bfloat16()
    delta = (torch.rand(2, 8, 33, generator=g) * 0.5).bfloat16()
    A = -torch.rand(8, 4, generator=g) - 0.5
    B = torch.randn(2, 2, 4, 33, generator=g)
    C = torch.randn(2, 2, 4, 33, generator=g)
    out = mb.selective_scan_ref(u, delta, A, B, C, z=torch.randn(2, 8, 33, generator=g))
    assert out.dtype == torch.bfloat16 and out.shape == u.shape
    # channel 5 reads group 1 (dim 8 / 2 groups): its row equals the ungrouped scan of group 1
    one = mb.selective_scan_ref(u[:, 4:], delta[:, 4:], A[4:], B[:, 1], C[:, 1])
    full = mb.selective_scan_ref(u, delta, A, B, C)
    assert torch.equal(full[:, 4:], one)
