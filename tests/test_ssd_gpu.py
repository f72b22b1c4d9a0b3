"""Mamba-2 SSD chunk scan forward (mamba_chunk_scan_combined) on the GPU.

Checked two ways: against the reference's own kernel on the equivalent Mamba-1 problem
(tests/golden/ssd.npz, tests/golden/make_golden.py:make_ssd), and against the float64 oracle
(oracle.f64.ssd_fwd, itself pinned to those fixtures by tests/test_oracle_golden.py) on the same
bf16-rounded inputs. Tolerances: bf16 outputs within 1e-2 of their largest magnitude (plus 2e-2
relative), the reference suite's bf16 forward bound (tests/test_selective_scan.py:44-50); the
float32 final states within 5e-3 of their largest magnitude (the kernel's M and X' operands are
bf16)."""

import ast
import os

import numpy as np
import pytest
import torch

import mamba_cpu_b200 as mb
from helpers import np64
from oracle import f64

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
BF = torch.bfloat16


def _close(got, want, tol, name, rel=2e-2):
    g, w = np64(got), np64(want)
    assert g.shape == w.shape, f"{name}: shape {g.shape} != {w.shape}"
    scale = max(float(np.abs(w).max()), 1e-6)
    err = np.abs(g - w)
    assert np.isfinite(g).all(), f"{name}: non-finite values"
    assert err.max() <= tol * scale + 1e-6, f"{name}: max err {err.max():.3e} vs max|ref| {scale:.3e}"
    bad = err > tol * scale + rel * np.abs(w)
    assert not bad.any(), f"{name}: {bad.sum()} elements outside tolerance (first at {np.argwhere(bad)[0]})"


def _golden():
    z = np.load(f"{GOLDEN}/ssd.npz")
    keys = sorted({"/".join(k.split("/")[:2]) for k in z.files if k.startswith("ssd/")})
    out = []
    for key in keys:
        arrays = {k[len(key) + 1:]: z[k] for k in z.files if k.startswith(key + "/")}
        meta = ast.literal_eval(bytes(arrays.pop("meta")).decode())
        out.append(pytest.param(meta, arrays, id=key))
    return out


def _cuda(a, key, dtype=torch.float32):
    v = a.get(key)
    return None if v is None else torch.from_numpy(np.ascontiguousarray(v)).to("cuda", dtype)


@pytest.mark.parametrize("meta,a", _golden())
def test_ssd_matches_reference_fixture(meta, a):
    out, fin = mb.mamba_chunk_scan_combined(
        _cuda(a, "in_x", BF), _cuda(a, "in_dt"), _cuda(a, "in_A"), _cuda(a, "in_B", BF), _cuda(a, "in_C", BF),
        chunk_size=256, D=_cuda(a, "in_D"), z=_cuda(a, "in_z", BF), dt_bias=_cuda(a, "in_dt_bias"),
        dt_softplus=meta["dt_softplus"], return_final_states=True)
    torch.cuda.synchronize()
    assert out.dtype == BF and out.shape == a["in_x"].shape
    _close(out, a["out"], 1e-2, "out")
    _close(fin, a["final_states"], 5e-3, "final_states")


def _inputs(b, l, h, p, g, n, seed=0, regime="mamba2", has_z=True, has_bias=True, dmode="h", init=False):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(b, l, h, p, generator=gen).to(BF)
    B = torch.randn(b, l, g, n, generator=gen).to(BF)
    C = torch.randn(b, l, g, n, generator=gen).to(BF)
    z = torch.randn(b, l, h, p, generator=gen).to(BF) if has_z else None
    A = -(1.0 + 15.0 * torch.rand(h, generator=gen))
    if regime == "mamba2":
        dt = torch.randn(b, l, h, generator=gen) * 0.1 - 4.0
    else:
        dt = torch.randn(b, l, h, generator=gen) * 0.5
    dt_bias = torch.rand(h, generator=gen) * 0.5 if has_bias else None
    D = None if dmode is None else (torch.randn(h, generator=gen) if dmode == "h" else torch.randn(h, p, generator=gen))
    h0 = torch.randn(b, h, p, n, generator=gen) if init else None
    return dict(x=x, dt=dt, A=A, B=B, C=C, D=D, z=z, dt_bias=dt_bias, initial_states=h0)


def _run_both(inp, dt_softplus=True, dt_limit=(0.0, float("inf")), seq_idx=None):
    dev = {k: (None if v is None else v.cuda()) for k, v in inp.items()}
    out, fin = mb.mamba_chunk_scan_combined(dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], 128, D=dev["D"],
                                            z=dev["z"], dt_bias=dev["dt_bias"], initial_states=dev["initial_states"],
                                            seq_idx=None if seq_idx is None else seq_idx.cuda(),
                                            dt_softplus=dt_softplus, dt_limit=dt_limit, return_final_states=True)
    torch.cuda.synchronize()
    ref_out, ref_fin = f64.ssd_fwd(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"],
                                   inp["dt_bias"], inp["initial_states"], dt_softplus=dt_softplus, dt_limit=dt_limit,
                                   seq_idx=seq_idx)
    return out, fin, ref_out, ref_fin


@pytest.mark.parametrize("b,l,h,p,g,n", [
    (1, 1, 1, 32, 1, 16),      # one step
    (1, 127, 2, 32, 1, 64),    # one partial chunk
    (2, 128, 2, 64, 2, 128),   # one full chunk, groups
    (1, 129, 3, 32, 1, 8),     # a step into the second chunk, dstate 8
    (2, 1000, 4, 64, 2, 24),   # dstate 24 (odd number of 8-wide pieces)
    (1, 700, 2, 128, 1, 128),  # headdim 128 (4 CTAs per head)
    (3, 300, 4, 96, 4, 32),    # headdim 96, ngroups = nheads
])
@pytest.mark.parametrize("regime", ["mamba2", "wide"])
def test_ssd_matches_oracle_shapes(b, l, h, p, g, n, regime):
    inp = _inputs(b, l, h, p, g, n, seed=b * 7 + l, regime=regime)
    out, fin, ro, rf = _run_both(inp)
    _close(out, ro, 1e-2, "out")
    _close(fin, rf, 5e-3, "final_states")


@pytest.mark.parametrize("has_z,has_bias,dmode,init,softplus", [
    (False, False, None, False, True),
    (True, True, "hp", True, True),
    (False, True, "h", True, False),
    (True, False, "hp", False, False),
])
def test_ssd_feature_combinations(has_z, has_bias, dmode, init, softplus):
    inp = _inputs(2, 333, 2, 64, 1, 64, seed=5, regime="wide", has_z=has_z, has_bias=has_bias, dmode=dmode,
                  init=init)
    if not softplus:  # raw steps must stay positive (dt_limit's default lower bound is 0)
        inp["dt"] = inp["dt"].abs() * 0.2
    out, fin, ro, rf = _run_both(inp, dt_softplus=softplus)
    _close(out, ro, 1e-2, "out")
    _close(fin, rf, 5e-3, "final_states")


def test_ssd_dt_limit_clamps_steps():
    inp = _inputs(1, 260, 2, 32, 1, 32, seed=9, regime="wide")
    out, fin, ro, rf = _run_both(inp, dt_limit=(0.05, 0.3))
    _close(out, ro, 1e-2, "out")
    _close(fin, rf, 5e-3, "final_states")


@pytest.mark.parametrize("starts,first_id,init", [
    ([0, 37, 64, 65, 200, 201, 330], 0, True),   # mid-chunk, at a chunk start, 1-step sequences
    ([0, 128, 256], 0, False),                  # boundaries on chunk starts
    ([0, 100], 3, True),                        # first id not 0: the initial state is dropped
])
def test_ssd_packed_sequences(starts, first_id, init):
    """seq_idx: several sequences packed into each row; the oracle restarts the state at every id
    change (tests/test_oracle_golden.py checks that against separate runs)."""
    b, l = 2, 333
    inp = _inputs(b, l, 2, 64, 1, 64, seed=21, regime="wide", init=init)
    seq = torch.zeros(b, l, dtype=torch.int32)
    for r in range(b):
        for k, s0 in enumerate(starts):
            seq[r, s0 + r:] = first_id + k  # row 1 shifted by one step
    out, fin, ro, rf = _run_both(inp, seq_idx=seq)
    _close(out, ro, 1e-2, "out")
    _close(fin, rf, 5e-3, "final_states")


def test_ssd_strided_views_from_one_projection():
    """x, z, B and C as slices of one (b, l, width) projection (the Mamba-2 in_proj split), read in
    place; dt as a strided slice too."""
    b, l, h, p, g, n = 2, 300, 4, 64, 1, 64
    d = h * p
    gen = torch.Generator().manual_seed(11)
    width = 2 * d + 2 * g * n + h
    zxbcdt = torch.randn(b, l, width, generator=gen).to(BF).cuda()
    z, x = zxbcdt[..., :d].view(b, l, h, p), zxbcdt[..., d:2 * d].view(b, l, h, p)
    B = zxbcdt[..., 2 * d:2 * d + g * n].view(b, l, g, n)
    C = zxbcdt[..., 2 * d + g * n:2 * d + 2 * g * n].view(b, l, g, n)
    dt = torch.randn(b, l, 2 * h, generator=gen).cuda()[..., ::2]
    A = -(1.0 + 15.0 * torch.rand(h, generator=gen)).cuda()
    dt_bias = (torch.rand(h, generator=gen) * 0.5).cuda()
    out = mb.mamba_chunk_scan_combined(x, dt, A, B, C, 256, z=z, dt_bias=dt_bias, dt_softplus=True)
    torch.cuda.synchronize()
    ro, _ = f64.ssd_fwd(x.cpu(), dt.cpu(), A.cpu(), B.cpu(), C.cpu(), None, z.cpu(), dt_bias.cpu(), dt_softplus=True)
    _close(out, ro, 1e-2, "out")


def test_ssd_large_mamba2_shape():
    """Mamba-2 2.7B layer shape (headdim 64, dstate 128, one group) on 8 of its 80 heads, L = 4096."""
    inp = _inputs(2, 4096, 8, 64, 1, 128, seed=3, regime="mamba2", dmode="h")
    out, fin, ro, rf = _run_both(inp)
    _close(out, ro, 1e-2, "out")
    _close(fin, rf, 5e-3, "final_states")


def test_ssd_deterministic_and_errors():
    inp = _inputs(1, 200, 2, 32, 1, 16, seed=1)
    dev = {k: (None if v is None else v.cuda()) for k, v in inp.items()}
    args = (dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], 64)
    o1 = mb.mamba_chunk_scan_combined(*args, D=dev["D"], z=dev["z"], dt_bias=dev["dt_bias"], dt_softplus=True)
    o2 = mb.mamba_chunk_scan_combined(*args, D=dev["D"], z=dev["z"], dt_bias=dev["dt_bias"], dt_softplus=True)
    assert torch.equal(o1, o2)
    with pytest.raises(NotImplementedError):
        mb.mamba_chunk_scan_combined(dev["x"].float(), *args[1:])
    with pytest.raises(NotImplementedError):
        mb.mamba_chunk_scan_combined(*args, cu_seqlens=torch.tensor([0, 200], dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError):
        mb.mamba_chunk_scan_combined(*args, seq_idx=torch.zeros(1, 199, dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError):
        mb.mamba_chunk_scan_combined(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], 64)
    with pytest.raises(ValueError):
        mb.mamba_chunk_scan_combined(*args[:-1], 0)
    x = dev["x"].clone().requires_grad_()
    out = mb.mamba_chunk_scan_combined(x, *args[1:])
    with pytest.raises(NotImplementedError):
        out.float().sum().backward()


@pytest.mark.slow
def test_ssd_long_sequence_slice():
    """seqlen 65536 (1,024 chunks of carried state) on two heads of the 2.7B layer shape (headdim 64,
    dstate 128), in the Mamba-2 initialisation regime (long memory), against float64."""
    inp = _inputs(1, 65536, 2, 64, 1, 128, seed=31, regime="mamba2", dmode="h", init=True)
    out, fin, ro, rf = _run_both(inp)
    _close(out, ro, 1e-2, "out")
    _close(fin, rf, 5e-3, "final_states")


@pytest.mark.parametrize("b,l,h,p,g,n,init,seq", [
    (2, 333, 2, 64, 1, 64, True, False),
    (1, 700, 2, 128, 2, 128, False, False),
    (2, 300, 4, 32, 1, 24, False, True),
])
def test_ssd_fp16_inputs(b, l, h, p, g, n, init, seq):
    """fp16 x / z / B / C: the products run on fp16 operands (kind::f16 with the fp16 format)."""
    inp = _inputs(b, l, h, p, g, n, seed=41, regime="wide", init=init)
    for k in ("x", "z", "B", "C"):
        inp[k] = inp[k].float().to(torch.float16)
    seq_idx = None
    if seq:
        seq_idx = torch.zeros(b, l, dtype=torch.int32)
        seq_idx[:, 90:] = 1
        seq_idx[:, 200:] = 2
    out, fin, ro, rf = _run_both(inp, seq_idx=seq_idx)
    assert out.dtype == torch.float16
    _close(out, ro, 1e-2, "out")
    _close(fin, rf, 5e-3, "final_states")
