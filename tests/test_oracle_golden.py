"""Pins the float64 oracle (oracle/oracle.c) to the REFERENCE's own outputs.

The fixtures in tests/golden/ were produced by the unmodified reference package running on its
own compiled C++ kernel (tests/golden/make_golden.py). The oracle must reproduce them to the
reference kernel's fp32 precision before the GPU parity tests may trust it. CPU only.
"""

import ast

import numpy as np
import pytest
import torch

from helpers import assert_close
from oracle import f64

GOLDEN = __import__("os").path.join(__import__("os").path.dirname(__file__), "golden")


def _cases(name, kind):
    z = np.load(f"{GOLDEN}/{name}.npz")
    keys = sorted({"/".join(k.split("/")[:2]) for k in z.files if k.startswith(kind + "/")})
    out = []
    for key in keys:
        arrays = {k[len(key) + 1:]: z[k] for k in z.files if k.startswith(key + "/")}
        meta = ast.literal_eval(bytes(arrays.pop("meta")).decode())
        out.append(pytest.param(meta, arrays, id=key))
    return out


def _get(a, k):
    return a.get(k)


@pytest.mark.parametrize("meta,a", _cases("scan", "scan"))
def test_scan_oracle_matches_reference(meta, a):
    args = [_get(a, "in_" + k) for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")]
    out, last = f64.scan_fwd(*args, delta_softplus=meta["softplus"])
    # the reference kernel is fp32 with a polynomial exp (~1-2 ulp): compare at its precision
    rtol, atol = (1e-5, 1e-5) if meta["dtype"] == "f32" else (1e-2, 1e-2)
    if meta["dtype"] != "f32":
        # low-precision cases: the reference rounds its fp32 output to bf16 / fp16
        out = torch.from_numpy(out).to(torch.bfloat16 if meta["dtype"] == "bf16" else torch.float16).double().numpy()
    assert_close(out, a["out"], rtol, atol, "out")
    assert_close(last, a["last_state"], 1e-5, 1e-5, "last_state")
    if "out_torch" in a:  # the reference's pure-torch oracle agrees too
        assert_close(f64.scan_fwd(*args, delta_softplus=meta["softplus"])[0], a["out_torch"],
                     1e-4 if meta["dtype"] == "f32" else 1e-2, 1e-4 if meta["dtype"] == "f32" else 1e-2)
    if "grad_u" not in a:
        return
    dout = a.get("dout")
    if dout is None:
        dout = np.zeros_like(a["in_u"], dtype=np.float32)
    g = f64.scan_bwd(*args, meta["softplus"], dout, a.get("dlast_state"))
    tol = (1e-4, 1e-4) if meta["dtype"] == "f32" else (3e-2, 3e-2)
    pairs = [("u", "du"), ("delta", "ddelta"), ("A", "dA"), ("B", "dB"), ("C", "dC"),
             ("D", "dD"), ("z", "dz"), ("delta_bias", "ddelta_bias")]
    for k, gk in pairs:
        if "grad_" + k not in a:
            continue
        if meta["kind"] == "decay" and k not in ("u", "B", "C"):
            # At dt*A <= -87 the reference's exp clamps to exp(-87) instead of 0
            # (selective_scan.cpp:68), which leaks an O(A * 1e-38) artifact into ddelta / dA; its
            # own extreme-decay test compares du, dB, dC only (tests/test_selective_scan.py:151-163).
            continue
        want = a["grad_" + k]
        got = g[gk].reshape(want.shape)
        scale = max(1.0, float(np.abs(want).max()))
        assert_close(got / scale, want / scale, *tol, name=k)


@pytest.mark.parametrize("meta,a", _cases("conv", "conv"))
def test_conv_oracle_matches_reference(meta, a):
    act = meta["activation"]
    res = f64.conv1d_fwd(a["in_x"], a["in_weight"], a.get("in_bias"), a.get("in_initial_states"), act,
                         return_final_states=meta["final"])
    out, fin = res if meta["final"] else (res, None)
    assert_close(out, a["out"], 1e-5, 1e-5, "out")
    if meta["final"]:
        assert_close(fin, a["final_states"], 0, 0, "final_states")
    g = f64.conv1d_bwd(a["in_x"], a["in_weight"], a.get("in_bias"), a.get("in_initial_states"), act, a["dout"])
    for k, gk in (("x", "dx"), ("weight", "dweight"), ("bias", "dbias"), ("initial_states", "dinitial_states")):
        if "grad_" + k in a:
            want = a["grad_" + k]
            # the reference output also depends on final_states only through out here
            assert_close(g[gk], want, 1e-4, 1e-4, k)


@pytest.mark.parametrize("meta,a", _cases("conv", "conv_update"))
def test_conv_update_oracle_matches_reference(meta, a):
    out, st = f64.conv1d_update(a["in_x"], a["in_conv_state"], a["in_weight"], a.get("in_bias"), meta["activation"])
    assert_close(out, a["out"], 1e-5, 1e-5, "out")
    assert_close(st, a["conv_state"], 0, 0, "conv_state")


@pytest.mark.parametrize("meta,a", _cases("state_update", "state_update"))
def test_state_update_oracle_matches_reference(meta, a):
    out, st = f64.state_update(a["in_state"], a["in_x"], a["in_dt"], a["in_A"], a["in_B"], a["in_C"],
                               a.get("in_D"), a.get("in_z"), a.get("in_dt_bias"), meta["softplus"])
    assert_close(out, a["out"], 1e-5, 1e-5, "out")
    assert_close(st, a["state"], 1e-5, 1e-5, "state")


def test_oracle_is_deterministic_across_thread_counts():
    from helpers import make_inputs

    inp = make_inputs(2, 32, 70, 16, 2, True, True, True, torch.float32)
    args = [inp[k] for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")]
    dout = torch.randn(2, 32, 70, generator=torch.Generator().manual_seed(3))
    try:
        f64.set_num_threads(1)
        a = f64.scan_bwd(*args, True, dout)
        f64.set_num_threads(5)
        b = f64.scan_bwd(*args, True, dout)
    finally:
        f64.set_num_threads(0)
    for k in a:
        if a[k] is not None:
            assert np.array_equal(a[k], b[k]), k


@pytest.mark.parametrize("meta,a", _cases("ssd", "ssd"))
def test_ssd_oracle_matches_reference(meta, a):
    """The float64 SSD recurrence against the reference's own kernel run on the equivalent Mamba-1
    problem (channels = nheads * headdim; tests/golden/make_golden.py:make_ssd)."""
    out, fin = f64.ssd_fwd(a["in_x"], a["in_dt"], a["in_A"], a["in_B"], a["in_C"], a.get("in_D"), a.get("in_z"),
                           a.get("in_dt_bias"), dt_softplus=meta["dt_softplus"])
    assert_close(out, a["out"], 1e-4, 1e-5, "out", norm_tol=1e-5)
    assert_close(fin, a["final_states"], 1e-4, 1e-5, "final_states", norm_tol=1e-5)


def test_ssd_oracle_packed_sequences_equal_separate_runs():
    """seq_idx semantics of the float64 SSD oracle: a row packing several sequences gives, on each
    sequence, exactly the oracle's run of that sequence alone (zero state at its start; the initial
    state only for sequence 0), so the packed oracle inherits the pinning of the plain one."""
    rng = np.random.default_rng(7)
    b, l, h, p, g, n = 2, 50, 2, 4, 1, 8
    x = rng.standard_normal((b, l, h, p)).astype(np.float32)
    dt = (rng.standard_normal((b, l, h)) * 0.5).astype(np.float32)
    A = -(1 + 15 * rng.random(h)).astype(np.float32)
    B = rng.standard_normal((b, l, g, n)).astype(np.float32)
    C = rng.standard_normal((b, l, g, n)).astype(np.float32)
    z = rng.standard_normal((b, l, h, p)).astype(np.float32)
    D = rng.standard_normal(h).astype(np.float32)
    h0 = rng.standard_normal((b, h, p, n)).astype(np.float32)
    bounds = [(0, 0, 13, 0), (0, 13, 14, 1), (0, 14, 50, 4), (1, 0, 30, 2), (1, 30, 50, 3)]  # (row, start, end, id)
    seq = np.zeros((b, l), np.int32)
    for r, s0, s1, sid in bounds:
        seq[r, s0:s1] = sid
    out, fin = f64.ssd_fwd(x, dt, A, B, C, D, z, None, h0, dt_softplus=True, seq_idx=seq)
    for r, s0, s1, sid in bounds:
        sl = slice(s0, s1)
        init = h0[r:r + 1] if (s0 == 0 and sid == 0) else None
        o1, f1 = f64.ssd_fwd(x[r:r + 1, sl], dt[r:r + 1, sl], A, B[r:r + 1, sl], C[r:r + 1, sl], D, z[r:r + 1, sl],
                             None, init, dt_softplus=True)
        np.testing.assert_allclose(out[r:r + 1, sl], o1, rtol=1e-12, atol=1e-12)
        if s1 == l:
            np.testing.assert_allclose(fin[r:r + 1], f1, rtol=1e-12, atol=1e-12)
