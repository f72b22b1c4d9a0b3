"""The CUDA path against the reference's own outputs (tests/golden/*.npz, produced by the
unmodified mamba-cpu package on its compiled C++ kernel by tests/golden/make_golden.py).

The tolerances are the reference suite's own (1e-5 forward / 1e-4 backward for float32, 1e-2 /
2e-2 for half precision); gradients are compared after dividing by max(|reference|, 1) as
mamba-cpu's tests/test_upstream.py:72-75 does."""

import ast
import os

import numpy as np
import pytest
import torch

import mamba_cpu_b200 as mb
from helpers import assert_close, np64

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
KEYS = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")
DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _cases(name, kind):
    z = np.load(f"{GOLDEN}/{name}.npz")
    keys = sorted({"/".join(k.split("/")[:2]) for k in z.files if k.startswith(kind + "/")})
    out = []
    for key in keys:
        arrays = {k[len(key) + 1:]: z[k] for k in z.files if k.startswith(key + "/")}
        meta = ast.literal_eval(bytes(arrays.pop("meta")).decode())
        out.append(pytest.param(meta, arrays, id=key))
    return out


@pytest.mark.parametrize("meta,a", _cases("scan", "scan"))
def test_scan_matches_reference_fixture(meta, a):
    dt = DT[meta["dtype"]]
    leaves = {}
    for k in KEYS:
        v = a.get("in_" + k)
        if v is None:
            leaves[k] = None
            continue
        t = torch.from_numpy(v)
        if k in ("u", "delta", "B", "C", "z"):
            t = t.to(dt)
        leaves[k] = t.cuda().requires_grad_("grad_u" in a)
    out, last = mb.selective_scan_fn(**leaves, delta_softplus=meta["softplus"], return_last_state=True)
    f32 = meta["dtype"] == "f32"
    assert_close(out, a["out"], 1e-5 if f32 else 1e-2, 1e-5 if f32 else 1e-2, "out")
    assert_close(last, a["last_state"], 1e-5 if f32 else 1e-2, 1e-5 if f32 else 1e-2, "last_state")
    if "grad_u" not in a:
        return
    loss = 0
    if a.get("dout") is not None:
        loss = loss + (out.float() * torch.from_numpy(a["dout"]).cuda()).sum()
    if a.get("dlast_state") is not None:
        loss = loss + (last * torch.from_numpy(a["dlast_state"]).cuda()).sum()
    loss.backward()
    tol = 1e-4 if f32 else 2e-2
    for k in KEYS:
        if leaves[k] is None:
            continue
        if meta["kind"] == "decay" and k not in ("u", "B", "C"):
            continue  # reference's exp clamp artifact (see test_oracle_golden.py)
        want = a["grad_" + k]
        got = leaves[k].grad
        if got is None:
            assert not np.any(want), k
            continue
        scale = max(1.0, float(np.abs(want).max()))
        assert_close(np64(got) / scale, want / scale, tol, tol, k)


@pytest.mark.parametrize("meta,a", _cases("conv", "conv"))
def test_conv_matches_reference_fixture(meta, a):
    names = ("x", "weight", "bias", "initial_states")
    leaves = [None if a.get("in_" + k) is None else torch.from_numpy(a["in_" + k]).cuda().requires_grad_()
              for k in names]
    res = mb.causal_conv1d_fn(leaves[0], leaves[1], leaves[2], initial_states=leaves[3],
                              return_final_states=meta["final"], activation=meta["activation"])
    out, fin = res if meta["final"] else (res, None)
    assert_close(out, a["out"], 1e-5, 1e-5, "out")
    if meta["final"]:
        assert_close(fin, a["final_states"], 0, 0, "final_states")
    (out * torch.from_numpy(a["dout"]).cuda()).sum().backward()
    for k, t in zip(names, leaves):
        if t is not None:
            assert_close(t.grad, a["grad_" + k], 1e-4, 1e-4, k)


@pytest.mark.parametrize("meta,a", _cases("conv", "conv_update"))
def test_conv_update_matches_reference_fixture(meta, a):
    st = torch.from_numpy(a["in_conv_state"]).cuda()
    out = mb.causal_conv1d_update(torch.from_numpy(a["in_x"]).cuda(), st, torch.from_numpy(a["in_weight"]).cuda(),
                                  torch.from_numpy(a["in_bias"]).cuda(), meta["activation"])
    assert_close(out, a["out"], 1e-5, 1e-5, "out")
    assert_close(st, a["conv_state"], 0, 0, "conv_state")


@pytest.mark.parametrize("meta,a", _cases("state_update", "state_update"))
def test_state_update_matches_reference_fixture(meta, a):
    g = lambda k: None if a.get("in_" + k) is None else torch.from_numpy(a["in_" + k]).cuda()  # noqa: E731
    st = g("state")
    if meta["ngroups"] is None:
        out = mb.selective_state_update(st, g("x"), g("dt"), g("A"), g("B"), g("C"), g("D"), g("z"), g("dt_bias"),
                                        meta["softplus"])
    else:
        b, d, n = st.shape
        s4 = st.view(b, d, 1, n)
        z = g("z")
        out = mb.selective_state_update(s4, g("x").view(b, d, 1), g("dt").view(b, d, 1), g("A").view(d, 1, n),
                                        g("B"), g("C"), g("D").view(d, 1), None if z is None else z.view(b, d, 1),
                                        g("dt_bias").view(d, 1), meta["softplus"]).view(b, d)
    assert_close(out, a["out"], 1e-5, 1e-5, "out")
    assert_close(st, a["state"], 1e-5, 1e-5, "state")
