"""Generate the golden fixtures in this folder from the REFERENCE implementation itself.

Run in the build container, where the reference (SandyTheAdventurer/mamba-cpu) is mounted:

    make -C oracle ref                      # compiles the reference's csrc/selective_scan.cpp
    python tests/golden/make_golden.py      # writes tests/golden/*.npz

The reference's own, unmodified Python package is imported from ``$MAMBA_REF_DIR/src`` with
``oracle.ref_c`` (its compiled C++ kernel behind the ``mamba_cpu._C`` interface) injected as
``mamba_cpu._C``, because nanobind is not installed here. Each case stores its inputs, the
reference's outputs (``selective_scan_fn`` / ``causal_conv1d_fn`` / ``selective_state_update`` /
``causal_conv1d_update``, gradients through the reference's own autograd) and, for the scan
forward, the reference's pure-PyTorch oracle ``selective_scan_ref`` as well.

The cases follow the reference's test suite: tests/test_selective_scan.py (shapes, groups,
feature combos, low precision, extreme decay, exp range, NaN), tests/test_causal_conv1d.py and
tests/test_selective_state_update.py. Input distributions follow its make_inputs (:9-26).
The GPU tests and the float64 oracle are checked against these files; nothing at run time on a
GPU box needs the reference.
"""

import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
# The reference checkout: $MAMBA_REF_DIR, else a directory named `reference` beside this
# repository's checkout.
REF_DIR = os.environ.get("MAMBA_REF_DIR", os.path.join(os.path.dirname(ROOT), "reference"))


def _import_reference():
    sys.path.insert(0, ROOT)
    import oracle
    import oracle.ref_c as ref_c

    if not oracle.ref_available():
        oracle.build(ref=True)
    sys.modules["mamba_cpu._C"] = ref_c.as_module()
    sys.path.insert(0, os.path.join(REF_DIR, "src"))
    import mamba_cpu

    return mamba_cpu


def _np(t):
    if t is None:
        return None
    return t.detach().float().cpu().numpy().copy()


class Store:
    def __init__(self):
        self.d = {}
        self.n = 0

    def add(self, kind, meta, arrays):
        key = f"{kind}/{self.n:03d}"
        self.n += 1
        self.d[f"{key}/meta"] = np.frombuffer(repr(meta).encode(), dtype=np.uint8)
        for k, v in arrays.items():
            if v is not None:
                self.d[f"{key}/{k}"] = v

    def save(self, name):
        path = os.path.join(HERE, name)
        np.savez_compressed(path, **self.d)
        print(f"{path}: {len(self.d)} arrays, {os.path.getsize(path) / 1024:.0f} KiB")


def scan_inputs(batch, dim, seqlen, dstate, ngroups, has_D, has_z, has_bias, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)

    def normal(*shape):
        return torch.randn(*shape, generator=g).to(dtype)

    bc = (batch, dstate, seqlen) if ngroups is None else (batch, ngroups, dstate, seqlen)
    return dict(
        u=normal(batch, dim, seqlen),
        delta=(torch.rand(batch, dim, seqlen, generator=g) * 0.5).to(dtype),
        A=-torch.rand(dim, dstate, generator=g) - 0.5,
        B=normal(*bc),
        C=normal(*bc),
        D=torch.randn(dim, generator=g) if has_D else None,
        z=normal(batch, dim, seqlen) if has_z else None,
        delta_bias=torch.rand(dim, generator=g) * 0.1 if has_bias else None,
    )


def scan_case(m, st, inp, softplus, loss_on=("out", "last"), grads=True, dtype_name="f32", kind="matrix"):
    leaves = {k: (None if v is None else v.clone().requires_grad_(grads)) for k, v in inp.items()}
    out, last = m.selective_scan_fn(**leaves, delta_softplus=softplus, return_last_state=True)
    with torch.no_grad():
        out_t, last_t = m.selective_scan_ref(**inp, delta_softplus=softplus, return_last_state=True)
    arrays = {f"in_{k}": _np(v) for k, v in inp.items()}
    arrays.update(out=_np(out), last_state=_np(last))
    if inp["u"].numel() <= 2048:
        arrays.update(out_torch=_np(out_t), last_state_torch=_np(last_t))
    meta = dict(softplus=softplus, ngroups_given=inp["B"].dim() == 4, loss_on=tuple(loss_on),
                dtype=dtype_name, kind=kind)
    if grads:
        g = torch.Generator().manual_seed(1234)
        w_out = torch.randn(out.shape, generator=g) if "out" in loss_on else None
        w_last = torch.randn(last.shape, generator=g) if "last" in loss_on else None
        loss = 0
        if w_out is not None:
            loss = loss + (out.float() * w_out).sum()
        if w_last is not None:
            loss = loss + (last * w_last).sum()
        loss.backward()
        arrays.update(dout=_np(w_out), dlast_state=_np(w_last))
        for k, v in leaves.items():
            if v is not None:
                arrays[f"grad_{k}"] = _np(v.grad) if v.grad is not None else np.zeros(v.shape, np.float32)
    st.add("scan", meta, arrays)


def decay_inputs(x, seqlen=4, dstate=8):
    dim = x.shape[0]
    g = torch.Generator().manual_seed(0)
    return dict(
        u=torch.randn(1, dim, seqlen, generator=g),
        delta=torch.ones(1, dim, seqlen),
        A=x[:, None].expand(dim, dstate).contiguous(),
        B=torch.randn(1, dstate, seqlen, generator=g),
        C=torch.randn(1, dstate, seqlen, generator=g),
        D=None, z=None, delta_bias=None,
    )


def make_scan(m):
    st = Store()
    combos_f = [(False, False, False, False), (True, True, True, True), (True, False, True, False)]
    # forward matrix (reference tests/test_selective_scan.py:29-41)
    for shape in [(1, 4, 1, 1), (2, 16, 33, 16), (3, 32, 128, 8)]:
        for ngroups in [None, 1, 2]:
            for has_D, has_z, has_bias, softplus in combos_f:
                if shape[1] == 32 and (not has_z or ngroups != 2):
                    continue  # keep the fixture small: the largest shape once, every feature on
                inp = scan_inputs(*shape, ngroups, has_D, has_z, has_bias, torch.float32)
                scan_case(m, st, inp, softplus, grads=shape[1] <= 16)
    # backward matrix (reference :68-86)
    combos_b = [(False, False, False, False), (True, True, True, True), (True, False, False, True)]
    for shape in [(1, 4, 1, 1), (2, 8, 17, 4)]:
        for ngroups in [None, 2, 4]:
            if ngroups is not None and shape[1] % ngroups:
                continue
            for has_D, has_z, has_bias, softplus in combos_b:
                for loss_on in [("out", "last"), ("out",), ("last",)]:
                    inp = scan_inputs(*shape, ngroups, has_D, has_z, has_bias, torch.float32)
                    scan_case(m, st, inp, softplus, loss_on=loss_on)
    inp = scan_inputs(2, 32, 64, 16, 2, True, True, True, torch.float32)
    scan_case(m, st, inp, True)
    # low precision inputs (reference :44-50, :89-95)
    for dtype, name in [(torch.bfloat16, "bf16"), (torch.float16, "f16")]:
        inp = scan_inputs(2, 16, 64, 16, None, True, True, True, dtype)
        scan_case(m, st, inp, True, loss_on=("out",), dtype_name=name)
    # extreme decay (reference :142-163) and exp range (:166-175)
    for x in [-1e2, -1e4, -1e6, -1e8, -1e12, -1e20, -1e30, -3e38, -float("inf")]:
        scan_case(m, st, decay_inputs(torch.full((16,), x)), False, loss_on=("out",), kind="decay")
    xs = torch.cat([torch.linspace(-80, 0, 512), torch.linspace(0, 40, 128)])
    inp = decay_inputs(xs, seqlen=2)
    for k in ("u", "B", "C"):
        inp[k] = torch.ones_like(inp[k])
    scan_case(m, st, inp, False, grads=False, kind="exp_range")
    # NaN propagation (reference :178-183)
    inp = decay_inputs(torch.full((16,), -1.0))
    inp["delta"][0, 3, 1] = float("nan")
    scan_case(m, st, inp, False, grads=False, kind="nan")
    st.save("scan.npz")


def make_conv(m):
    st = Store()

    def conv_case(x, w, b, init, activation, final=False):
        leaves = [None if t is None else t.clone().requires_grad_() for t in (x, w, b, init)]
        res = m.causal_conv1d_fn(leaves[0], leaves[1], leaves[2], initial_states=leaves[3],
                                 return_final_states=final, activation=activation)
        out, fin = (res if final else (res, None))
        g = torch.Generator().manual_seed(99)
        dout = torch.randn(out.shape, generator=g)
        (out.float() * dout).sum().backward()
        arrays = dict(in_x=_np(x), in_weight=_np(w), in_bias=_np(b), in_initial_states=_np(init),
                      out=_np(out), final_states=_np(fin), dout=_np(dout))
        for name, t in zip(("x", "weight", "bias", "initial_states"), leaves):
            if t is not None:
                arrays[f"grad_{name}"] = _np(t.grad)
        st.add("conv", dict(activation=activation, final=final), arrays)

    # reference tests/test_causal_conv1d.py:7-16 (+ width 3, and initial states :19-26)
    for width in [2, 3, 4]:
        for activation in [None, "silu"]:
            for has_bias in [False, True]:
                torch.manual_seed(0)
                x = torch.randn(2, 8, 37)
                w = torch.randn(8, width)
                b = torch.randn(8) if has_bias else None
                conv_case(x, w, b, None, activation)
    torch.manual_seed(0)
    x = torch.randn(2, 8, 40)
    w = torch.randn(8, 4)
    init = torch.randn(2, 8, 3)
    conv_case(x, w, torch.randn(8), init, "silu", final=True)
    conv_case(x[..., :2], w, None, init, None, final=True)  # seqlen < width - 1
    # conv1d_update (reference :29-52)
    torch.manual_seed(0)
    for state_len in [3, 4, 6]:
        for seqlen in [None, 1, 5]:
            x = torch.randn(2, 8) if seqlen is None else torch.randn(2, 8, seqlen)
            w = torch.randn(8, 4)
            bias = torch.randn(8)
            state = torch.randn(2, 8, state_len)
            state0 = state.clone()
            out = m.causal_conv1d_update(x, state, w, bias, "silu")
            st.add("conv_update", dict(activation="silu"), dict(
                in_x=_np(x), in_conv_state=_np(state0), in_weight=_np(w), in_bias=_np(bias),
                out=_np(out), conv_state=_np(state)))
    st.save("conv.npz")


def make_state_update(m):
    st = Store()
    torch.manual_seed(0)
    for has_z, softplus in [(True, True), (False, False)]:
        for ngroups in [None, 2]:
            b, d, n = 2, 16, 8
            state = torch.randn(b, d, n)
            x, dt, z = torch.randn(b, d), torch.rand(b, d) * 0.5, torch.randn(b, d)
            A = -torch.rand(d, n) - 0.5
            B = torch.randn(b, n) if ngroups is None else torch.randn(b, ngroups, n)
            C = torch.randn_like(B)
            D, dt_bias = torch.randn(d), torch.rand(d) * 0.1
            state0 = state.clone()
            if ngroups is None:
                out = m.selective_state_update(state, x, dt, A, B, C, D, z if has_z else None,
                                               dt_bias, softplus)
            else:
                # multi-head layout with headdim 1 lets ngroups differ from 1 (:31-50)
                s4 = state.view(b, d, 1, n)
                out = m.selective_state_update(
                    s4, x.view(b, d, 1), dt.view(b, d, 1), A.view(d, 1, n), B, C,
                    D.view(d, 1), (z if has_z else x).view(b, d, 1) if has_z else None,
                    dt_bias.view(d, 1), softplus).view(b, d)
            st.add("state_update", dict(softplus=softplus, ngroups=ngroups), dict(
                in_state=_np(state0), in_x=_np(x), in_dt=_np(dt), in_A=_np(A), in_B=_np(B),
                in_C=_np(C), in_D=_np(D), in_z=_np(z) if has_z else None, in_dt_bias=_np(dt_bias),
                out=_np(out), state=_np(state)))
    st.save("state_update.npz")


def _bf16_exact(t):
    """Values representable in bfloat16 (the SSD kernel's input dtype), kept in float32."""
    return t.to(torch.bfloat16).float()


def make_ssd(m):
    """Mamba-2 SSD cases. The reference has no SSD scan (README.md:94 lists it as a roadmap item), but
    the SSD recurrence is its Mamba-1 selective scan with channels = nheads * headdim, A[h] repeated
    over dstate and dt[b, t, h] repeated over headdim, so the reference's own selective_scan_fn (its
    compiled kernel) produces the outputs and final states recorded here."""
    st = Store()
    cases = [
        # b, l, h, p, g, n, D mode, z, dt_bias, dt regime
        (1, 200, 2, 32, 1, 16, "h", True, True, "wide"),
        (2, 200, 2, 64, 2, 64, "hp", False, False, "wide"),
        (1, 130, 2, 32, 1, 128, None, True, False, "wide"),
        (2, 257, 2, 32, 2, 8, "h", True, True, "mamba2"),
        (1, 64, 1, 32, 1, 24, "hp", False, True, "mamba2"),
        (1, 260, 2, 64, 1, 128, "h", True, True, "mamba2"),
    ]
    for seed, (b, l, h, p, g, n, dmode, has_z, has_bias, regime) in enumerate(cases):
        gen = torch.Generator().manual_seed(100 + seed)
        x = _bf16_exact(torch.randn(b, l, h, p, generator=gen))
        B = _bf16_exact(torch.randn(b, l, g, n, generator=gen))
        C = _bf16_exact(torch.randn(b, l, g, n, generator=gen))
        z = _bf16_exact(torch.randn(b, l, h, p, generator=gen)) if has_z else None
        A = -(1.0 + 15.0 * torch.rand(h, generator=gen))  # Mamba-2 A = -exp(U(log 1, log 16)) range
        if regime == "wide":
            dt = torch.randn(b, l, h, generator=gen) * 0.5
            dt_bias = torch.rand(h, generator=gen) * 0.1 if has_bias else None
        else:  # Mamba-2 initialisation: softplus(dt_bias) in [1e-3, 1e-1], long memory
            dt = torch.randn(b, l, h, generator=gen) * 0.1
            tgt = torch.exp(torch.rand(h, generator=gen) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
            dt_bias = tgt + torch.log(-torch.expm1(-tgt)) if has_bias else None
            if not has_bias:
                dt = dt - 4.0
        D = None if dmode is None else (torch.randn(h, generator=gen) if dmode == "h" else
                                        torch.randn(h, p, generator=gen))
        u1 = x.permute(0, 2, 3, 1).reshape(b, h * p, l)
        d1 = dt.permute(0, 2, 1)[:, :, None, :].expand(b, h, p, l).reshape(b, h * p, l)
        A1 = A[:, None, None].expand(h, p, n).reshape(h * p, n)
        B1, C1 = B.permute(0, 2, 3, 1).contiguous(), C.permute(0, 2, 3, 1).contiguous()
        D1 = None if D is None else (D[:, None].expand(h, p) if D.dim() == 1 else D).reshape(h * p)
        z1 = None if z is None else z.permute(0, 2, 3, 1).reshape(b, h * p, l)
        b1 = None if dt_bias is None else dt_bias[:, None].expand(h, p).reshape(h * p)
        with torch.no_grad():
            out1, last1 = m.selective_scan_fn(u1.contiguous(), d1.contiguous(), A1.contiguous(), B1, C1,
                                              None if D1 is None else D1.contiguous(),
                                              None if z1 is None else z1.contiguous(),
                                              None if b1 is None else b1.contiguous(),
                                              delta_softplus=True, return_last_state=True)
        out = out1.reshape(b, h, p, l).permute(0, 3, 1, 2)
        final = last1.reshape(b, h, p, n)
        st.add("ssd", dict(dt_softplus=True, D=dmode, regime=regime), dict(
            in_x=_np(x), in_dt=_np(dt), in_A=_np(A), in_B=_np(B), in_C=_np(C), in_D=_np(D), in_z=_np(z),
            in_dt_bias=_np(dt_bias), out=_np(out), final_states=_np(final)))
    st.save("ssd.npz")


if __name__ == "__main__":
    mod = _import_reference()
    print("reference:", mod.__file__, "isa:", sys.modules["mamba_cpu._C"].cpu_isa())
    make_scan(mod)
    make_conv(mod)
    make_state_update(mod)
    make_ssd(mod)
