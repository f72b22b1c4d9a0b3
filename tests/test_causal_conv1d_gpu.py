"""CUDA causal conv1d (+ SiLU), its backward and decode step vs the float64 oracle.

Cases follow mamba-cpu tests/test_causal_conv1d.py (widths, activation, bias, state chaining,
update == full conv, final_states_out, dtypes) and tests/test_upstream.py:107-130 (width 3)."""

import numpy as np
import pytest
import torch

import mamba_cpu_b200 as mb
from helpers import assert_close, np64
from oracle import f64

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("width", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("activation", [None, "silu"])
@pytest.mark.parametrize("has_bias", [False, True])
@pytest.mark.parametrize("shape", [(2, 8, 37), (2, 64, 100), (1, 16, 1), (3, 24, 2048 + 13)])
def test_matches_oracle_fwd_bwd(width, activation, has_bias, shape):
    torch.manual_seed(0)
    x = torch.randn(*shape)
    w = torch.randn(shape[1], width)
    b = torch.randn(shape[1]) if has_bias else None
    xg, wg = x.cuda().requires_grad_(), w.cuda().requires_grad_()
    bg = b.cuda().requires_grad_() if b is not None else None
    out = mb.causal_conv1d_fn(xg, wg, bg, activation=activation)
    assert_close(out, f64.conv1d_fwd(x, w, b, None, activation), 1e-5, 1e-5, "out")
    dout = torch.randn(*shape)
    (out * dout.cuda()).sum().backward()
    g = f64.conv1d_bwd(x, w, b, None, activation, dout)
    assert_close(xg.grad, g["dx"], 1e-5, 1e-5, "dx")
    sc = max(1.0, float(np.abs(g["dweight"]).max()))
    assert_close(np64(wg.grad) / sc, g["dweight"] / sc, 1e-5, 1e-5, "dweight")
    if b is not None:
        sc = max(1.0, float(np.abs(g["dbias"]).max()))
        assert_close(np64(bg.grad) / sc, g["dbias"] / sc, 1e-5, 1e-5, "dbias")


_BATCHED = [
    ((8, 32, 256), torch.float32), ((8, 32, 256), torch.bfloat16),
    ((9, 16, 2048 + 64), torch.float32), ((9, 16, 2048 + 64), torch.bfloat16),
    # rows of 16-byte but not 32-byte multiples: the thread covering the row end stages a
    # partial span (cp.async copies mixed with plain stores)
    ((8, 16, 2052), torch.float32), ((8, 16, 2056), torch.bfloat16),
]


@pytest.mark.parametrize("width", [2, 4, 8])
@pytest.mark.parametrize("with_init", [False, True])
@pytest.mark.parametrize("shape,dtype", _BATCHED)
@pytest.mark.parametrize("activation,has_bias", [("silu", True), (None, False)])
def test_batched_pipeline_matches_oracle(width, with_init, shape, dtype, activation, has_bias):
    """Batches of 8 or more with 16-byte aligned rows take the forward and backward that stream a
    channel's batch rows through shared memory (several CTAs per row and a partial last span in
    the larger shapes); they must agree with the float64 oracle like the register-load kernels."""
    torch.manual_seed(3)
    x = torch.randn(*shape).to(dtype)
    w = torch.randn(shape[1], width)
    b = torch.randn(shape[1]) if has_bias else None
    init = torch.randn(shape[0], shape[1], width - 1).to(dtype) if with_init else None
    leaves = [t.cuda().requires_grad_() if t is not None else None for t in (x, w, b, init)]
    out, fin = mb.causal_conv1d_fn(leaves[0], leaves[1], leaves[2], initial_states=leaves[3], activation=activation,
                                   return_final_states=True)
    xf, initf = x.float(), (init.float() if init is not None else None)
    o64, fin64 = f64.conv1d_fwd(xf, w, b, initf, activation, return_final_states=True)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert_close(out.float(), o64, tol, tol, "out")
    assert_close(fin.float(), fin64, 0, 0, "final_states")
    dout = torch.randn(*shape).to(dtype)
    (out * dout.cuda()).sum().backward()
    g = f64.conv1d_bwd(xf, w, b, initf, activation, dout.float())
    assert_close(leaves[0].grad.float(), g["dx"], tol, tol, "dx")
    grads = [(leaves[1], "dweight")] + ([(leaves[2], "dbias")] if has_bias else [])
    for t, k in grads:
        sc = max(1.0, float(np.abs(g[k]).max()))
        assert_close(np64(t.grad) / sc, g[k] / sc, tol, tol, k)
    if with_init:
        assert_close(leaves[3].grad.float(), g["dinitial_states"], tol, tol, "dinitial_states")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_final_states_gradient_rounds_once(dtype):
    """With return_final_states, the gradient flowing into final_states is added to dx in fp32 and
    rounded to x's dtype once: dx equals the float64 gradient of out and final_states together."""
    torch.manual_seed(4)
    x = torch.randn(2, 16, 64).to(dtype)
    w = torch.randn(16, 4)
    xg, wg = x.cuda().requires_grad_(), w.cuda().requires_grad_()
    out, fin = mb.causal_conv1d_fn(xg, wg, activation="silu", return_final_states=True)
    dout = torch.randn(2, 16, 64).to(dtype)
    dfin = torch.randn(2, 16, 3)  # fp32 upstream gradient of the final states
    torch.autograd.backward([out, fin], [dout.cuda(), dfin.cuda().to(fin.dtype)])
    want = f64.conv1d_bwd(x.float(), w, None, None, "silu", dout.float())["dx"]
    want[..., -3:] += np64(dfin.to(fin.dtype))
    tol = 1e-5 if dtype == torch.float32 else 8e-3
    assert_close(xg.grad.float(), want, tol, tol, "dx")


def test_initial_and_final_states_chain():
    torch.manual_seed(0)
    x = torch.randn(2, 8, 40).cuda()
    w = torch.randn(8, 4).cuda()
    full = mb.causal_conv1d_fn(x, w, activation="silu")
    a, state = mb.causal_conv1d_fn(x[..., :25], w, activation="silu", return_final_states=True)
    b = mb.causal_conv1d_fn(x[..., 25:], w, initial_states=state, activation="silu")
    torch.testing.assert_close(torch.cat([a, b], -1), full)


@pytest.mark.parametrize("seqlen", [1, 2, 3, 40])
def test_initial_states_gradients(seqlen):
    torch.manual_seed(1)
    x, w, bias, init = torch.randn(2, 8, seqlen), torch.randn(8, 4), torch.randn(8), torch.randn(2, 8, 3)
    leaves = [t.cuda().requires_grad_() for t in (x, w, bias, init)]
    out, fin = mb.causal_conv1d_fn(leaves[0], leaves[1], leaves[2], initial_states=leaves[3],
                                   return_final_states=True, activation="silu")
    o64, f64s = f64.conv1d_fwd(x, w, bias, init, "silu", return_final_states=True)
    assert_close(out, o64, 1e-5, 1e-5, "out")
    assert_close(fin, f64s, 0, 0, "final_states")
    dout = torch.randn(2, 8, seqlen)
    (out * dout.cuda()).sum().backward()
    g = f64.conv1d_bwd(x, w, bias, init, "silu", dout)
    for t, k in zip(leaves, ("dx", "dweight", "dbias", "dinitial_states")):
        assert_close(t.grad, g[k], 1e-5, 1e-5, k)


def test_final_states_gradient_flows():
    torch.manual_seed(2)
    x = torch.randn(1, 4, 2).cuda().requires_grad_()
    init = torch.randn(1, 4, 3).cuda().requires_grad_()
    w = torch.randn(4, 4).cuda()
    _, fin = mb.causal_conv1d_fn(x, w, initial_states=init, return_final_states=True)
    fin.sum().backward()
    # final = [init | x][-3:] = init[..., 2:] ++ x
    assert torch.equal(x.grad, torch.ones_like(x))
    assert torch.equal(init.grad[..., 2:], torch.ones(1, 4, 1, device="cuda"))
    assert not init.grad[..., :2].any()


def test_final_states_out_buffer():
    x = torch.randn(2, 8, 10).cuda()
    w = torch.randn(8, 4).cuda()
    buf = torch.empty(2, 8, 3, device="cuda")
    _, final = mb.causal_conv1d_fn(x, w, return_final_states=True, final_states_out=buf)
    assert final is buf
    torch.testing.assert_close(buf, x[..., -3:])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_low_precision_dtypes(dtype):
    torch.manual_seed(0)
    x = torch.randn(2, 64, 300).to(dtype)
    w, b = torch.randn(64, 4), torch.randn(64)
    out = mb.causal_conv1d_fn(x.cuda(), w.cuda(), b.cuda(), activation="silu")
    assert out.dtype == dtype
    assert_close(out, f64.conv1d_fwd(x, w, b, None, "silu"), 1e-2, 1e-2, "out")


def test_rejects():
    x, w = torch.randn(1, 4, 8).cuda(), torch.randn(4, 4).cuda()
    with pytest.raises(NotImplementedError):
        mb.causal_conv1d_fn(x, w, seq_idx=torch.zeros(1, 8, dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError):
        mb.causal_conv1d_fn(x, w, activation="relu")
    with pytest.raises(ValueError):
        mb.causal_conv1d_fn(x.cpu(), w.cpu())


def test_update_matches_full_conv():
    torch.manual_seed(0)
    x = torch.randn(2, 8, 12).cuda()
    w = torch.randn(8, 4).cuda()
    bias = torch.randn(8).cuda()
    full = mb.causal_conv1d_fn(x, w, bias, activation="silu")
    state = torch.zeros(2, 8, 4, device="cuda")
    steps = [mb.causal_conv1d_update(x[..., t], state, w, bias, "silu") for t in range(12)]
    torch.testing.assert_close(torch.stack(steps, -1), full, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("state_len", [3, 4, 6, 7])
@pytest.mark.parametrize("seqlen", [1, 3, 5])
def test_update_multi_token_matches_oracle(state_len, seqlen):
    torch.manual_seed(0)
    x = torch.randn(2, 64, seqlen)
    w, bias = torch.randn(64, 4), torch.randn(64)
    state = torch.randn(2, 64, state_len)
    sg = state.cuda()
    out = mb.causal_conv1d_update(x.cuda(), sg, w.cuda(), bias.cuda(), "silu")
    o64, s64 = f64.conv1d_update(x, state, w, bias, "silu")
    assert_close(out, o64, 1e-5, 1e-5, "out")
    assert_close(sg, s64, 0, 0, "conv_state")


def test_update_rejects():
    x, st, w = torch.randn(1, 4).cuda(), torch.zeros(1, 4, 2).cuda(), torch.randn(4, 4).cuda()
    with pytest.raises(ValueError):
        mb.causal_conv1d_update(x, st, w)
    with pytest.raises(NotImplementedError):
        mb.causal_conv1d_update(x, torch.zeros(1, 4, 3).cuda(), w, cache_seqlens=torch.zeros(1).cuda())


def _conv_f64_cuda(x, w, b, silu):
    """Causal depthwise conv (+ SiLU) evaluated in float64 on the GPU, differentiable."""
    W, L = w.shape[1], x.shape[-1]
    xp = torch.nn.functional.pad(x, (W - 1, 0))
    out = sum(w[:, k, None] * xp[..., k:k + L] for k in range(W))
    if b is not None:
        out = out + b[:, None]
    return torch.nn.functional.silu(out) if silu else out


@pytest.mark.parametrize("b,d,l,dtype", [(4, 1536, 1024, torch.float32), (8, 4096, 2048, torch.bfloat16)])
def test_full_size_configs(b, d, l, dtype):
    """The conv1d of BASELINE config 2 (fp32, batch 4, d_inner 1536, seqlen 1024) and of a config-4
    layer (bf16, batch 8, d_inner 4096, seqlen 2048) at full size, width 4 with bias and SiLU,
    forward and backward, against a float64 evaluation on the GPU."""
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(b, d, l, device="cuda", generator=g).to(dtype)
    w = torch.randn(d, 4, device="cuda", generator=g) * 0.5
    bias = torch.randn(d, device="cuda", generator=g)
    dy = torch.randn(b, d, l, device="cuda", generator=g).to(dtype)
    leaves = [t.clone().requires_grad_() for t in (x, w, bias)]
    out = mb.causal_conv1d_fn(*leaves, activation="silu")
    out.backward(dy)
    ref64 = [t.double().requires_grad_() for t in (x, w, bias)]
    o64 = _conv_f64_cuda(*ref64, True)
    o64.backward(dy.double())
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert_close(out.float(), o64, tol, tol, "out")
    assert_close(leaves[0].grad.float(), ref64[0].grad, tol, tol, "dx")
    for t, r, k in ((leaves[1], ref64[1], "dweight"), (leaves[2], ref64[2], "dbias")):
        sc = max(1.0, float(r.grad.abs().max()))
        # sums over batch x seqlen (4M / 16M terms): fp32 accumulation order against float64
        assert_close(t.grad.double() / sc, r.grad / sc, 1e-4, 1e-5, k)
