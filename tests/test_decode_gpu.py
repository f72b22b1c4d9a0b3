"""CUDA selective_state_update (decode) vs the float64 oracle and vs the full scan.

Follows mamba-cpu tests/test_selective_state_update.py (step-by-step == full scan, multi-head ==
flattened) and tests/test_upstream.py:87-104."""

import pytest
import torch

import mamba_cpu_b200 as mb
from helpers import assert_close
from oracle import f64

pytestmark = pytest.mark.gpu


def test_steps_match_full_scan():
    torch.manual_seed(0)
    batch, dim, seqlen, dstate = 2, 16, 10, 8
    u = torch.randn(batch, dim, seqlen).cuda()
    delta = (torch.rand(batch, dim, seqlen) * 0.5).cuda()
    A = (-torch.rand(dim, dstate) - 0.5).cuda()
    B = torch.randn(batch, dstate, seqlen).cuda()
    C = torch.randn(batch, dstate, seqlen).cuda()
    D = torch.randn(dim).cuda()
    z = torch.randn(batch, dim, seqlen).cuda()
    dt_bias = (torch.rand(dim) * 0.1).cuda()
    full, last = mb.selective_scan_fn(u, delta, A, B, C, D, z, dt_bias, True, return_last_state=True)
    state = torch.zeros(batch, dim, dstate, device="cuda")
    steps = [mb.selective_state_update(state, u[..., t], delta[..., t], A, B[..., t], C[..., t], D, z[..., t],
                                       dt_bias, True) for t in range(seqlen)]
    torch.testing.assert_close(torch.stack(steps, -1), full, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(state, last, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("multihead", [False, True])
@pytest.mark.parametrize("state_dtype", [torch.float32, torch.bfloat16])
def test_matches_oracle(multihead, state_dtype):
    torch.manual_seed(0)
    b, n = 2, 16
    lead = (4, 8) if multihead else (32,)
    state = torch.randn(b, *lead, n).to(state_dtype)
    x, dt, z = torch.randn(b, *lead), torch.rand(b, *lead), torch.randn(b, *lead)
    A = -torch.rand(*lead, n) - 0.5
    B = torch.randn(b, 2, n) if multihead else torch.randn(b, n)
    C = torch.randn_like(B)
    D, dt_bias = torch.randn(*lead), torch.rand(*lead)
    sg = state.cuda()
    out = mb.selective_state_update(sg, *[t.cuda() for t in (x, dt, A, B, C, D, z, dt_bias)], True)
    dim = 32
    o64, s64 = f64.state_update(state.reshape(b, dim, n), x.reshape(b, dim), dt.reshape(b, dim),
                                A.reshape(dim, n), B if multihead else B[:, None], C if multihead else C[:, None],
                                D.reshape(dim), z.reshape(b, dim), dt_bias.reshape(dim), True)
    tol = 1e-5 if state_dtype == torch.float32 else 1e-2
    assert_close(out.reshape(b, dim), o64, 1e-5 if state_dtype == torch.float32 else 2e-2, tol, "out")
    assert_close(sg.reshape(b, dim, n).float(), s64, tol, tol, "state")


def test_multihead_matches_flattened():
    torch.manual_seed(0)
    batch, nheads, headdim, dstate = 2, 4, 3, 8
    state = torch.randn(batch, nheads, headdim, dstate).cuda()
    x = torch.randn(batch, nheads, headdim).cuda()
    dt = torch.rand(batch, nheads, headdim).cuda()
    A = (-torch.rand(nheads, headdim, dstate)).cuda()
    B = torch.randn(batch, 1, dstate).cuda()
    C = torch.randn(batch, 1, dstate).cuda()
    D = torch.randn(nheads, headdim).cuda()
    flat_state = state.reshape(batch, -1, dstate).clone()
    out = mb.selective_state_update(state, x, dt, A, B, C, D)
    flat_out = mb.selective_state_update(flat_state, x.reshape(batch, -1), dt.reshape(batch, -1),
                                         A.reshape(-1, dstate), B[:, 0], C[:, 0], D.reshape(-1))
    torch.testing.assert_close(out.reshape(batch, -1), flat_out)
    torch.testing.assert_close(state.reshape(batch, -1, dstate), flat_state)


def test_rejects():
    st = torch.zeros(1, 4, 8).cuda()
    x = torch.zeros(1, 4).cuda()
    with pytest.raises(NotImplementedError):
        mb.selective_state_update(st, x, x, torch.zeros(4, 8).cuda(), torch.zeros(1, 8).cuda(),
                                  torch.zeros(1, 8).cuda(), state_batch_indices=torch.zeros(1).cuda())


@pytest.mark.parametrize("dstate", [40, 64, 128])
@pytest.mark.parametrize("state_dtype", [torch.float32, torch.bfloat16])
def test_wide_state_matches_oracle(dstate, state_dtype):
    """Mamba-2 decode shapes (multi-head layout, dstate 64 / 128 per head channel) on the wide-state
    kernel; the reference's PyTorch selective_state_update takes any dstate."""
    torch.manual_seed(1)
    b, h, p, n = 2, 3, 16, dstate
    state = torch.randn(b, h, p, n).to(state_dtype)
    x, z = torch.randn(b, h, p).to(torch.bfloat16), torch.randn(b, h, p).to(torch.bfloat16)
    dt = torch.rand(b, h, p).to(torch.bfloat16)
    A = -torch.rand(h, p, n) - 0.5
    B, C = torch.randn(b, 1, n).to(torch.bfloat16), torch.randn(b, 1, n).to(torch.bfloat16)
    D, dt_bias = torch.randn(h, p), torch.rand(h, p)
    sg = state.cuda()
    out = mb.selective_state_update(sg, *[t.cuda() for t in (x, dt, A, B, C, D, z, dt_bias)], True)
    dim = h * p
    o64, s64 = f64.state_update(state.reshape(b, dim, n), x.reshape(b, dim), dt.reshape(b, dim),
                                A.reshape(dim, n), B, C, D.reshape(dim), z.reshape(b, dim), dt_bias.reshape(dim), True)
    tol = 1e-5 if state_dtype == torch.float32 else 1e-2
    assert_close(out.reshape(b, dim).float(), o64, 2e-2, 2e-2 * max(1.0, abs(o64).max()), "out")
    assert_close(sg.reshape(b, dim, n).float(), s64, tol, tol, "state")


def test_ssd_prefill_then_decode_steps():
    """Mamba-2 generation: the SSD prefill's final state followed by decode steps of the multi-head
    selective_state_update gives the outputs of one longer prefill (bf16 tolerance)."""
    torch.manual_seed(2)
    b, l1, k, h, p, n = 2, 150, 5, 4, 32, 128
    bf = torch.bfloat16
    x = torch.randn(b, l1 + k, h, p).to(bf).cuda()
    z = torch.randn(b, l1 + k, h, p).to(bf).cuda()
    B = torch.randn(b, l1 + k, 1, n).to(bf).cuda()
    C = torch.randn(b, l1 + k, 1, n).to(bf).cuda()
    dt = (torch.randn(b, l1 + k, h) * 0.5).cuda()
    A = (-(1 + 15 * torch.rand(h))).cuda()
    D, dt_bias = torch.randn(h).cuda(), (torch.rand(h) * 0.5).cuda()
    full = mb.mamba_chunk_scan_combined(x, dt, A, B, C, 64, D=D, z=z, dt_bias=dt_bias, dt_softplus=True)
    _, state = mb.mamba_chunk_scan_combined(x[:, :l1], dt[:, :l1], A, B[:, :l1], C[:, :l1], 64, D=D, z=z[:, :l1],
                                            dt_bias=dt_bias, dt_softplus=True, return_final_states=True)
    A3 = A[:, None, None].expand(h, p, n)
    for t in range(l1, l1 + k):
        y = mb.selective_state_update(state, x[:, t], dt[:, t, :, None].expand(b, h, p), A3, B[:, t], C[:, t],
                                      D[:, None].expand(h, p), z=z[:, t], dt_bias=dt_bias[:, None].expand(h, p),
                                      dt_softplus=True)
        want = full[:, t].float()
        err = (y.float() - want).abs().max().item()
        assert err <= 2e-2 * want.abs().max().item() + 1e-3, f"step {t}: {err}"
