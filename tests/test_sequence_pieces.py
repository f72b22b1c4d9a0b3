"""Sequence pieces inside one GPU: rows cut into runs of whole 64-step chunks, each run by its own
CTAs, every piece starting from the state (forward) or adjoint (backward) its neighbours' summaries
compose to. The scans split rows only when whole rows leave most of the GPU's resident CTA slots
empty -- a small batch x dim, such as one rank's shard of a dim-sharded problem (the reference
parallelises over rows only, csrc/selective_scan.cpp:320-324).

CPU: the automatic choice of the piece count. GPU: with the count forced (2, 3, 5 pieces, partial
last pieces and chunks, groups, gate, bias, softplus on and off, initial states, strided views,
bf16), every output and gradient against the float64 oracle at the usual tolerances, and against
the same call on whole rows to rounding.
"""

import numpy as np
import pytest
import torch

from mamba_cpu_b200 import _lib



def test_automatic_piece_count():
    """The modelled-cost choice: (1 + s (G-1)/G) ceil(G w) / (G w) over G = 1..8, w = CTAs / slots,
    s = 0.8 (forward) / 0.23 (backward), at least 4 chunks per piece, a split gaining 2 %."""
    if torch.cuda.is_available():
        pytest.skip("the rule's slot count comes from the GPU here")
    pieces = _lib.lib.mb200_sequence_pieces
    # config 5 on one GPU (640 CTAs, 1.44 rounds of the 444 slots): the backward splits in two
    assert (pieces(640, 1024, 0), pieces(640, 1024, 1)) == (1, 2)
    assert (pieces(384, 16, 0), pieces(384, 16, 1)) == (1, 1)      # config 2 (0.86 rounds)
    assert (pieces(80, 1024, 0), pieces(80, 1024, 1)) == (5, 5)    # one rank's shard at 8 ranks
    assert pieces(10, 1024, 1) == 8                                # at most 8
    assert pieces(10, 12, 1) == 3                                  # at least 4 chunks per piece
    assert pieces(10, 3, 1) == 1
    assert pieces(0, 100, 1) == 1
    _lib.set_sequence_pieces(3)
    try:
        assert pieces(640, 1024, 0) == 3  # forced
        assert pieces(640, 2, 1) == 2     # never more pieces than chunks
    finally:
        _lib.set_sequence_pieces(0)
    assert pieces(640, 1024, 0) == 1


def _fwd_params(batch, dim, seqlen, dstate=16):
    p = _lib.ScanFwdParams()
    p.u = p.delta = p.A = p.B = p.C = p.out = 0x1000
    p.batch, p.dim, p.seqlen, p.dstate, p.ngroups = batch, dim, seqlen, dstate, 1
    p.B_batch_stride = p.C_batch_stride = dstate * seqlen
    p.B_group_stride = p.C_group_stride = dstate * seqlen
    p.B_dstate_stride = p.C_dstate_stride = seqlen
    p.B_seqlen_stride = p.C_seqlen_stride = 1
    return p


def test_forward_keeps_short_rows_whole():
    """Short rows of small problems (under 64 chunks and 4096 rows) are not split by the automatic
    choice: the forward's piece summaries would need workspace, and there is none (BASELINE
    config 1's shape); a forced count still splits them, and long rows of few channels still split."""
    if torch.cuda.is_available():
        pytest.skip("the long-row case's slot count comes from the GPU here")
    ws = _lib.lib.mb200_selective_scan_fwd_workspace_size
    assert ws(_fwd_params(1, 1536, 2048)) == 0           # config 1: whole rows
    _lib.set_sequence_pieces(2)
    try:
        assert ws(_fwd_params(1, 1536, 2048)) > 0        # forced: split
    finally:
        _lib.set_sequence_pieces(0)
    assert ws(_fwd_params(2, 640, 65536)) > 0            # one rank's config-5 shard at 8 ranks


# ---------------------------------------------------------------------------------------------
# GPU parity

KEYS = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")
GRAD_OF = {"u": "du", "delta": "ddelta", "A": "dA", "B": "dB", "C": "dC", "D": "dD", "z": "dz",
           "delta_bias": "ddelta_bias"}


class _Pieces:
    def __init__(self, n):
        self.n = n

    def __enter__(self):
        _lib.set_sequence_pieces(self.n)

    def __exit__(self, *exc):
        _lib.set_sequence_pieces(0)


def _run(inp, softplus, w_out, w_last, pieces):
    import mamba_cpu_b200 as mb
    from helpers import to_cuda

    leaves = to_cuda(inp, requires_grad=True)
    with _Pieces(pieces):
        out, last = mb.selective_scan_fn(**leaves, delta_softplus=softplus, return_last_state=True)
        loss = (out.float() * w_out.cuda()).sum() + (last * w_last.cuda()).sum()
        loss.backward()
    torch.cuda.synchronize()
    grads = {k: (None if v is None else v.grad.detach().clone()) for k, v in leaves.items()}
    return out.detach(), last.detach(), grads


CASES = [
    # batch, dim, seqlen, dstate, ngroups, has_D, has_z, has_bias, softplus
    (2, 32, 64 * 7 + 13, 16, None, True, True, True, True),   # partial last chunk, 8 chunks
    (1, 48, 640, 16, 2, True, False, False, True),             # aligned rows, two groups
    (2, 16, 64 * 5, 13, None, False, True, True, False),       # odd dstate, no softplus
    (1, 8, 64 * 3 + 1, 4, None, True, True, False, True),      # 4 chunks, the last one step long
    (1, 16, 64 * 130 + 7, 16, None, True, True, True, True),   # long pieces: summaries in run groups
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("pieces", [2, 3, 5])
def test_pieces_match_oracle_and_whole_rows(case, pieces):
    from helpers import assert_close, make_inputs, np64
    from oracle import f64

    b, d, l, n, g, has_D, has_z, has_bias, softplus = case
    inp = make_inputs(b, d, l, n, g, has_D, has_z, has_bias, torch.float32, a_scale=4.0)
    gen = torch.Generator().manual_seed(11)
    w_out = torch.randn(b, d, l, generator=gen)
    w_last = torch.randn(b, d, n, generator=gen)
    out, last, grads = _run(inp, softplus, w_out, w_last, pieces)
    out1, last1, grads1 = _run(inp, softplus, w_out, w_last, 1)
    o64, l64 = f64.scan_fwd(*[inp.get(k) for k in KEYS], delta_softplus=softplus)
    assert_close(out, o64, 1e-5, 1e-5, "out")
    assert_close(last, l64, 1e-5, 1e-5, "last_state")
    torch.testing.assert_close(out, out1, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(last, last1, rtol=1e-5, atol=1e-6)
    want = f64.scan_bwd(*[inp.get(k) for k in KEYS], softplus, w_out, w_last)
    for k, gk in GRAD_OF.items():
        if inp.get(k) is None:
            continue
        w = want[gk].reshape(inp[k].shape)
        scale = max(1.0, float(np.abs(w).max()))
        assert_close(np64(grads[k]) / scale, w / scale, 1e-4, 1e-4, name=k)
        sc = max(1.0, float(grads1[k].abs().max()))
        torch.testing.assert_close(grads[k] / sc, grads1[k] / sc, rtol=1e-5, atol=2e-6, msg=k)


@pytest.mark.gpu
@pytest.mark.parametrize("pieces", [2, 4])
def test_pieces_with_initial_state(pieces):
    """A given initial state enters piece 0 and reaches the later pieces through the summaries;
    its gradient comes from piece 0."""
    from helpers import assert_close, make_inputs
    from oracle import f64

    ops = torch.ops.mamba_b200
    x = make_inputs(2, 32, 64 * 6 + 30, 16, 1, True, True, True, torch.float32, seed=7)
    h0 = torch.randn(2, 32, 16, generator=torch.Generator().manual_seed(8))
    dout = torch.randn(2, 32, 64 * 6 + 30, generator=torch.Generator().manual_seed(9))
    args = [x[k].cuda() if x[k] is not None else None for k in KEYS]  # B / C as (b, g, n, l)
    h0c = h0.cuda().requires_grad_()
    with _Pieces(pieces):
        out, last, _ = ops.selective_scan_fwd_init(*args, True, h0c)
        (out * dout.cuda()).sum().backward()
    want_out, want_last = f64.scan_fwd(*[x[k] for k in KEYS], True, initial_state=h0)
    want = f64.scan_bwd(*[x[k] for k in KEYS], True, dout, initial_state=h0)
    assert_close(out, want_out, 1e-4, 1e-5, "out")
    assert_close(last, want_last, 1e-4, 1e-5, "last_state")
    assert_close(h0c.grad, want["dinitial_state"], 1e-4, 1e-5, "dinitial_state")


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pieces_strided_views_and_low_precision(dtype):
    """u / delta / z as strided views (the pieces' summary kernels read them through their batch
    and dim strides) and bf16 I/O; against whole rows on the same views."""
    from helpers import make_inputs

    b, d, l, n = 2, 40, 64 * 9 + 20, 16
    inp = make_inputs(b, d, l, n, None, True, True, True, dtype)
    wide = torch.zeros(b, d + 2, l, dtype=dtype)
    wide[:, 1:d + 1] = inp["u"]
    proj = inp["delta"].transpose(0, 1).contiguous()  # (d, b, l)
    views = {"u": wide.cuda()[:, 1:d + 1], "delta": proj.cuda().transpose(0, 1)}
    gen = torch.Generator().manual_seed(3)
    dout = torch.randn(b, d, l, generator=gen).to(dtype).cuda()
    res = []
    for pieces in (1, 3):
        leaves = {k: (v.cuda() if k not in views else views[k]).detach().requires_grad_(v is not None)
                  if v is not None else None for k, v in inp.items()}
        import mamba_cpu_b200 as mb

        with _Pieces(pieces):
            out = mb.selective_scan_fn(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"],
                                       leaves["D"], leaves["z"], leaves["delta_bias"], True)
            out.backward(dout)
        torch.cuda.synchronize()
        res.append([out.detach().float()] + [leaves[k].grad.float() for k in KEYS])
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    for name, a, c in zip(("out",) + KEYS, res[0], res[1]):
        sc = max(1.0, float(a.abs().max()))
        torch.testing.assert_close(c / sc, a / sc, rtol=tol, atol=tol, msg=name)


@pytest.mark.gpu
def test_automatic_pieces_on_a_rank_shard():
    """One rank's shard of config 5 at 8 ranks (640 channels, bf16): the automatic choice splits
    the rows; results agree with whole rows at bf16 rounding."""
    import mamba_cpu_b200 as mb
    from helpers import make_inputs, to_cuda

    b, d, l, n = 2, 640, 4096, 16
    ctas = b * (d // 16)
    assert _lib.lib.mb200_sequence_pieces(ctas, l // 64, 0) > 1 and _lib.lib.mb200_sequence_pieces(ctas, l // 64, 1) > 1
    inp = make_inputs(b, d, l, n, 1, True, True, False, torch.bfloat16, a_scale=15.5)
    dout = torch.randn(b, d, l, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).cuda()
    res = []
    for pieces in (0, 1):
        leaves = to_cuda(inp, requires_grad=True)
        with _Pieces(pieces):
            out = mb.selective_scan_fn(**leaves, delta_softplus=True)
            out.backward(dout)
        torch.cuda.synchronize()
        res.append([out.detach().float()] + [leaves[k].grad.float() for k in KEYS if leaves[k] is not None])
    for a, c in zip(res[0], res[1]):
        sc = max(1.0, float(c.abs().max()))
        torch.testing.assert_close(a / sc, c / sc, rtol=2e-2, atol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("seed", range(6))
def test_random_shapes_and_piece_counts(seed):
    """Random small problems (batch, dim, seqlen, dstate, groups, gate, bias, softplus, dtype) with
    a random forced piece count: split rows agree with whole rows (fp32 to 1e-5 relative of each
    tensor's largest value, bf16 to 2e-2)."""
    import random

    import mamba_cpu_b200 as mb
    from helpers import make_inputs, to_cuda

    rnd = random.Random(seed)
    b, d = rnd.choice([1, 2, 3]), rnd.choice([8, 24, 40])
    L = rnd.randint(65, 64 * 12 + 40)
    n = rnd.choice([4, 13, 16])
    g = rnd.choice([None, 1, 2]) if d % 2 == 0 else None
    has_z, has_bias, softplus = rnd.random() < 0.5, rnd.random() < 0.5, rnd.random() < 0.7
    dtype = rnd.choice([torch.float32, torch.bfloat16])
    pieces = rnd.randint(2, 8)
    inp = make_inputs(b, d, L, n, g, True, has_z, has_bias, dtype, seed=seed, a_scale=4.0)
    dout = torch.randn(b, d, L, generator=torch.Generator().manual_seed(seed)).to(dtype).cuda()
    res = []
    for pc in (1, pieces):
        leaves = to_cuda(inp, requires_grad=True)
        with _Pieces(pc):
            out, last = mb.selective_scan_fn(**leaves, delta_softplus=softplus, return_last_state=True)
            (out.float() * dout.float()).sum().add(last.sum()).backward()
        torch.cuda.synchronize()
        res.append([out.detach().float(), last.detach()] + [leaves[k].grad.float() for k in KEYS if leaves[k] is not None])
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    for a, c in zip(res[0], res[1]):
        sc = max(1.0, float(a.abs().max()))
        torch.testing.assert_close(c / sc, a / sc, rtol=tol, atol=tol)
