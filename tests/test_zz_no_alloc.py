"""The no-allocation backward entry point against the regular one, on the GPU.

mb200_selective_scan_bwd_noalloc exists for callers that cannot allocate device memory or hand
the library a workspace -- for example a host framework that owns all device memory and forbids
allocations inside its execute callbacks. Instead of a workspace it uses a static device array
inside the library. These tests call it through the C ABI on the same inputs as
mb200_selective_scan_bwd (given a workspace allocated here) and require bit-identical gradients
(both run the same deterministic kernels) on two calls in a row, the second running on the scratch
the first one left behind, and across problems of different sizes whose scratch layouts differ;
and they check that a request larger than the static scratch is refused before any work is
enqueued.

The file name makes pytest collect it after every other test module.
"""

import pytest
import torch

from mamba_cpu_b200 import _lib
from mamba_cpu_b200.ops.selective_scan_interface import _fwd_params, _nchunks

pytestmark = pytest.mark.gpu

GRADS = ("du", "ddelta", "dz", "dA", "dB", "dC", "dD", "ddelta_bias")


def _inputs(b, d, l, n, g, dtype):
    gen = torch.Generator().manual_seed(11)

    def rnd(*shape, dt=dtype):
        return torch.randn(*shape, generator=gen).to(dt).cuda()

    return dict(
        u=rnd(b, d, l), delta=rnd(b, d, l), A=(-torch.rand(d, n, generator=gen) * 4 - 0.5).cuda(),
        B=rnd(b, g, n, l), C=rnd(b, g, n, l), D=rnd(d, dt=torch.float32), z=rnd(b, d, l),
        delta_bias=(torch.rand(d, generator=gen) * 0.2).cuda(), dout=rnd(b, d, l),
        dlast=rnd(b, d, n, dt=torch.float32),
    )


def _bwd_params(x, chunk_states):
    p = _lib.ScanBwdParams()
    p.fwd = _fwd_params(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"], x["delta_bias"], True)
    p.fwd.chunk_states = _lib.ptr(chunk_states)
    out = dict(du=torch.empty_like(x["u"]), ddelta=torch.empty_like(x["u"]), dz=torch.empty_like(x["u"]),
               dA=torch.empty_like(x["A"]), dB=torch.empty(x["B"].shape, device="cuda"),
               dC=torch.empty(x["C"].shape, device="cuda"), dD=torch.empty_like(x["D"]),
               ddelta_bias=torch.empty_like(x["delta_bias"]))
    p.dout, p.dlast_state = _lib.ptr(x["dout"]), _lib.ptr(x["dlast"])
    for k in GRADS:
        setattr(p, k, _lib.ptr(out[k]))
    p.dbc_dtype = _lib.F32
    return p, out


def _chunk_states(x):
    b, d, l = x["u"].shape
    n = x["A"].shape[1]
    st = torch.empty(b, d, _nchunks(l), n, device="cuda")
    p = _fwd_params(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"], x["delta_bias"], True)
    out = torch.empty_like(x["u"])
    p.out, p.chunk_states = _lib.ptr(out), _lib.ptr(st)
    assert _lib.lib.mb200_selective_scan_fwd(p, _lib.stream_of(out)) == 0
    return st


SCRATCH_BYTES = 16 << 20  # MB200_NOALLOC_SCRATCH_BYTES


def _run_both(x, states, stream, call):
    """The workspace entry point and the no-allocation one on the same inputs; both run the same
    deterministic kernels, so every gradient must agree bit for bit."""
    p, want = _bwd_params(x, states)
    nbytes = _lib.lib.mb200_selective_scan_bwd_workspace_size(p)
    assert 0 < nbytes <= SCRATCH_BYTES, f"this case must fit the static scratch ({nbytes} bytes)"
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    assert _lib.lib.mb200_selective_scan_bwd(p, _lib.ptr(ws), nbytes, stream) == 0
    q, got = _bwd_params(x, states)
    for t in got.values():
        t.fill_(float("nan"))
    assert _lib.lib.mb200_selective_scan_bwd_noalloc(q, stream) == 0
    torch.cuda.synchronize()
    for k in GRADS:
        assert torch.equal(got[k], want[k]), f"call {call}: {k} differs from the workspace entry point"


@pytest.mark.parametrize("dtype,with_states", [(torch.float32, True), (torch.bfloat16, False)])
def test_noalloc_matches_workspace_entry_point_twice(dtype, with_states):
    x = _inputs(2, 96, 300, 16, 2, dtype)
    states = _chunk_states(x) if with_states else None
    stream = _lib.stream_of(x["u"])
    for call in range(2):  # the second call runs on whatever the first left in the static scratch
        _run_both(x, states, stream, call)


def test_noalloc_scratch_reuse_across_layouts():
    """A larger problem, a smaller one with another layout of the scratch, then the larger one
    again: each call must be correct whatever the previous call left in the shared array."""
    big = _inputs(2, 192, 1000, 16, 2, torch.float32)
    small = _inputs(1, 64, 130, 12, 1, torch.float32)
    stream = _lib.stream_of(big["u"])
    for call, x in enumerate((big, small, big)):
        _run_both(x, None, stream, call)


def test_noalloc_refuses_requests_beyond_its_scratch():
    p = _lib.ScanBwdParams()
    f = p.fwd
    f.u = f.delta = f.A = f.B = f.C = 0x1000
    f.batch, f.dim, f.seqlen, f.dstate, f.ngroups = 4, 1536, 65536, 16, 1
    f.B_batch_stride = f.C_batch_stride = 16 * 65536
    f.B_group_stride = f.C_group_stride = 16 * 65536
    f.B_dstate_stride = f.C_dstate_stride = 65536
    f.B_seqlen_stride = f.C_seqlen_stride = 1
    p.dout = p.du = p.ddelta = p.dA = p.dB = p.dC = 0x2000
    assert _lib.lib.mb200_selective_scan_bwd_workspace_size(p) > (16 << 20)
    # refused on the host before any device work (the pointers above are never dereferenced)
    assert _lib.lib.mb200_selective_scan_bwd_noalloc(p, None) == 8
    assert "static" in _lib.status_string(8)
