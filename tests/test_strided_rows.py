"""u / delta / z as strided views: the scan reads rows that are contiguous along seqlen in place,
whatever their batch and dim strides (mamba_b200.h: u_batch_stride ... z_dim_stride).

The Mamba-1 mixer produces such views for free -- delta as the transposed dt projection, z as one
half of the in_proj output -- and copying them costs two (batch, dim, seqlen) round trips per
layer. Results must not depend on the layout: every output and gradient of a run on views equals
the run on contiguous copies bit for bit (same arithmetic, only the addressing differs), on the
vectorised path (16-byte aligned rows), on the scalar path (unaligned rows) and with a partial
last chunk.
"""

import pytest
import torch

from mamba_cpu_b200.ops import selective_scan_interface as ssi


def _views(batch, dim, seqlen, dtype, device, pad=0):
    """u as a slice of a wider buffer, delta as a transposed projection, z as a chunk of xz:
    the layouts mamba_inner_fn hands to the scan. pad > 0 makes the rows unaligned."""
    g = torch.Generator().manual_seed(batch * 1000 + dim + seqlen + pad)
    wide = torch.randn(batch, dim + 3, seqlen + pad, generator=g).to(dtype).to(device)
    u = wide[:, 1:dim + 1, :seqlen]
    proj = (torch.randn(dim, batch * (seqlen + pad), generator=g) * 0.5 - 1.0).to(dtype).to(device)
    delta = proj.reshape(dim, batch, seqlen + pad).transpose(0, 1)[..., :seqlen]
    xz = torch.randn(batch, 2 * dim, seqlen + pad, generator=g).to(dtype).to(device)
    z = xz.chunk(2, dim=1)[1][..., :seqlen]
    return u, delta, z


def test_views_are_read_in_place_when_rows_are_aligned():
    u, delta, z = _views(2, 8, 64, torch.float32, "cpu")
    for t in (u, delta, z):
        assert not t.is_contiguous()
        assert ssi._as_rows(t, torch.float32).data_ptr() == t.data_ptr()  # no copy
    u, delta, z = _views(2, 8, 64, torch.float32, "cpu", pad=1)  # rows 4 bytes off 16
    assert ssi._as_rows(delta, torch.float32).is_contiguous()
    assert ssi._as_rows(u[..., ::2], torch.float32).is_contiguous()  # seqlen stride 2: copied


def test_op_accepts_seqlen_contiguous_views_only():
    u, delta, z = _views(2, 8, 64, torch.float32, "cpu")
    A = -torch.rand(8, 16)
    B = torch.randn(2, 1, 16, 64)
    ssi._check_op_inputs("t", u, delta, A, B, B, None, z, None)
    every_other = torch.randn(2, 8, 64)[..., ::2]  # seqlen stride 2
    with pytest.raises(ValueError, match="contiguous along seqlen"):
        ssi._check_op_inputs("t", torch.randn(2, 8, 32), every_other, A, B[..., :32], B[..., :32], None, None, None)


def _run(u, delta, z, A, B, C, D, bias, dout):
    # detach() keeps each tensor's layout (a view stays a view)
    leaves = [t.detach().requires_grad_() for t in (u, delta, A, B, C, D, z, bias)]
    lu, ld, lA, lB, lC, lD, lz, lb = leaves
    out = ssi.selective_scan_fn(lu, ld, lA, lB, lC, lD, z=lz, delta_bias=lb, delta_softplus=True)
    out.backward(dout)
    return [out.detach()] + [t.grad for t in leaves]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("seqlen,pad", [(256, 0), (300, 0), (256, 1)])
def test_strided_views_equal_contiguous_bitwise(dtype, seqlen, pad):
    from mamba_cpu_b200 import _lib

    batch, dim, n = 2, 96, 16
    u, delta, z = _views(batch, dim, seqlen, dtype, "cuda", pad)
    g = torch.Generator().manual_seed(5)
    A = (-torch.rand(dim, n, generator=g) * 4.0 - 0.1).cuda()
    B = torch.randn(batch, 1, n, seqlen, generator=g).to(dtype).cuda()
    C = torch.randn(batch, 1, n, seqlen, generator=g).to(dtype).cuda()
    D = torch.randn(dim, generator=g).cuda()
    bias = (torch.rand(dim, generator=g) * 0.5).cuda()
    dout = torch.randn(batch, dim, seqlen, generator=g).to(dtype).cuda()
    got = _run(u, delta, z, A, B, C, D, bias, dout)
    want = _run(u.contiguous(), delta.contiguous(), z.contiguous(), A, B, C, D, bias, dout)
    names = ("out", "du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias")
    assert not got[0].requires_grad
    for nm, a, b in zip(names, got, want):
        assert torch.equal(a, b), f"{nm} differs between strided views and contiguous copies"
    assert _lib.device_fault() == 0


@pytest.mark.gpu
def test_strided_views_through_the_op_keep_their_layout():
    """Called on the op directly (no _as_rows copy), unaligned views take the scalar path."""
    batch, dim, seqlen, n = 2, 32, 200, 16
    u, delta, z = _views(batch, dim, seqlen, torch.float32, "cuda", pad=3)
    assert delta.stride(1) * 4 % 16 != 0
    g = torch.Generator().manual_seed(9)
    A = (-torch.rand(dim, n, generator=g)).cuda()
    B = torch.randn(batch, 1, n, seqlen, generator=g).cuda()
    ops = torch.ops.mamba_b200
    got = ops.selective_scan_fwd(u, delta, A, B, B, None, z, None, True)
    want = ops.selective_scan_fwd(u.contiguous(), delta.contiguous(), A, B, B, None, z.contiguous(), None, True)
    for a, b in zip(got, want):
        assert a.is_contiguous() and torch.equal(a, b)


@pytest.mark.gpu
def test_negative_strides_are_a_layout_error():
    import ctypes

    from mamba_cpu_b200 import _lib

    batch, dim, seqlen, n = 1, 4, 64, 16
    u = torch.randn(batch, dim, seqlen, device="cuda")
    A = -torch.rand(dim, n, device="cuda")
    B = torch.randn(batch, 1, n, seqlen, device="cuda")
    out = torch.empty_like(u)
    p = ssi._fwd_params(u, u, A, B, B, None, None, None, True)
    p.out = _lib.ptr(out)
    p.delta_dim_stride = -seqlen
    st = _lib.lib.mb200_selective_scan_fwd(ctypes.byref(p), _lib.stream_of(u))
    assert st == 4  # MB200_ERR_BAD_LAYOUT


def _xproj_bc(batch, seqlen, n, r, dtype, device):
    """B / C as mamba_inner_fn slices them out of x_proj's output (b*l, r + 2n): (b, n, l) views
    with seqlen stride r + 2n and dstate stride 1."""
    g = torch.Generator().manual_seed(seqlen + r)
    x_dbl = torch.randn(batch * seqlen, r + 2 * n, generator=g).to(dtype).to(device)
    B = x_dbl[:, r:r + n].reshape(batch, seqlen, n).transpose(1, 2)
    C = x_dbl[:, r + n:].reshape(batch, seqlen, n).transpose(1, 2)
    return B, C


def test_xproj_bc_slices_kept_in_place_for_float32():
    """float32 B / C slices go to the kernels' strided path as they are; 2-byte ones are copied
    (their per-lane strided loads are slower than a copy)."""
    B, _ = _xproj_bc(2, 64, 16, 48, torch.float32, "cpu")
    Bk = ssi._as_kernel_bc(B, torch.float32)
    assert Bk.data_ptr() == B.data_ptr() and Bk.stride(-1) == 80 and Bk.shape == (2, 1, 16, 64)
    Bh, _ = _xproj_bc(2, 64, 16, 48, torch.bfloat16, "cpu")
    assert ssi._as_kernel_bc(Bh, torch.bfloat16).stride(-1) == 1
    u = torch.randn(2, 8, 64)
    ssi._check_op_inputs("t", u, u, -torch.rand(8, 16), Bk, Bk, None, None, None)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("seqlen", [256, 300])
def test_xproj_bc_slices_match_contiguous(dtype, seqlen):
    batch, dim, n = 2, 64, 16
    u, delta, z = _views(batch, dim, seqlen, dtype, "cuda")
    B, C = _xproj_bc(batch, seqlen, n, 48, dtype, "cuda")
    g = torch.Generator().manual_seed(9)
    A = (-torch.rand(dim, n, generator=g) * 4.0 - 0.1).cuda()
    D = torch.randn(dim, generator=g).cuda()
    bias = (torch.rand(dim, generator=g) * 0.5).cuda()
    dout = torch.randn(batch, dim, seqlen, generator=g).to(dtype).cuda()
    got = _run(u, delta, z, A, B, C, D, bias, dout)
    want = _run(u, delta, z, A, B.contiguous(), C.contiguous(), D, bias, dout)
    names = ("out", "du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias")
    for nm, a, b in zip(names, got, want):
        torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-6, msg=nm)
