"""Initial-state scans on the GPU: the kernels' path for a sequence scanned in pieces.

A sequence split at an arbitrary timestep and scanned as two pieces -- the second starting from
the first's end state (selective_scan_fwd_init), the first's backward receiving the adjoint the
second hands back (dinitial_state) -- must reproduce the scan of the whole sequence. The NCCL
test runs parallel.selective_scan_seq_sharded on 2 GPUs when the process sees at least 2.
"""

import os
import socket

import numpy as np
import pytest
import torch

from helpers import assert_close, make_inputs, np64, to_cuda

pytestmark = pytest.mark.gpu

ops = torch.ops.mamba_b200


def _prep(x):
    g = to_cuda(x)
    return (g["u"], g["delta"], g["A"], g["B"], g["C"], g["D"], g["z"], g["delta_bias"])


def _cut(t, lo, hi):
    return t[..., lo:hi].contiguous()


@pytest.mark.parametrize("dtype,ngroups,seqlen,cut", [(torch.float32, 1, 300, 137), (torch.float32, 2, 257, 64),
                                                      (torch.bfloat16, 1, 200, 100)])
def test_forward_in_two_pieces(dtype, ngroups, seqlen, cut):
    x = make_inputs(2, 64, seqlen, 16, ngroups, True, True, True, dtype, seed=4)
    u, dl, A, B, C, D, z, bias = _prep(x)
    out, last, _ = ops.selective_scan_fwd(u, dl, A, B, C, D, z, bias, True)
    o1, l1, _ = ops.selective_scan_fwd(_cut(u, 0, cut), _cut(dl, 0, cut), A, _cut(B, 0, cut), _cut(C, 0, cut), D,
                                       _cut(z, 0, cut), bias, True)
    o2, l2, _ = ops.selective_scan_fwd_init(_cut(u, cut, seqlen), _cut(dl, cut, seqlen), A, _cut(B, cut, seqlen),
                                            _cut(C, cut, seqlen), D, _cut(z, cut, seqlen), bias, True, l1)
    tol = 1e-4 if dtype == torch.float32 else 1e-2
    assert_close(torch.cat([o1, o2], -1).float(), out.float(), tol, tol, "out")
    assert_close(l2, last, 1e-4, 1e-5, "last_state")


@pytest.mark.parametrize("seqlen,cut", [(300, 137), (256, 128), (130, 64)])
def test_backward_in_two_pieces(seqlen, cut):
    x = make_inputs(2, 64, seqlen, 16, 1, True, True, True, torch.float32, seed=5)
    u, dl, A, B, C, D, z, bias = _prep(x)
    dout = torch.randn(u.shape, generator=torch.Generator().manual_seed(6)).cuda()
    _, _, cs = ops.selective_scan_fwd(u, dl, A, B, C, D, z, bias, True)
    full = ops.selective_scan_bwd(u, dl, A, B, C, D, z, bias, True, dout, None, cs)
    p1 = [_cut(t, 0, cut) for t in (u, dl)] + [A, _cut(B, 0, cut), _cut(C, 0, cut), D, _cut(z, 0, cut), bias]
    p2 = [_cut(t, cut, seqlen) for t in (u, dl)] + [A, _cut(B, cut, seqlen), _cut(C, cut, seqlen), D,
                                                     _cut(z, cut, seqlen), bias]
    _, l1, cs1 = ops.selective_scan_fwd(*p1, True)
    _, _, cs2 = ops.selective_scan_fwd_init(*p2, True, l1)
    g2 = ops.selective_scan_bwd_init(*p2, True, _cut(dout, cut, seqlen), None, cs2, l1)
    g1 = ops.selective_scan_bwd(*p1, True, _cut(dout, 0, cut), g2[8].contiguous(), cs1)
    names = ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias")
    for i, k in enumerate(names):
        if k in ("dA", "dD", "ddelta_bias"):
            got = g1[i] + g2[i]
        else:
            got = torch.cat([g1[i], g2[i]], -1)
        scale = max(1.0, float(full[i].abs().max()))
        assert_close(got / scale, full[i] / scale, 1e-4, 1e-5, k)
    # without chunk states (the backward recomputes them from the initial state)
    g2b = ops.selective_scan_bwd_init(*p2, True, _cut(dout, cut, seqlen), None, None, l1)
    for a, b in zip(g2, g2b):
        assert_close(a, b, 1e-5, 1e-6, "recomputed restart states")


def test_gradient_of_initial_state_matches_oracle():
    from oracle import f64

    x = make_inputs(2, 32, 150, 16, 1, True, True, True, torch.float32, seed=7)
    h0 = torch.randn(2, 32, 16, generator=torch.Generator().manual_seed(8))
    dout = torch.randn(2, 32, 150, generator=torch.Generator().manual_seed(9))
    u, dl, A, B, C, D, z, bias = _prep(x)
    h0c = h0.cuda().requires_grad_()
    out, _, _ = ops.selective_scan_fwd_init(u, dl, A, B, C, D, z, bias, True, h0c)
    (out * dout.cuda()).sum().backward()
    want_out, _ = f64.scan_fwd(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"], x["delta_bias"], True,
                               initial_state=h0)
    want = f64.scan_bwd(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"], x["delta_bias"], True, dout,
                        initial_state=h0)
    assert_close(out, want_out, 1e-4, 1e-5, "out")
    assert_close(h0c.grad, want["dinitial_state"], 1e-4, 1e-5, "dinitial_state")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist

    import mamba_cpu_b200 as mb
    from mamba_cpu_b200 import parallel

    torch.cuda.set_device(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        x = make_inputs(2, 64, 1000, 16, 1, True, True, True, torch.float32, seed=11)
        dout = torch.randn(2, 64, 1000, generator=torch.Generator().manual_seed(12))
        lo, hi = rank * 1000 // world, (rank + 1) * 1000 // world
        leaves = {k: (None if v is None else
                      (v[..., lo:hi] if k in ("u", "delta", "z", "B", "C") else v).contiguous().cuda().requires_grad_())
                  for k, v in x.items()}
        out = parallel.selective_scan_seq_sharded(**leaves, delta_softplus=True)
        out.backward(dout[..., lo:hi].contiguous().cuda())
        res = {"out": out.detach().cpu().numpy()}
        res.update({"d" + k: v.grad.cpu().numpy() for k, v in leaves.items()})
        if rank == 0:  # the whole sequence on one GPU
            full = {k: (None if v is None else v.cuda().requires_grad_()) for k, v in x.items()}
            fo = mb.selective_scan_fn(**full, delta_softplus=True)
            fo.backward(dout.cuda())
            res.update({"full_out": fo.detach().cpu().numpy()})
            res.update({"full_d" + k: v.grad.cpu().numpy() for k, v in full.items()})
        np.savez(os.path.join(outdir, f"r{rank}.npz"), lo=lo, hi=hi, **res)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_sharded_over_two_gpus(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_nccl_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    r0 = np.load(tmp_path / "r0.npz")
    for r in range(2):
        p = np.load(tmp_path / f"r{r}.npz")
        lo, hi = int(p["lo"]), int(p["hi"])
        assert_close(p["out"], r0["full_out"][..., lo:hi], 1e-4, 1e-5, "out")
        for k in ("du", "ddelta", "dz", "dB", "dC"):
            w = r0["full_" + k][..., lo:hi]
            scale = max(1.0, float(np.abs(w).max()))
            assert_close(p[k] / scale, w / scale, 1e-4, 1e-5, k)
        for k in ("dA", "dD", "ddelta_bias"):
            w = r0["full_" + k]
            scale = max(1.0, float(np.abs(w).max()))
            assert_close(p[k] / scale, w / scale, 1e-4, 1e-5, k)
