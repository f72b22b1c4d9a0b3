"""Channel-sharded backward over 2- and 4-rank gloo process groups, on CPU.

The sharding contract (mamba_cpu_b200.parallel): every rank owns a contiguous, group-aligned
slice of the channels (rows of the scan are independent, mamba-cpu csrc/selective_scan.cpp:320-324)
and reads the replicated B / C groups of those channels. Per-channel gradients come out of each
rank's own backward; dB / dC are sums over all channels of a group, so the autograd backward
all-reduces the partial sums of the ranks sharing a group, once per call.

These tests run that host logic -- shard bounds, the reduce groups, the context that marks a
forward as sharded, the backward's all-reduce of [dB | dC] -- in spawned gloo ranks. The per-shard backward is
the float64 oracle standing in for the CUDA op (this machine has no GPU); the check is that the
sharded result equals the oracle's unsharded backward of the full problem.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mamba_cpu_b200 import parallel

WORLD = 2


def test_shard_bounds():
    assert parallel.shard_bounds(1536, 1, 0, 2) == (0, 768)
    assert parallel.shard_bounds(1536, 1, 1, 2) == (768, 1536)
    assert parallel.shard_bounds(64, 4, 3, 4) == (48, 64)  # one whole group per rank
    assert parallel.shard_bounds(64, 2, 1, 4) == (16, 32)  # half a group per rank
    with pytest.raises(ValueError):
        parallel.shard_bounds(10, 1, 0, 4)  # not divisible
    with pytest.raises(ValueError):
        parallel.shard_bounds(40, 5, 0, 4)  # 10 channels would split a group of 8
    with pytest.raises(ValueError):
        parallel.shard_bounds(36, 3, 0, 2)  # 18 channels would split a group of 12


def test_bc_groups_and_reduce_ranks():
    assert parallel.bc_groups(8, 1, 1, 2) == (0, 1)
    assert parallel.bc_groups(8, 2, 1, 2) == (1, 2)
    assert parallel.bc_groups(16, 8, 1, 2) == (4, 8)
    assert parallel.reduce_ranks(8, 1, 0, 4) == [0, 1, 2, 3]
    assert parallel.reduce_ranks(8, 2, 3, 4) == [2, 3]
    assert parallel.reduce_ranks(16, 8, 1, 2) == [1]


def test_channel_sharded_context_nests_and_resets():
    assert parallel.current_group() is None
    with parallel.channel_sharded("g1"):
        assert parallel.current_group() == "g1"
        with parallel.channel_sharded("g2"):
            assert parallel.current_group() == "g2"
        assert parallel.current_group() == "g1"
    assert parallel.current_group() is None


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(ngroups):
    g = torch.Generator().manual_seed(5)
    b, d, l, n = 2, 8, 37, 4
    return dict(
        u=torch.randn(b, d, l, generator=g),
        delta=torch.rand(b, d, l, generator=g) * 0.5,
        A=-torch.rand(d, n, generator=g) - 0.5,
        B=torch.randn(b, ngroups, n, l, generator=g),
        C=torch.randn(b, ngroups, n, l, generator=g),
        D=torch.randn(d, generator=g),
        z=torch.randn(b, d, l, generator=g),
        delta_bias=torch.rand(d, generator=g) * 0.1,
        dout=torch.randn(b, d, l, generator=g),
    )


class _Ctx:
    """Stand-in for the autograd context of mamba_b200::selective_scan_fwd."""

    def save_for_backward(self, *t):
        self.saved_tensors = t


def _oracle_bwd_op(u, delta, A, B, C, D, z, delta_bias, softplus, dout, dlast, chunk_states):
    """The shard's backward, computed by the float64 oracle (test stand-in for the CUDA op)."""
    from oracle import f64

    r = f64.scan_bwd(u, delta, A, B, C, D, z, delta_bias, softplus, dout, dlast)
    t = {k: torch.from_numpy(v).float() for k, v in r.items() if v is not None}
    return t["du"], t["ddelta"], t["dA"], t["dB"], t["dC"], t["dD"], t["dz"], t["ddelta_bias"]


def _worker(rank, world, port, ngroups, outdir):
    import torch.distributed as dist

    from mamba_cpu_b200.ops import selective_scan_interface as ssi

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        x = _inputs(ngroups)
        dim = x["u"].shape[1]
        lo, hi = parallel.shard_bounds(dim, ngroups, rank, world)
        glo, ghi = parallel.bc_groups(dim, ngroups, rank, world)
        group = parallel.new_reduce_group(dim, ngroups, rank, world)
        sh = {k: (v[:, lo:hi] if k in ("u", "delta", "z", "dout") else v[lo:hi] if k in ("A", "D", "delta_bias")
                  else v[:, glo:ghi]) for k, v in x.items()}
        # the forward marks its context as sharded; the backward all-reduces dB / dC
        ctx = _Ctx()
        inputs = (sh["u"], sh["delta"], sh["A"], sh["B"], sh["C"], sh["D"], sh["z"], sh["delta_bias"], True)
        with parallel.channel_sharded(group):
            ssi._setup_context(ctx, inputs, (None, None, None))
        assert ctx.shard_group is group
        ops = torch.ops.mamba_b200
        saved = getattr(ops, "selective_scan_bwd")
        setattr(ops, "selective_scan_bwd", _oracle_bwd_op)
        try:
            grads = ssi._backward(ctx, sh["dout"], None, None)
        finally:
            setattr(ops, "selective_scan_bwd", saved)
        names = ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias")
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), lo=lo, hi=hi, glo=glo, ghi=ghi,
                 **{k: g.numpy() for k, g in zip(names, grads)})
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world,ngroups", [(2, 1), (2, 2), (4, 2)])
def test_sharded_backward_equals_unsharded(tmp_path, world, ngroups):
    """(2, 1): both ranks read the one group (all-reduce over both). (2, 2): each rank holds a
    whole group (no collective). (4, 2): ranks {0, 1} and {2, 3} share a group each."""
    from oracle import f64

    port = _free_port()
    mp.start_processes(_worker, args=(world, port, ngroups, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    x = _inputs(ngroups)
    want = f64.scan_bwd(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"], x["delta_bias"], True,
                        x["dout"])
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    # every rank holds dB / dC of its groups summed over ALL channels of those groups
    for p in parts:
        glo, ghi = int(p["glo"]), int(p["ghi"])
        for k in ("dB", "dC"):
            np.testing.assert_allclose(p[k], want[k][:, glo:ghi], rtol=1e-5, atol=1e-5, err_msg=k)
    # per-channel gradients are the rank's own slice of the unsharded result
    for p in parts:
        lo, hi = int(p["lo"]), int(p["hi"])
        for k in ("du", "ddelta", "dz"):
            np.testing.assert_allclose(p[k], want[k][:, lo:hi], rtol=1e-5, atol=1e-6, err_msg=k)
        for k in ("dA", "dD", "ddelta_bias"):
            np.testing.assert_allclose(p[k], want[k][lo:hi], rtol=1e-5, atol=1e-6, err_msg=k)


def _reduce_worker(rank, port, outdir):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
    try:
        dB = torch.full((2, 1, 3, 5), float(rank + 1))
        dC = torch.arange(30, dtype=torch.float32).view(2, 1, 3, 5) * (rank + 1)
        rB, rC = parallel.all_reduce_bc(dB, dC, dist.group.WORLD)
        np.savez(os.path.join(outdir, f"r{rank}.npz"), dB=rB.numpy(), dC=rC.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_all_reduce_bc_is_one_sum_over_ranks(tmp_path):
    mp.start_processes(_reduce_worker, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True,
                       start_method="spawn")
    for r in range(WORLD):
        got = np.load(tmp_path / f"r{r}.npz")
        np.testing.assert_array_equal(got["dB"], np.full((2, 1, 3, 5), 3.0, np.float32))
        np.testing.assert_array_equal(got["dC"], np.arange(30, dtype=np.float32).reshape(2, 1, 3, 5) * 3)


# ---- sequence sharding (parallel.selective_scan_seq_sharded) -------------------------------


def _oracle_fwd_init(u, delta, A, B, C, D, z, delta_bias, softplus, initial_state):
    from oracle import f64

    out, last = f64.scan_fwd(u, delta, A, B, C, D, z, delta_bias, softplus, initial_state=initial_state)
    return torch.from_numpy(out).float(), torch.from_numpy(last).float(), torch.zeros(1)


def _oracle_bwd_init(u, delta, A, B, C, D, z, delta_bias, softplus, dout, dlast, chunk_states, initial_state):
    from oracle import f64

    r = f64.scan_bwd(u, delta, A, B, C, D, z, delta_bias, softplus, dout, dlast, initial_state=initial_state)
    t = {k: torch.from_numpy(v).float() for k, v in r.items() if v is not None}
    return (t["du"], t["ddelta"], t["dA"], t["dB"], t["dC"], t["dD"], t["dz"], t["ddelta_bias"],
            t["dinitial_state"])


def _seq_inputs(L):
    g = torch.Generator().manual_seed(9)
    b, d, n = 2, 6, 4
    return dict(
        u=torch.randn(b, d, L, generator=g),
        delta=torch.rand(b, d, L, generator=g) * 0.5,
        A=-torch.rand(d, n, generator=g) * 0.5 - 0.05,  # long memories: the pieces interact
        B=torch.randn(b, 1, n, L, generator=g),
        C=torch.randn(b, 1, n, L, generator=g),
        D=torch.randn(d, generator=g),
        z=torch.randn(b, d, L, generator=g),
        delta_bias=torch.rand(d, generator=g) * 0.1,
        dout=torch.randn(b, d, L, generator=g),
    )


def _seq_worker(rank, world, port, L, outdir):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        x = _seq_inputs(L)
        lo, hi = rank * L // world, (rank + 1) * L // world
        piece = {k: (v[..., lo:hi].contiguous() if k in ("u", "delta", "z", "B", "C", "dout") else v.clone())
                 for k, v in x.items()}
        leaves = {k: piece[k].requires_grad_() for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")}
        ops = torch.ops.mamba_b200
        saved = {n: getattr(ops, n) for n in ("selective_scan_fwd_init", "selective_scan_bwd_init")}
        setattr(ops, "selective_scan_fwd_init", _oracle_fwd_init)
        setattr(ops, "selective_scan_bwd_init", _oracle_bwd_init)
        try:
            out = parallel._SeqShardedScan.apply(
                leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"], leaves["D"], leaves["z"],
                leaves["delta_bias"], True, dist.group.WORLD)
            out.backward(piece["dout"])
        finally:
            for n, f in saved.items():
                setattr(ops, n, f)
        np.savez(os.path.join(outdir, f"seq{rank}.npz"), lo=lo, hi=hi, out=out.detach().numpy(),
                 **{"d" + k: v.grad.numpy() for k, v in leaves.items()})
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world,L", [(2, 150), (3, 200)])
def test_sequence_sharded_scan_equals_unsharded(tmp_path, world, L):
    """Rank r holds timesteps [r L / W, (r + 1) L / W); the composed result equals the oracle's
    scan of the whole sequence, outputs and all gradients."""
    from oracle import f64

    mp.start_processes(_seq_worker, args=(world, _free_port(), L, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    x = _seq_inputs(L)
    args = [x[k] for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")]
    out, _ = f64.scan_fwd(*args, True)
    want = f64.scan_bwd(*args, True, x["dout"])
    for r in range(world):
        p = np.load(tmp_path / f"seq{r}.npz")
        lo, hi = int(p["lo"]), int(p["hi"])
        np.testing.assert_allclose(p["out"], out[..., lo:hi], rtol=1e-5, atol=1e-5, err_msg="out")
        for k, key in (("du", "du"), ("ddelta", "ddelta"), ("dz", "dz"), ("dB", "dB"), ("dC", "dC")):
            np.testing.assert_allclose(p[k], want[key][..., lo:hi], rtol=1e-4, atol=1e-5, err_msg=k)
        for k, key in (("dA", "dA"), ("dD", "dD"), ("ddelta_bias", "ddelta_bias")):
            np.testing.assert_allclose(p[k], want[key], rtol=1e-4, atol=1e-5, err_msg=k)


class _FakePeerLib:
    """Stands in for libmamba_b200's peer entry points on CPU: hands out fake addresses, records
    what is released, and fails the call named in ``fail`` (on the rank it is given to). Other
    entry points (status strings) come from the real library."""

    def __init__(self, fail, real):
        self.fail = fail
        self.real = real
        self.live = set()
        self.next = 0x1000

    def __getattr__(self, name):
        return getattr(self.real, name)

    def _new(self, out):
        self.next += 0x1000
        out._obj.value = self.next
        self.live.add(self.next)
        return 0

    def mb200_peer_alloc(self, nbytes, out):
        return 7 if self.fail == "alloc" else self._new(out)

    def mb200_ipc_handle(self, ptr, handle):
        handle[0] = 1
        return 0

    def mb200_ipc_open(self, handle, out):
        return 7 if self.fail == "open" else self._new(out)

    def mb200_peer_free(self, ptr):
        self.live.discard(int(ptr))
        return 0

    def mb200_ipc_close(self, ptr):
        self.live.discard(int(ptr))
        return 0


def _peer_setup_worker(rank, port, fail_rank, fail, outdir):
    import torch.distributed as dist

    from mamba_cpu_b200 import _lib

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
    try:
        fake = _FakePeerLib(fail if rank == fail_rank else None, _lib.lib)
        _lib.lib = fake
        red = parallel.PeerReducer.create(1000, 24, dist.group.WORLD)
        np.save(os.path.join(outdir, f"p{rank}.npy"), {"none": red is None, "leaked": len(fake.live)})
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("fail", ["alloc", "open"])
def test_peer_exchange_setup_failure_falls_back_on_every_rank(tmp_path, fail):
    """One rank cannot allocate (or map) the exchange buffers: every rank gets None -- the NCCL
    path -- instead of hanging in the set-up's collectives, and nothing set up stays allocated or
    mapped."""
    mp.start_processes(_peer_setup_worker, args=(_free_port(), 1, fail, str(tmp_path)), nprocs=WORLD, join=True,
                       start_method="spawn")
    for r in range(WORLD):
        res = np.load(tmp_path / f"p{r}.npy", allow_pickle=True).item()
        assert res["none"], f"rank {r} built a reducer although rank 1 failed"
        assert res["leaked"] == 0, f"rank {r} kept {res['leaked']} buffers or mappings"
