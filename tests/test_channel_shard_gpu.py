"""Channel-sharded selective scan on 2 (and 4) B200s against the same problem on one GPU.

Every rank runs the whole problem on its own GPU through ``selective_scan_fn`` + autograd, then
its channel shard inside ``parallel.channel_sharded`` (forward without communication, backward
with the one dB / dC exchange: the peer-memory sum, or NCCL's all_reduce). Per-channel results
(out, du, ddelta, dz, dA, dD, ddelta_bias) must equal the single-GPU run's slice bit for bit:
rows are independent and the kernels pick the same layout for both sizes here. dB / dC are sums
over channels taken in a different order (per-shard trees, then the exchange), so they are held
to a tolerance.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPE = dict(batch=2, dim=256, seqlen=300, dstate=16)  # 300: a partial last chunk


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(ngroups):
    b, d, l, n = SHAPE["batch"], SHAPE["dim"], SHAPE["seqlen"], SHAPE["dstate"]
    g = torch.Generator().manual_seed(1234 + ngroups)
    return {
        "u": torch.randn(b, d, l, generator=g),
        "delta": torch.randn(b, d, l, generator=g) * 0.5 - 1.0,
        "A": -torch.rand(d, n, generator=g) * 4.0 - 0.1,
        "B": torch.randn(b, ngroups, n, l, generator=g),
        "C": torch.randn(b, ngroups, n, l, generator=g),
        "D": torch.randn(d, generator=g),
        "z": torch.randn(b, d, l, generator=g),
        "delta_bias": torch.rand(d, generator=g) * 0.5,
        "dout": torch.randn(b, d, l, generator=g),
    }


def _run(x, dev):
    from mamba_cpu_b200 import selective_scan_fn

    leaves = {k: v.to(dev).requires_grad_(k != "dout") for k, v in x.items()}
    out = selective_scan_fn(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"], leaves["D"],
                            z=leaves["z"], delta_bias=leaves["delta_bias"], delta_softplus=True)
    out.backward(leaves["dout"])
    res = {"out": out.detach()}
    for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias"):
        res["d" + k] = leaves[k].grad
    return res


def _worker(rank, world, port, outdir, ngroups, peer):
    import torch.distributed as dist

    from mamba_cpu_b200 import _lib, parallel

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["LOCAL_WORLD_SIZE"] = str(world)
    os.environ["MAMBA_B200_PEER_REDUCE"] = "1" if peer else "0"
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        x = _inputs(ngroups)
        full = _run(x, dev)
        dim = SHAPE["dim"]
        lo, hi = parallel.shard_bounds(dim, ngroups, rank, world)
        glo, ghi = parallel.bc_groups(dim, ngroups, rank, world)
        group = parallel.new_reduce_group(dim, ngroups, rank, world)
        sh = {k: (v[:, lo:hi] if k in ("u", "delta", "z", "dout") else v[lo:hi] if k in ("A", "D", "delta_bias")
                  else v[:, glo:ghi]).contiguous() for k, v in x.items()}
        for _ in range(2):  # twice: both exchange slots of the peer path
            with parallel.channel_sharded(group):
                part = _run(sh, dev)
        res = {}
        for k in ("out", "du", "ddelta", "dz"):
            res[f"bitwise_{k}"] = bool(torch.equal(part[k], full[k][:, lo:hi]))
        for k in ("dA", "dD", "ddelta_bias"):
            res[f"bitwise_{k}"] = bool(torch.equal(part[k], full[k][lo:hi]))
        for k in ("dB", "dC"):
            want = full[k][:, glo:ghi]
            err = float((part[k] - want).abs().max())
            res[f"close_{k}"] = err <= 1e-5 * float(want.abs().max()) + 1e-6
        res["fault"] = _lib.device_fault()
        np.save(os.path.join(outdir, f"shard{rank}.npy"), res)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("world,ngroups,peer", [(2, 1, True), (2, 1, False), (2, 2, True), (4, 2, True),
                                                 (4, 1, True)])
def test_channel_sharded_equals_single_gpu(tmp_path, world, ngroups, peer):
    """(2, 1): both ranks share the one group (exchange over both). (2, 2): each rank holds a
    whole group (no exchange). (4, 2): ranks {0, 1} and {2, 3} share a group each."""
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), ngroups, peer), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        res = np.load(tmp_path / f"shard{r}.npy", allow_pickle=True).item()
        assert res.pop("fault") == 0, "a kernel recorded a device-side fault"
        bad = [k for k, v in res.items() if not v]
        assert not bad, f"rank {r}: sharded result differs from the single-GPU run in {bad}"
