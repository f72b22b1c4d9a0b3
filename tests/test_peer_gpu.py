"""One-shot dB/dC sum over NVLink peer memory (parallel.PeerReducer, mb200_peer_sum_f32).

On one GPU, this process plays both ranks of a 2-rank exchange through local buffers: with the
other rank's signals already set the call returns the bitwise sum of the two slots and signals the
other rank; with no signal the bounded wait runs out (short timeout) and sets fault bit 1 while
the context stays usable.

Runs when the process sees at least 2 GPUs: 2 (and, with 4 GPUs visible, 4) NCCL ranks compare
the peer-memory sum with the rank-ordered fp32 sum of all ranks' inputs (all-gathered; the kernel
adds ranks in rank order, so the bits must agree) over several calls (both exchange slots; sizes that are not multiples of 4; a source
that is 16-byte aligned on one rank and not on the other), inside a captured CUDA graph, and
check the kernels' fault word (no wait timed out).
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_ordered_sum(dB, dC, group, world):
    import torch.distributed as dist

    flat = torch.cat([dB.reshape(-1), dC.reshape(-1)])
    parts = [torch.empty_like(flat) for _ in range(world)]
    dist.all_gather(parts, flat, group=group)
    want = parts[0].clone()
    for p in parts[1:]:
        want += p
    return want


def _fake_exchange(na, nb):
    """Exchange buffers, signal pads and call counters of a 2-rank exchange, both on this GPU."""
    from mamba_cpu_b200.parallel import PEER_BLOCKS

    nq = (na + nb + 3) // 4
    bufs = [torch.zeros(2 * 4 * nq, device="cuda") for _ in range(2)]
    pads = [torch.zeros(2 * PEER_BLOCKS, dtype=torch.int32, device="cuda") for _ in range(2)]
    counters = torch.zeros(PEER_BLOCKS + 1, dtype=torch.int32, device="cuda")  # + the timeout flag
    return bufs, pads, counters


def _peer_sum_as_rank0(a, b, bufs, pads, counters, timeout_us):
    from mamba_cpu_b200 import _lib

    dev_bufs = torch.tensor([t.data_ptr() for t in bufs], dtype=torch.int64, device="cuda")
    dev_pads = torch.tensor([t.data_ptr() for t in pads], dtype=torch.int64, device="cuda")
    st = _lib.lib.mb200_peer_sum_f32(a.data_ptr(), a.numel(), b.data_ptr(), b.numel(), dev_bufs.data_ptr(),
                                     dev_pads.data_ptr(), counters.data_ptr(), 0, 2, timeout_us, _lib.stream_of(a))
    _lib.check(st, "mb200_peer_sum_f32")
    torch.cuda.synchronize()


@pytest.mark.parametrize("na,nb", [(4096, 4096), (1003, 518)])
def test_peer_sum_one_gpu_two_fake_ranks(na, nb):
    from mamba_cpu_b200 import _lib
    from mamba_cpu_b200.parallel import PEER_BLOCKS

    g = torch.Generator().manual_seed(na + nb)
    a, b = torch.randn(na, generator=g).cuda(), torch.randn(nb, generator=g).cuda()
    other = torch.randn(na + nb, generator=g).cuda()
    bufs, pads, counters = _fake_exchange(na, nb)
    nq = (na + nb + 3) // 4
    bufs[1][4 * nq:4 * nq + na + nb] = other  # call 1 uses slot 1
    pads[0][PEER_BLOCKS:] = 1  # rank 1 has signalled call 1 to rank 0 from every CTA
    want = torch.cat([a, b]) + other
    _peer_sum_as_rank0(a, b, bufs, pads, counters, 10**6)
    assert _lib.device_fault() == 0
    assert torch.equal(torch.cat([a, b]), want)
    assert bool((pads[1][:PEER_BLOCKS] == 1).all()), "rank 0 did not signal rank 1 from every CTA"
    assert bool((counters[:PEER_BLOCKS] == 1).all())
    assert int(counters[PEER_BLOCKS]) == 0, "no wait timed out, the flag must stay clear"


def test_peer_wait_times_out_and_flags_fault():
    """Nothing sets the other rank's signal: the wait gives up after the timeout (0.1 s), records
    fault bit 1, poisons the result with NaN instead of summing a slot the other rank never
    filled, sets the sticky flag word, and the device stays usable."""
    import time

    from mamba_cpu_b200 import _lib
    from mamba_cpu_b200.parallel import PEER_BLOCKS

    a, b = torch.ones(256, device="cuda"), torch.ones(250, device="cuda")
    bufs, pads, counters = _fake_exchange(256, 250)
    t0 = time.perf_counter()
    _peer_sum_as_rank0(a, b, bufs, pads, counters, 100_000)
    elapsed = time.perf_counter() - t0
    assert _lib.device_fault() == 2
    assert 0.02 < elapsed < 20.0
    assert bool(torch.isnan(a).all()) and bool(torch.isnan(b).all()), "a timed-out call must not return sums"
    assert int(counters[PEER_BLOCKS]) == 1
    x = torch.arange(10, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 45.0  # the context is still usable


def test_peer_reducer_refuses_a_timed_out_result():
    """The host side of a timeout: PeerReducer reads the flag of its previous call and raises
    PeerExchangeTimeout (one GPU; the reducer is assembled around a fake 2-rank exchange whose
    other rank never signals)."""
    from mamba_cpu_b200 import _lib, parallel

    bufs, pads, counters = _fake_exchange(64, 64)
    r = parallel.PeerReducer.__new__(parallel.PeerReducer)
    r.na, r.nb, r.rank, r.world = 64, 64, 0, 2
    r.dev_bufs = torch.tensor([t.data_ptr() for t in bufs], dtype=torch.int64, device="cuda")
    r.dev_pads = torch.tensor([t.data_ptr() for t in pads], dtype=torch.int64, device="cuda")
    r.counters = counters
    r.timeout_us = 50_000
    r._flag_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    r._flag_event = None
    a, b = torch.ones(64, device="cuda"), torch.ones(64, device="cuda")
    r.all_reduce_(a, b)  # times out on the device; the host learns of it at the next check
    with pytest.raises(parallel.PeerExchangeTimeout):
        r.check()
    with pytest.raises(parallel.PeerExchangeTimeout):
        r.all_reduce_(a, b)  # the next call refuses to run on a poisoned exchange
    assert _lib.device_fault() == 2


def _worker(rank, world, port, outdir):
    import torch.distributed as dist

    from mamba_cpu_b200 import _lib, parallel

    torch.cuda.set_device(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["LOCAL_WORLD_SIZE"] = str(world)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        group = dist.group.WORLD
        results = {}
        for size in (1003, 64 * 1024 + 1):
            for it in range(5):  # alternates the two exchange slots
                g = torch.Generator().manual_seed(100 * it + rank + size)
                dB = torch.randn(2, 1, 4, size // 16, generator=g).cuda()
                dC = torch.randn(size - dB.numel(), generator=g).cuda()
                want = _rank_ordered_sum(dB, dC, group, world)
                got_b, got_c = parallel.all_reduce_bc(dB, dC, group)
                got = torch.cat([got_b.reshape(-1), got_c.reshape(-1)])
                results[f"eq_{size}_{it}"] = bool(torch.equal(got, want))
        # float4-sized pieces; odd ranks' dB starts 4 bytes into its storage, so the ranks access
        # their sources differently (vector / scalar) while exchanging the same slot layout
        for it in range(3):
            g = torch.Generator().manual_seed(31 + it + rank)
            dB = torch.randn(2 * 4 * 256 + 1, generator=g).cuda()[rank % 2:rank % 2 + 2 * 4 * 256].view(2, 1, 4, 256)
            dC = torch.randn(2, 1, 4, 256, generator=g).cuda()
            want = _rank_ordered_sum(dB, dC, group, world)
            got_b, got_c = parallel.all_reduce_bc(dB, dC, group)
            results[f"eq_vec_{it}"] = bool(torch.equal(torch.cat([got_b.reshape(-1), got_c.reshape(-1)]), want))
        # inside a CUDA graph: static input, replayed with new contents
        dB = torch.zeros(2, 1, 4, 1003 // 16, device="cuda")
        dC = torch.zeros(1003 - dB.numel(), device="cuda")
        parallel.all_reduce_bc(dB, dC, group)  # reducer exists before capture
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s), torch.cuda.graph(graph):
            out_b, out_c = parallel.all_reduce_bc(dB, dC, group)
        torch.cuda.current_stream().wait_stream(s)
        for it in range(3):
            g = torch.Generator().manual_seed(7 + it + 10 * rank)
            dB.copy_(torch.randn(dB.shape, generator=g))
            dC.copy_(torch.randn(dC.shape, generator=g))
            want = _rank_ordered_sum(dB, dC, group, world)
            graph.replay()
            torch.cuda.synchronize()
            results[f"graph_{it}"] = bool(torch.equal(torch.cat([out_b.reshape(-1), out_c.reshape(-1)]), want))
        del graph
        results["fault"] = _lib.device_fault()
        np.save(os.path.join(outdir, f"peer{rank}.npy"), results)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 4])
def test_peer_sum_is_the_rank_ordered_sum(tmp_path, world):
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        res = np.load(tmp_path / f"peer{r}.npy", allow_pickle=True).item()
        assert res.pop("fault") == 0, "a peer wait timed out"
        bad = [k for k, v in res.items() if not v]
        assert not bad, f"rank {r}: peer sum differs from the rank-ordered sum in {bad}"
