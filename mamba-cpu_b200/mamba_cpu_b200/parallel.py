"""Channel (``dim`` / d_inner) sharding of the selective scan over a process group.

Every (batch, channel) row of the scan is an independent recurrence (mamba-cpu
csrc/selective_scan.cpp:320-324), so ranks can each own a contiguous slice of the channels with
u, delta, z, out, A, D, delta_bias (and their gradients) sharded along ``dim``. B and C are
replicated: a rank passes the B / C groups its channels read (:func:`bc_groups`; all of B / C when
ngroups = 1). The forward needs no communication. In the backward, dB and dC are sums over ALL
channels of a group, so the partial sums of the ranks that share a group are combined with one
all-reduce(SUM) of the fp32 [dB | dC] buffer per call, over :func:`new_reduce_group`'s process
group. A shard holds whole groups or a part of one group, never a part of two (checked by
:func:`shard_bounds`); a rank that holds whole groups needs no collective at all.

Usage (one process per GPU, ``torch.distributed`` initialised with the NCCL backend)::

    from mamba_cpu_b200 import selective_scan_fn, parallel
    lo, hi = parallel.shard_bounds(dim, ngroups, rank, world)
    glo, ghi = parallel.bc_groups(dim, ngroups, rank, world)      # B, C: (b, g, n, l)
    group = parallel.new_reduce_group(dim, ngroups, rank, world)  # collective: every rank calls it
    with parallel.channel_sharded(group):
        out = selective_scan_fn(u[:, lo:hi], delta[:, lo:hi], A[lo:hi], B[:, glo:ghi], C[:, glo:ghi],
                                D[lo:hi], ...)
        out.backward(...)         # dB / dC arrive summed over the ranks sharing the groups

The group is captured when the forward runs, so the backward may run outside the context.
"""

import contextlib
import contextvars
from typing import Optional

import torch

_group: contextvars.ContextVar = contextvars.ContextVar("mamba_b200_shard_group", default=None)


def current_group():
    """The process group channel sharding is active for, or None."""
    return _group.get()


@contextlib.contextmanager
def channel_sharded(group):
    """Make selective_scan_fn calls in this context treat their channels as one shard of
    ``group``: their backward all-reduces dB/dC across the group."""
    token = _group.set(group)
    try:
        yield group
    finally:
        _group.reset(token)


def shard_bounds(dim: int, ngroups: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous channel range [lo, hi) of ``rank``. Shards are group-aligned: a rank holds whole
    groups when ngroups >= world, or a contiguous part of one group otherwise."""
    if dim % world != 0:
        raise ValueError(f"dim ({dim}) must be divisible by the number of shards ({world})")
    per = dim // world
    dpg = dim // ngroups
    if not (per % dpg == 0 or dpg % per == 0):
        raise ValueError(f"a shard of {per} channels would split a group of {dpg} channels")
    return rank * per, (rank + 1) * per


def bc_groups(dim: int, ngroups: int, rank: int, world: int) -> tuple[int, int]:
    """Range [glo, ghi) of the B / C groups that ``rank``'s channels read."""
    lo, hi = shard_bounds(dim, ngroups, rank, world)
    dpg = dim // ngroups
    return lo // dpg, (hi - 1) // dpg + 1


def reduce_ranks(dim: int, ngroups: int, rank: int, world: int) -> list[int]:
    """The ranks whose channels read the same B / C groups as ``rank`` (``rank`` included): their
    partial dB / dC are summed. A single rank when shards hold whole groups."""
    mine = bc_groups(dim, ngroups, rank, world)
    return [r for r in range(world) if bc_groups(dim, ngroups, r, world) == mine]


def new_reduce_group(dim: int, ngroups: int, rank: int, world: int):
    """Process group over :func:`reduce_ranks` for ``rank`` (None when that is ``rank`` alone).

    Creates the process groups of ALL rank sets with ``torch.distributed.new_group``, which every
    rank of the default group must call in the same order, so every rank calls this function."""
    import torch.distributed as dist

    sets = []
    for r in range(world):
        s = reduce_ranks(dim, ngroups, r, world)
        if s not in sets:
            sets.append(s)
    if all(len(s) == world for s in sets):
        return dist.group.WORLD if world > 1 else None
    mine = None
    for s in sets:
        pg = dist.new_group(ranks=s) if len(s) > 1 else None
        if rank in s:
            mine = pg
    return mine


def all_reduce_bc(dB: torch.Tensor, dC: torch.Tensor, group, async_op: bool = False):
    """Sum the fp32 partial dB / dC over the shards of ``group`` with ONE collective."""
    import torch.distributed as dist

    flat = torch.cat([dB.reshape(-1), dC.reshape(-1)])
    work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
    if async_op:
        work.wait()
    n = dB.numel()
    return flat[:n].view_as(dB), flat[n:].view_as(dC)


def world_of(group) -> Optional[int]:
    import torch.distributed as dist

    return dist.get_world_size(group) if group is not None else None
