"""Channel (``dim`` / d_inner) sharding of the selective scan over a process group.

Every (batch, channel) row of the scan is an independent recurrence (mamba-cpu
csrc/selective_scan.cpp:320-324), so ranks can each own a contiguous slice of the channels with
u, delta, z, out, A, D, delta_bias (and their gradients) sharded along ``dim``. B and C are
replicated: a rank passes the B / C groups its channels read (:func:`bc_groups`; all of B / C when
ngroups = 1). The forward needs no communication. In the backward, dB and dC are sums over ALL
channels of a group, so the partial sums of the ranks that share a group are combined once per
call over :func:`new_reduce_group`'s process group (:func:`all_reduce_bc`: a one-kernel sum read
from the other GPUs' memory over NVLink when the group is node-local and NCCL-backed, else one
NCCL / gloo all_reduce). A shard holds whole groups or a part of one group, never a part of two (checked by
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
    ``group``: their backward sums dB/dC across the group (:func:`all_reduce_bc`)."""
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


PEER_BLOCKS = 148  # MB200_PEER_BLOCKS: CTAs of one mb200_peer_sum_f32 call


class PeerReducer:
    """One-shot sum of a pair of fp32 buffers (``na`` + ``nb`` elements) over the ranks of a
    node-local group, read directly from every rank's memory over NVLink
    (``mb200_peer_sum_f32``).

    Each rank allocates an exchange buffer (two slots of na + nb floats, rounded up to a multiple
    of 4) and a signal pad, exports them with CUDA IPC and maps the other ranks' (all ranks build
    the reducer together with :meth:`create`, a collective). A call is one kernel launch on the
    current stream and no host work, so it can be captured in a CUDA graph; every rank receives
    the same bits (ranks are added in rank order). The buffers and mappings live until the
    process exits.
    """

    def __init__(self, na: int, nb: int, group, bufs, pads, owned):
        import os

        import torch.distributed as dist

        self.na, self.nb = int(na), int(nb)
        self.group = group  # held: the reducer cache is keyed by id(group), which must stay unique
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self._owned = owned  # this rank's allocations and its mappings of the others'
        self.dev_bufs = torch.tensor(bufs, dtype=torch.int64, device="cuda")
        self.dev_pads = torch.tensor(pads, dtype=torch.int64, device="cuda")
        # PEER_BLOCKS call numbers, then the sticky timeout flag the kernel sets when a wait ran out
        self.counters = torch.zeros(PEER_BLOCKS + 1, dtype=torch.int32, device="cuda")
        # how long a rank's kernel waits for the others before flagging fault bit 1 (a straggler
        # that checkpoints between steps must stay under it)
        self.timeout_us = int(float(os.environ.get("MAMBA_B200_PEER_TIMEOUT_S", "30")) * 1e6)
        self._flag_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._flag_event = None

    @classmethod
    def create(cls, na: int, nb: int, group):
        """Build the reducer on every rank of ``group`` (a collective), or return None on every
        rank when any rank could not allocate, export or map the buffers (no CUDA IPC between
        the processes, for instance): the caller then uses NCCL. Every rank takes the same
        collective steps whatever fails locally. Not allowed while a CUDA graph is captured."""
        import ctypes

        import torch.distributed as dist

        from . import _lib

        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            raise RuntimeError("the dB/dC peer exchange is set up by the first sharded backward, which must run "
                               "before CUDA graph capture")
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        na, nb = int(na), int(nb)
        owned = []  # (kind, pointer): "alloc" -> mb200_peer_free, "map" -> mb200_ipc_close

        def release():
            for kind, ptr in reversed(owned):
                (_lib.lib.mb200_peer_free if kind == "alloc" else _lib.lib.mb200_ipc_close)(ptr)
            owned.clear()

        handles, err = None, ""
        try:  # local: allocate and export
            ptrs = []
            for nbytes in (2 * 16 * ((na + nb + 3) // 4), world * PEER_BLOCKS * 4):
                p = ctypes.c_void_p()
                _lib.check(_lib.lib.mb200_peer_alloc(nbytes, ctypes.byref(p)), "mb200_peer_alloc")
                owned.append(("alloc", p.value))
                ptrs.append(p.value)
            handles = []
            for ptr in ptrs:
                h = (ctypes.c_ubyte * 64)()
                _lib.check(_lib.lib.mb200_ipc_handle(ctypes.c_void_p(ptr), h), "mb200_ipc_handle")
                handles.append(bytes(h))
        except (RuntimeError, ValueError, OSError) as e:
            handles, err = None, str(e)
        everyone = [None] * world
        dist.all_gather_object(everyone, (handles, err), group=group)
        bufs, pads = [], []
        if all(h is not None for h, _ in everyone):
            try:  # local: map the other ranks' buffers
                for q, (hq, _) in enumerate(everyone):
                    if q == rank:
                        bufs.append(owned[0][1])
                        pads.append(owned[1][1])
                        continue
                    for h, dst in zip(hq, (bufs, pads)):
                        mapped = ctypes.c_void_p()
                        _lib.check(_lib.lib.mb200_ipc_open((ctypes.c_ubyte * 64).from_buffer_copy(h),
                                                           ctypes.byref(mapped)), "mb200_ipc_open")
                        owned.append(("map", mapped.value))
                        dst.append(mapped.value)
            except (RuntimeError, ValueError, OSError) as e:
                err = str(e)
        else:
            err = err or "another rank could not set up its exchange buffers"
        oks = [None] * world
        dist.all_gather_object(oks, err == "", group=group)
        if not all(oks):
            release()
            return None
        reducer = cls(na, nb, group, bufs, pads, owned)
        torch.cuda.synchronize()
        dist.barrier(group=group)  # every rank has mapped every buffer before anyone signals
        return reducer

    def check(self):
        """Raise :class:`PeerExchangeTimeout` if an earlier call's wait for another rank ran out
        (that call's sums were replaced by NaN). Waits for the flag copy of the latest call issued
        outside graph capture; calls replayed from a CUDA graph are not tracked."""
        if self._flag_event is None:
            return
        self._flag_event.synchronize()
        if int(self._flag_host[0]) != 0:
            raise PeerExchangeTimeout(
                "the dB/dC peer exchange timed out waiting for another rank "
                f"(MAMBA_B200_PEER_TIMEOUT_S = {self.timeout_us / 1e6:g} s); its sums were replaced by NaN")

    def all_reduce_(self, a: torch.Tensor, b: torch.Tensor):
        """Sum ``a`` and ``b`` (contiguous fp32 of the sizes given at construction) in place.

        Outside graph capture each call first checks the timeout flag left by the previous call
        (its copy to host memory completed long before, so this does not stall the stream) and
        raises :class:`PeerExchangeTimeout` if it is set; :meth:`check` checks the latest call."""
        from . import _lib

        for t, n in ((a, self.na), (b, self.nb)):
            assert t.dtype == torch.float32 and t.is_contiguous() and t.numel() == n
        capturing = torch.cuda.is_current_stream_capturing()
        if not capturing:
            self.check()
        st = _lib.lib.mb200_peer_sum_f32(a.data_ptr(), self.na, b.data_ptr(), self.nb, self.dev_bufs.data_ptr(),
                                         self.dev_pads.data_ptr(), self.counters.data_ptr(), self.rank, self.world,
                                         self.timeout_us, _lib.stream_of(a))
        _lib.check(st, "mb200_peer_sum_f32")
        if not capturing:
            self._flag_host.copy_(self.counters[PEER_BLOCKS:], non_blocking=True)
            if self._flag_event is None:
                self._flag_event = torch.cuda.Event()
            self._flag_event.record()
        return a, b


class PeerExchangeTimeout(RuntimeError):
    """A peer-memory dB/dC exchange gave up waiting for another rank; its result is NaN."""


_reducers: dict = {}


def _use_peer_sum(group, t: torch.Tensor) -> bool:
    """Peer-memory sums need CUDA tensors, an NCCL group of ranks on one node, and are on unless
    MAMBA_B200_PEER_REDUCE=0. Every rank evaluates the same conditions."""
    import os

    import torch.distributed as dist

    if not t.is_cuda or os.environ.get("MAMBA_B200_PEER_REDUCE", "1") == "0":
        return False
    if dist.get_backend(group) != "nccl":
        return False
    world = dist.get_world_size(group)
    return world > 1 and int(os.environ.get("LOCAL_WORLD_SIZE", str(world))) >= world


# Largest [dB | dC] exchange (bytes) the one-shot peer-memory sum takes; larger ones go to one
# NCCL all_reduce. Measured on 2 B200s: 13.7 / 15.1 us (peer / NCCL) at 0.5 MB, 108 / 65 us at
# 16.8 MB -- the one-shot sum reads every peer's whole buffer, NCCL's reduce-scatter + all-gather
# moves about twice the buffer whatever the rank count -- crossing near 1 MB.
PEER_MAX_BYTES_DEFAULT = 1 << 20


def all_reduce_bc(dB: torch.Tensor, dC: torch.Tensor, group, async_op: bool = False):
    """Sum the fp32 partial dB / dC over the shards of ``group`` in ONE exchange and return the
    sums. For node-local NCCL groups and exchanges up to MAMBA_B200_PEER_REDUCE_MAX_BYTES (1 MiB)
    this is a one-shot sum over NVLink peer memory (:class:`PeerReducer`) that overwrites dB and dC
    in place (ranks added in rank order); otherwise one ``all_reduce`` of their concatenation,
    whose sums are returned as views of the concatenated buffer."""
    import os

    import torch.distributed as dist

    nbytes = (dB.numel() + dC.numel()) * 4
    small = nbytes <= int(os.environ.get("MAMBA_B200_PEER_REDUCE_MAX_BYTES", str(PEER_MAX_BYTES_DEFAULT)))
    if (small and _use_peer_sum(group, dB) and dB.dtype == dC.dtype == torch.float32
            and dB.is_contiguous() and dC.is_contiguous()):
        key = (id(group), dB.numel(), dC.numel())
        if key not in _reducers:  # None: the peer exchange is unavailable for this group (NCCL)
            _reducers[key] = (group, PeerReducer.create(dB.numel(), dC.numel(), group))
        reducer = _reducers[key][1]
        if reducer is not None:
            return reducer.all_reduce_(dB, dC)
    flat = torch.cat([dB.reshape(-1), dC.reshape(-1)])
    work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
    if async_op:
        work.wait()
    n = dB.numel()
    return flat[:n].view_as(dB), flat[n:].view_as(dC)


def world_of(group) -> Optional[int]:
    import torch.distributed as dist

    return dist.get_world_size(group) if group is not None else None


# ---- sequence sharding ---------------------------------------------------------------------
# A sequence too long for one GPU is split along seqlen: rank r holds timesteps
# [r * L_r, (r + 1) * L_r) of u, delta, z, B, C (all ranks: every channel; A, D, delta_bias
# replicated). The recurrence h_t = a_t h_{t-1} + b_t is linear in its initial state, so a rank's
# piece maps an incoming state h to P h + e, with P = prod_t a_t = exp(A * sum_t dt) and e the
# piece's end state from h = 0. Forward: every rank scans its piece from zero, the ranks
# all-gather (P, e), rank r composes the pieces before it into its true initial state and scans
# again from it (rank 0's first pass is already exact). The backward mirrors this with the
# adjoint, which enters a piece from the right: a rank's piece maps an incoming adjoint g to
# P g + f, f being the adjoint at the piece start for g = 0. dB / dC belong to the rank's own
# timesteps; dA, dD and ddelta_bias are sums over time and are all-reduced. Cost: about two scans
# per rank and direction, one all-gather of 2 x (batch, dim, dstate) fp32 per direction.


def _piece_decay(delta, A, delta_bias, delta_softplus):
    dt = delta.float()
    if delta_bias is not None:
        dt = dt + delta_bias.float()[:, None]
    if delta_softplus:
        dt = torch.nn.functional.softplus(dt)
    return torch.exp(A.float()[None] * dt.sum(-1)[..., None])  # (batch, dim, dstate)


def _all_gather_pair(P, e, group):
    import torch.distributed as dist

    world = dist.get_world_size(group)
    stacked = torch.stack([P, e]).contiguous()
    out = [torch.empty_like(stacked) for _ in range(world)]
    dist.all_gather(out, stacked, group=group)
    return out


class _SeqShardedScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, delta, A, B, C, D, z, delta_bias, delta_softplus, group):
        import torch.distributed as dist

        ops = torch.ops.mamba_b200
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        b, d, _ = u.shape
        n = A.shape[-1]
        zero = torch.zeros(b, d, n, dtype=torch.float32, device=u.device)
        out, last, cs = ops.selective_scan_fwd_init(u, delta, A, B, C, D, z, delta_bias, delta_softplus, zero)
        P = _piece_decay(delta, A, delta_bias, delta_softplus)
        pieces = _all_gather_pair(P, last, group)
        h0 = zero
        for q in range(rank):
            h0 = pieces[q][0] * h0 + pieces[q][1]
        h0 = h0.contiguous()
        if rank > 0:
            out, last, cs = ops.selective_scan_fwd_init(u, delta, A, B, C, D, z, delta_bias, delta_softplus, h0)
        ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, cs, h0, P)
        ctx.delta_softplus = delta_softplus
        ctx.group = group
        return out

    @staticmethod
    def backward(ctx, dout):
        import torch.distributed as dist

        ops = torch.ops.mamba_b200
        u, delta, A, B, C, D, z, delta_bias, cs, h0, P = ctx.saved_tensors
        group = ctx.group
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        dout = dout.to(u.dtype).contiguous()
        args = (u, delta, A, B, C, D, z, delta_bias, ctx.delta_softplus, dout)
        grads = ops.selective_scan_bwd_init(*args, None, cs, h0)
        pieces = _all_gather_pair(P, grads[8], group)
        g = torch.zeros_like(h0)
        for q in range(world - 1, rank, -1):
            g = pieces[q][0] * g + pieces[q][1]
        if rank < world - 1:
            grads = ops.selective_scan_bwd_init(*args, g.contiguous(), cs, h0)
        du, ddelta, dA, dB, dC, dD, dz, ddelta_bias, _ = grads
        flat = torch.cat([dA.reshape(-1), dD, ddelta_bias])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        dA = flat[:dA.numel()].view_as(dA)
        dD = flat[dA.numel():dA.numel() + dD.numel()]
        ddelta_bias = flat[dA.numel() + dD.numel():]
        return (du, ddelta, dA, dB.to(B.dtype), dC.to(C.dtype),
                dD if D is not None else None, dz if z is not None else None,
                ddelta_bias if delta_bias is not None else None, None, None)


def selective_scan_seq_sharded(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                               group=None):
    """Selective scan of a sequence split along seqlen across the ranks of ``group``.

    Each rank passes its own timesteps of u, delta, z (batch, dim, L_r) and B, C
    ((batch, [ngroups,] dstate, L_r)), in rank order along the sequence, and the same A, D,
    delta_bias. Returns this rank's piece of ``out`` (as ``selective_scan_fn`` would return it for
    the whole sequence); gradients flow back through autograd (dA / dD / ddelta_bias summed over
    all ranks). Collectives: one all-gather per direction plus one all-reduce in the backward.
    """
    import torch.distributed as dist

    if group is None:
        group = dist.group.WORLD
    if u.device.type != "cuda":
        raise ValueError(f"mamba_cpu_b200 runs on CUDA tensors, got device {u.device}")
    if B.dim() == 3:
        B = B.unsqueeze(1)
    if C.dim() == 3:
        C = C.unsqueeze(1)
    io = u.dtype if u.dtype in (torch.float32, torch.bfloat16, torch.float16) else torch.float32
    Bk, Ck = B.to(io if B.dtype == io else torch.float32), C.to(io if C.dtype == io else torch.float32)
    if Bk.dtype != Ck.dtype:
        Bk, Ck = Bk.float(), Ck.float()
    Bk = Bk if Bk.stride(-1) == 1 else Bk.contiguous()
    Ck = Ck if Ck.stride(-1) == 1 else Ck.contiguous()
    out = _SeqShardedScan.apply(
        u.to(io).contiguous(), delta.to(io).contiguous(), A.float().contiguous(), Bk, Ck,
        None if D is None else D.float().contiguous(), None if z is None else z.to(io).contiguous(),
        None if delta_bias is None else delta_bias.float().contiguous(), bool(delta_softplus), group)
    return out.to(u.dtype)
