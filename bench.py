"""Benchmark: selective_scan fwd+bwd elements/s and % of HBM peak on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N

One step = one forward + backward selective scan over one batch of the configuration. The default
is BASELINE config 5 at its longest sequence (bf16 u/delta/B/C/z, fp32 A/D, batch 2, dim 5120,
seqlen 65536, dstate 16, z, softplus), strong-scaled: with N GPUs every rank owns 5120/N channels
of the same problem. The forward needs no communication; the backward sums the fp32 [dB | dC]
partial sums over the ranks in one exchange (a one-kernel sum read from the other GPUs' memory over
NVLink, parallel.PeerReducer, for exchanges up to 1 MiB; one NCCL all_reduce above that or with
MAMBA_B200_PEER_REDUCE=0 -- config 5's is 16.8 MB at seqlen 65536). At N > 1 rank 0
checks one step's exchanged dB / dC against the rank-ordered sum of the all-gathered partials
("exchange_check") and the exchange alone is timed ("exchange_us_per_step").

Inputs are resident in HBM when the timed region starts. Configurations whose inputs exceed L2
(126 MB) are not flushed; smaller ones get a 256 MiB write before the forward and before the
backward of every step. Kernel time is taken with CUDA events on the launching stream (max over
ranks); each phase is replayed from a CUDA graph, so host launch latency is not measured. A
"sustained" block repeats the step back to back for about 1.5 s under clock sampling.

`e2e` runs the public API (selective_scan_fn + autograd) with the step's inputs copied from pinned
host memory and every output and gradient copied back, all inside the timed region; consecutive
steps are pipelined (copies of neighbouring steps overlap the current step's kernels).

At N = 1 the line also carries a "c1" block (the reference README's forward-only
fp32 shape, with its roofline and the reference kernel's CPU time on the same problem), a "c2" block: BASELINE config 2 (fp32, batch 4, dim 1536, seqlen
1024, z, delta_bias), the north-star's fp32 configuration, with its own roofline and CPU baseline;
and "c3" / "c4" blocks: BASELINE configs 3 and 4 at model level (transformers' MambaForCausalLM,
random init, routed to this package by hf.patch_transformers): the 130M prefill in fp32 and the
1.4B-shape training step in bf16, in tokens/s, device-timed and end to end; and an "ssd" block: the
Mamba-2 SSD chunk scan forward (mamba_chunk_scan_combined) at the Mamba-2 2.7B layer shape, with its
roofline and the reference's CPU kernel on the equivalent Mamba-1 problem as its CPU baseline.

`--impl reference` times the reference's own CPU kernel (mamba-cpu csrc/selective_scan.cpp built
into oracle/_ref) with the reference's Python-side steps (B/C transpose to (b, g, l, n), zeroed
dB/dC, per-batch partial sums) on the host's cores, on a bounded channel slice of the workload.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mamba-cpu_b200"))
sys.path.insert(0, ROOT)

METRIC = "selective_scan fwd+bwd elements/s & % HBM peak at 1/2/4/8 B200"
L2_BYTES = 126 * 1024 * 1024

CONFIGS = {
    # name: (batch, global dim, seqlen, dstate, dtype, has_z, description); dim is split over ranks
    "c5": (2, 5120, 65536, 16, "bf16", True,
           "BASELINE config 5 (seqlen 65536): fwd+bwd bf16 u/delta/B/C/z, fp32 A/D, b=2 d=5120 n=16, softplus"),
    "c5_16k": (2, 5120, 16384, 16, "bf16", True,
               "BASELINE config 5 (seqlen 16384): fwd+bwd bf16 u/delta/B/C/z, fp32 A/D, b=2 d=5120 n=16, softplus"),
    "c5_4k": (2, 5120, 4096, 16, "bf16", True,
              "BASELINE config 5 (seqlen 4096): fwd+bwd bf16 u/delta/B/C/z, fp32 A/D, b=2 d=5120 n=16, softplus"),
    "c2": (4, 1536, 1024, 16, "f32", True,
           "BASELINE config 2: selective_scan_fn fwd+bwd fp32, b=4 d=1536 l=1024 n=16, z, delta_bias, softplus"),
    "c4_layer": (8, 4096, 2048, 16, "bf16", True,
                 "BASELINE config 4 scan of one layer: fwd+bwd bf16, b=8 d_inner=4096 l=2048 n=16"),
}


def algorithmic_bytes(b, d, l, n, s, s_bc, has_z, ngroups=1):
    """Bytes a fwd / bwd pass must move at minimum (u/delta/z/out/grads + B/C + small params)."""
    E = b * d * l
    Z = 1 if has_z else 0
    fwd = E * s * (3 + Z) + 2 * b * ngroups * n * l * s_bc + 4 * (d * n + 2 * d)
    bwd = E * s * (5 + 2 * Z) + 2 * b * ngroups * n * l * (s_bc + 4) + 4 * (d * n * 2 + 4 * d)
    return fwd, bwd


def load_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic(config):
    """Per-element DRAM traffic of the scan kernels from the committed ncu summaries, if any."""
    path = os.path.join(ROOT, "profiles", "roofline_traffic.txt")
    out = {}
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) == 3 and not line.startswith("#") and parts[0] == config:
                    out[parts[1]] = float(parts[2])
    except OSError:
        return {}
    return out


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during a timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index, interval_ms=50):
        self.index = index
        self.interval_ms = interval_ms
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", str(self.interval_ms)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.samples = []
        if self.proc is None:
            return
        time.sleep(0.2)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.samples.append(parts)

    def summary(self):
        if not getattr(self, "samples", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None

        rec = [(num(p[1]), num(p[2]), num(p[3])) for p in self.samples]
        sm = [r[0] for r in rec if r[0] is not None]
        mx = [r[1] for r in rec if r[1] is not None]
        pw = [r[2] for r in rec if r[2] is not None]
        # "under load": power well above the lowest sample (taken while the GPU worked)
        floor = min(pw) if pw else 0.0
        loaded = [r[0] for r in rec if r[0] is not None and r[2] is not None and r[2] > floor + 100.0]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for p in self.samples for i in range(4) if p[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(loaded or sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples), "samples_under_load": len(loaded),
                "interval_ms": self.interval_ms}


def make_inputs(cfg, lo, hi, device, torch, seed=1000):
    """Seeded synthetic inputs with the BASELINE distributions for channels [lo, hi) of the
    configuration (B / C are shared by all channels and identical on every rank)."""
    b, _, l, n, dt_name, has_z, _ = cfg
    dt = {"f32": torch.float32, "bf16": torch.bfloat16}[dt_name]
    d = hi - lo
    g = torch.Generator(device=device).manual_seed(seed + lo)  # this slice's channels
    gs = torch.Generator(device=device).manual_seed(7)          # B, C: the same on every rank

    def randn(*shape, gen=g):
        return torch.randn(*shape, generator=gen, device=device).to(dt)

    u, delta = randn(b, d, l), randn(b, d, l)
    z = randn(b, d, l) if has_z else None
    dout = randn(b, d, l)
    B, C = randn(b, 1, n, l, gen=gs), randn(b, 1, n, l, gen=gs)
    D = torch.randn(d, generator=g, device=device)
    if dt_name == "f32":
        bias = torch.rand(d, generator=g, device=device) * 3 - 4  # config 2: U(-4, -1)
        A = -torch.arange(1, n + 1, dtype=torch.float32, device=device).repeat(d, 1)  # -exp(log(1..16))
    else:
        bias = None  # config 5 has no delta_bias
        A = -(torch.rand(d, n, generator=g, device=device) * 15.5 + 0.5)  # -U(0.5, 16)
    return dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z, delta_bias=bias, dout=dout)


def shard(cfg, rank, world):
    """Channels [lo, hi) of this rank: the global dim split in equal contiguous shards."""
    per = cfg[1] // world
    if per * world != cfg[1]:
        raise SystemExit(f"dim {cfg[1]} is not divisible by {world} ranks")
    return rank * per, (rank + 1) * per


def device_timing(cfg, args, ctx, sustain_s=1.5):
    """Device-timed fwd + bwd steps of this rank's shard; returns a dict of per-step times (max over
    ranks), launch counts, the L2 policy and the clock records of the timed and sustained regions."""
    torch, dev, rank, world, group = ctx["torch"], ctx["dev"], ctx["rank"], ctx["world"], ctx["group"]
    dist = ctx["dist"]
    from mamba_cpu_b200 import _lib, parallel

    b, _, l, n, dt_name, has_z, _ = cfg
    lo, hi = shard(cfg, rank, world)
    x = make_inputs(cfg, lo, hi, dev, torch)
    s = 4 if dt_name == "f32" else 2
    big = b * (hi - lo) * l * s > L2_BYTES
    flush = None if big else torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    ops = torch.ops.mamba_b200
    launches = {}
    args_in = [x[k] for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")]

    def fwd():
        r = ops.selective_scan_fwd(*args_in, True)
        launches["fwd"] = _lib.last_launch_count()
        return r

    def bwd(chunk_states, exchange=True):
        r = ops.selective_scan_bwd(*args_in, True, x["dout"], None, chunk_states)
        launches["bwd"] = _lib.last_launch_count()
        if group is not None and exchange:
            parallel.all_reduce_bc(r[3], r[4], group)
            launches["bwd"] += 1
        return r

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for _ in range(3):
            o = fwd()
            bwd(o[2])
    torch.cuda.current_stream(dev).wait_stream(stream)
    torch.cuda.synchronize(dev)
    g_fwd, g_bwd = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_fwd):
        fo = fwd()
    with torch.cuda.graph(g_bwd):
        bo = bwd(fo[2])

    def step(events):
        if flush is not None:
            flush.zero_()
        events[0].record()
        g_fwd.replay()
        events[1].record()
        if flush is not None:
            flush.zero_()
        events[2].record()
        g_bwd.replay()
        events[3].record()

    for _ in range(args.warmup):
        step([torch.cuda.Event(enable_timing=True) for _ in range(4)])
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    if group is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with Clocks(ctx["local"]) as clk:
        for i in range(args.steps):
            step(evs[i])
        torch.cuda.synchronize(dev)
    if group is not None:
        dist.barrier()
    ms_fwd = sum(e[0].elapsed_time(e[1]) for e in evs) / len(evs)
    ms_bwd = sum(e[2].elapsed_time(e[3]) for e in evs) / len(evs)

    # sustained: the same steps back to back for about sustain_s, under clock sampling
    n_sus = max(args.steps, int(sustain_s / max((ms_fwd + ms_bwd) * 1e-3, 1e-6)))
    if group is not None:
        n_t = torch.tensor([n_sus], dtype=torch.int64, device=dev)
        dist.all_reduce(n_t, op=dist.ReduceOp.MAX)
        n_sus = int(n_t.item())
    # (per-phase events as in the timed region, so an L2 flush between phases is not counted)
    sev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n_sus)]
    if group is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with Clocks(ctx["local"]) as clk_sus:
        for i in range(n_sus):
            step(sev[i])
        torch.cuda.synchronize(dev)
    ms_sus = sum(e[0].elapsed_time(e[1]) + e[2].elapsed_time(e[3]) for e in sev) / n_sus
    del sev

    stat = torch.tensor([ms_fwd, ms_bwd, ms_sus], dtype=torch.float64, device=dev)
    if group is not None:
        dist.all_reduce(stat, op=dist.ReduceOp.MAX)
    ms_fwd, ms_bwd, ms_sus = stat.tolist()
    out = dict(ms_fwd=ms_fwd, ms_bwd=ms_bwd, ms_step=ms_fwd + ms_bwd, launches=launches["fwd"] + launches["bwd"],
               clocks=clk.summary(), sustained={"ms_per_step": ms_sus, "steps": n_sus,
                                                "clocks": clk_sus.summary()},
               l2=("inputs larger than L2 (126 MB): no flush between steps" if big else
                   "flushed (256 MiB write) before the forward and before the backward of every step"),
               x=x, lo=lo, hi=hi)

    if group is not None:
        # exchange check: one step's exchanged dB / dC against the rank-ordered sum of the partials
        r = bwd(fo[2], exchange=False)
        part = torch.cat([r[3].reshape(-1), r[4].reshape(-1)]).clone()
        sB, sC = parallel.all_reduce_bc(r[3], r[4], group)
        got = torch.cat([sB.reshape(-1), sC.reshape(-1)])
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part, group=group)
        want = parts[0].clone()
        for p_ in parts[1:]:
            want += p_
        # the peer-memory sum adds the ranks in rank order (bit-exact); NCCL's order is its own, so
        # its sums are held to float32 rounding of the largest magnitude
        exact = torch.equal(got, want)
        close = bool(((got - want).abs().max() <= 1e-6 * want.abs().max().clamp_min(1.0)).item())
        ok = torch.tensor([2 if exact else (1 if close else 0)], dtype=torch.int32, device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        out["exchange_check"] = {2: "ok (bit-exact rank-ordered sum)", 1: "ok (to float32 rounding)"}.get(
            int(ok.item()), "MISMATCH")
        # the exchange alone, event-timed (max over ranks)
        dB, dC = r[3], r[4]
        for _ in range(3):
            parallel.all_reduce_bc(dB, dC, group)
        dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        e0.record()
        for _ in range(reps):
            parallel.all_reduce_bc(dB, dC, group)
        e1.record()
        torch.cuda.synchronize(dev)
        us = torch.tensor([1e3 * e0.elapsed_time(e1) / reps], dtype=torch.float64, device=dev)
        dist.all_reduce(us, op=dist.ReduceOp.MAX)
        out["exchange_us_per_step"] = float(us.item())
        out["exchange_bytes"] = int(part.numel() * 4)
        del parts, want, part, got
    del g_fwd, g_bwd, fo, bo
    torch.cuda.synchronize(dev)
    return out


def e2e_timing(cfg, args, ctx, x):
    """The public API (selective_scan_fn + autograd backward) with every input copied from pinned
    host memory and every output and gradient copied back inside the timed region; steps pipelined
    as an input pipeline feeds a training loop. Returns the e2e block (max over ranks)."""
    torch, dev, group, dist = ctx["torch"], ctx["dev"], ctx["group"], ctx["dist"]
    import mamba_cpu_b200 as mb
    from mamba_cpu_b200 import parallel

    pinned = {k: (None if v is None else v.cpu().pin_memory()) for k, v in x.items()}
    names_in = ["u", "delta", "A", "B", "C", "D", "z", "delta_bias"]
    nbuf = 2
    comp = torch.cuda.current_stream(dev)
    h2d_stream, d2h_stream = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    dbufs = [{k: (None if v is None else torch.empty(v.shape, dtype=v.dtype, device=dev))
              for k, v in pinned.items()} for _ in range(nbuf)]
    in_ready = [torch.cuda.Event() for _ in range(nbuf)]
    in_free = [torch.cuda.Event() for _ in range(nbuf)]
    out_ready = torch.cuda.Event()
    for ev in in_free:
        ev.record(comp)
    outs_host = []  # one set: D2H of consecutive steps are ordered on d2h_stream

    def issue_h2d(i):
        bi = i % nbuf
        h2d_stream.wait_event(in_free[bi])
        with torch.cuda.stream(h2d_stream):
            for k, v in pinned.items():
                if v is not None:
                    dbufs[bi][k].copy_(v, non_blocking=True)
        in_ready[bi].record(h2d_stream)

    def compute(i):
        bi = i % nbuf
        comp.wait_event(in_ready[bi])
        dv = dbufs[bi]
        leaves = {k: (None if dv[k] is None else dv[k].detach().requires_grad_()) for k in names_in}
        with parallel.channel_sharded(group):
            out = mb.selective_scan_fn(**leaves, delta_softplus=True)
        out.backward(dv["dout"])
        res = [out.detach()] + [leaves[k].grad for k in names_in if leaves[k] is not None]
        in_free[bi].record(comp)
        out_ready.record(comp)
        return res

    def issue_d2h(res):
        if not outs_host:
            outs_host.extend(torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in res)
        d2h_stream.wait_event(out_ready)
        with torch.cuda.stream(d2h_stream):
            for hbuf, r in zip(outs_host, res):
                hbuf.copy_(r, non_blocking=True)
                r.record_stream(d2h_stream)

    def run_pipeline(nsteps):
        issue_h2d(0)
        for i in range(nsteps):
            if i + 1 < nsteps:
                issue_h2d(i + 1)
            issue_d2h(compute(i))
        comp.wait_stream(d2h_stream)

    h2d = sum(v.numel() * v.element_size() for v in pinned.values() if v is not None)
    run_pipeline(max(args.warmup, 3))
    torch.cuda.synchronize(dev)
    d2h = sum(v.numel() * v.element_size() for v in outs_host)
    steps = max(3, args.steps)  # the same K steps as the device-timed region
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if group is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0.record(comp)
    h2d_stream.wait_event(e0)
    run_pipeline(steps)
    e1.record(comp)
    torch.cuda.synchronize(dev)
    ms = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)

    # the copy floor of that step on this box right now: the same bytes both ways, no compute
    dev_in = dbufs[0]
    dev_out = [torch.empty_like(hb, device=dev) for hb in outs_host]

    def copies_only():
        with torch.cuda.stream(h2d_stream):
            for k, v in pinned.items():
                if v is not None:
                    dev_in[k].copy_(v, non_blocking=True)
        with torch.cuda.stream(d2h_stream):
            for hb, dvv in zip(outs_host, dev_out):
                hb.copy_(dvv, non_blocking=True)

    copies_only()
    torch.cuda.synchronize(dev)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(comp)
    h2d_stream.wait_event(c0)
    d2h_stream.wait_event(c0)
    for _ in range(steps):
        copies_only()
    comp.wait_stream(h2d_stream)
    comp.wait_stream(d2h_stream)
    c1.record(comp)
    torch.cuda.synchronize(dev)
    floor = torch.tensor([c0.elapsed_time(c1) / steps], dtype=torch.float64, device=dev)
    if group is not None:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(floor, op=dist.ReduceOp.MAX)
    del dbufs, dev_out, pinned, outs_host
    torch.cuda.synchronize(dev)
    return dict(ms=float(ms.item()), copy_floor_ms=float(floor.item()), h2d=h2d, d2h=d2h, steps=steps)


MODEL_CONFIGS = {
    # BASELINE configs 3 and 4 at model level: transformers' MambaForCausalLM, random init, with
    # hf.patch_transformers() routing its mixers to this package (the reference's hf route,
    # mamba-cpu src/mamba_cpu/hf.py; timed end to end by its benchmarks/check_hf_model.py:25-60).
    "c3": dict(desc="BASELINE config 3: random-init Mamba-1 130M (24 layers, d_model 768, d_inner 1536, n 16, "
                    "dt_rank 48, vocab 50280, tied embeddings, weights N(0, 0.02)) prefill fp32, batch 1, seqlen "
                    "1024, MambaForCausalLM through hf.patch_transformers",
               hidden=768, layers=24, dt_rank=48, batch=1, seqlen=1024, dtype="f32", train=False),
    "c4": dict(desc="BASELINE config 4 on one GPU: random-init Mamba-1 1.4B shape (48 layers, d_model 2048, d_inner "
                    "4096, n 16, dt_rank 128, vocab 50280) training step (forward, loss, backward; no optimizer "
                    "update, as the reference's check_hf_model train step) bf16, batch 8, seqlen 2048, "
                    "MambaForCausalLM through hf.patch_transformers",
               hidden=2048, layers=48, dt_rank=128, batch=8, seqlen=2048, dtype="bf16", train=True),
}


def model_timing(name, args, ctx, steps=5, warmup=3):
    """One BASELINE model-level configuration on this GPU: device time per step (token ids
    resident) and an end-to-end time per step through the public call with the ids copied from
    pinned host memory and the step's result (prefill: all logits; training: the loss) copied back."""
    torch, dev = ctx["torch"], ctx["dev"]
    from transformers import MambaConfig, MambaForCausalLM

    from mamba_cpu_b200 import hf

    m = MODEL_CONFIGS[name]
    dtype = torch.float32 if m["dtype"] == "f32" else torch.bfloat16
    vocab = 50280
    mcfg = MambaConfig(vocab_size=vocab, hidden_size=m["hidden"], state_size=16, num_hidden_layers=m["layers"],
                       expand=2, conv_kernel=4, time_step_rank=m["dt_rank"], use_mambapy=False,
                       tie_word_embeddings=True, initializer_range=0.02)
    torch.manual_seed(0)
    hf.patch_transformers()
    try:
        with torch.device(dev):
            model = MambaForCausalLM(mcfg).to(dtype)
        params = sum(p.numel() for p in model.parameters())
        b, l = m["batch"], m["seqlen"]
        g = torch.Generator().manual_seed(1)
        ids_host = torch.randint(0, vocab, (b, l), generator=g).pin_memory()
        ids = ids_host.to(dev)
        model.train(m["train"])

        def step(x):
            if m["train"]:
                model.zero_grad(set_to_none=True)
                loss = model(x, labels=x).loss
                loss.backward()
                return loss.detach()
            with torch.no_grad():
                return model(x).logits

        out_host = None

        def e2e_step():
            nonlocal out_host
            x = ids_host.to(dev, non_blocking=True)
            r = step(x)
            if out_host is None:
                out_host = torch.empty(r.shape, dtype=r.dtype, pin_memory=True)
            out_host.copy_(r, non_blocking=True)
            return r

        for _ in range(warmup):
            r = step(ids)
        torch.cuda.synchronize()
        finite = bool(torch.isfinite(r.float()).all())
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        for _ in range(steps):
            step(ids)
        ev[1].record()
        torch.cuda.synchronize()
        e2e_step()
        torch.cuda.synchronize()
        ev[2].record()
        for _ in range(steps):
            e2e_step()
        ev[3].record()
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1]) / steps
        ms_e2e = ev[2].elapsed_time(ev[3]) / steps
        d2h = out_host.numel() * out_host.element_size()
    finally:
        hf.unpatch_transformers()
    block = {
        "workload": m["desc"], "value": b * l / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
        "steps": steps, "warmup": warmup, "dtype": m["dtype"], "params": params,
        "data": "synthetic (random-init weights, uniform token ids)",
        "result_finite": finite,
        "e2e": {"value": b * l / (ms_e2e * 1e-3), "unit": "tokens/s", "ms_per_step": ms_e2e,
                "h2d_bytes_per_step": ids_host.numel() * ids_host.element_size(), "d2h_bytes_per_step": d2h},
    }
    del model
    torch.cuda.empty_cache()
    return block


def exchange_kind(nbytes):
    from mamba_cpu_b200 import parallel

    limit = int(os.environ.get("MAMBA_B200_PEER_REDUCE_MAX_BYTES", str(parallel.PEER_MAX_BYTES_DEFAULT)))
    if os.environ.get("MAMBA_B200_PEER_REDUCE", "1") != "0" and nbytes <= limit:
        return "peer-memory one-shot sum (NVLink)"
    return "NCCL all_reduce"


def roofline_block(name, kernel, nbytes, ms, peak, peak_kind, traffic_per_elem, elems):
    achieved = nbytes / (ms * 1e-3) / 1e9
    out = {"kernel": kernel, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
           "frac": achieved / peak, "algorithmic_bytes_per_launch": nbytes,
           "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback"}
    if traffic_per_elem is not None:
        out["traffic"] = traffic_per_elem * elems
        out["traffic_source"] = (f"profiles/roofline_traffic.txt: ncu dram__bytes_read.sum + dram__bytes_write.sum "
                                 f"per element of the {name} kernels (config 5 captured at seqlen 4096), scaled to "
                                 f"the elements of this launch")
    else:
        out["traffic"] = None
    return out


def _host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def sample_channels(cfg, target_elems=16 * 1024 * 1024):
    """Channels of the bounded CPU sample: about target_elems elements, a multiple of 16."""
    b, d, l = cfg[0], cfg[1], cfg[2]
    ch = max(16, target_elems // (b * l) // 16 * 16)
    return min(d, ch)


def reference_step_fn(cfg, channels, torch):
    """One fwd+bwd of the reference CPU path on `channels` channels of the configuration (the
    reference's own kernel via oracle/_ref, with its Python-side steps)."""
    import oracle
    from oracle import f64, ref_c

    b, _, l, n, dt_name, has_z, _ = cfg
    host = make_inputs(cfg, 0, channels, torch.device("cpu"), torch)
    f32 = {k: (None if v is None else v.float().contiguous()) for k, v in host.items()}
    d = channels
    if oracle.ref_available():
        kind = "reference"

        def step():
            # selective_scan_interface.py:127-135 (_as_f32 / _as_kernel_bc) and :16-97
            Bk = f32["B"].transpose(-1, -2).contiguous()
            Ck = f32["C"].transpose(-1, -2).contiguous()
            th = torch.get_num_threads()
            out = torch.empty(b, d, l)
            last = torch.empty(b, d, n)
            P = lambda t: 0 if t is None else t.data_ptr()  # noqa: E731
            ref_c.selective_scan_fwd_f32(P(f32["u"]), P(f32["delta"]), P(f32["A"]), P(Bk), P(Ck), P(f32["D"]),
                                         P(f32["z"]), P(f32["delta_bias"]), P(out), P(last), b, d, l, n, 1, True, th)
            du, ddelta = torch.empty(b, d, l), torch.empty(b, d, l)
            dA_part = torch.empty(b, d, n)
            dB, dC = torch.zeros_like(Bk), torch.zeros_like(Ck)
            dD_part, db_part = torch.empty(b, d), torch.empty(b, d)
            dz = torch.empty(b, d, l) if has_z else None
            ref_c.selective_scan_bwd_f32(P(f32["u"]), P(f32["delta"]), P(f32["A"]), P(Bk), P(Ck), P(f32["D"]),
                                         P(f32["z"]), P(f32["delta_bias"]), P(f32["dout"]), 0, P(du), P(ddelta),
                                         P(dA_part), P(dB), P(dC), P(dD_part), P(dz), P(db_part), b, d, l, n, 1,
                                         True, th)
            return dA_part.sum(0), dD_part.sum(0), db_part.sum(0)
    else:
        kind = "port"

        def step():
            args = [f32[k] for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")]
            f64.scan_fwd(*args, delta_softplus=True)
            f64.scan_bwd(*args, True, f32["dout"])
    return step, kind


def cpu_baseline(cfg, budget_s):
    import torch

    cores = _host_cores()
    torch.set_num_threads(cores)
    try:
        from oracle import f64

        f64.set_num_threads(cores)
    except Exception:
        pass
    ch = sample_channels(cfg)
    step, kind = reference_step_fn(cfg, ch, torch)
    b, l = cfg[0], cfg[2]
    t0 = time.perf_counter()
    step()  # warmup (bench_selective_scan.py:16-22 method)
    first = time.perf_counter() - t0
    iters = max(1, min(5, int(budget_s / max(first, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(iters):
        step()
    dt = (time.perf_counter() - t0) / iters
    return {"value": b * ch * l / dt, "unit": "elements/s", "cores": cores, "kind": kind,
            "sample": f"{iters} timed fwd+bwd passes (after 1 warm-up) of b={b} x {ch} of the config's {cfg[1]} "
                      f"channels x l={l}, {cores} threads, time.perf_counter",
            "ms_per_step": dt * 1e3}


def run_reference(args):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    cores = _host_cores()
    torch.set_num_threads(cores)
    ch = sample_channels(cfg)
    step, kind = reference_step_fn(cfg, ch, torch)
    b, l = cfg[0], cfg[2]
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    value = b * ch * l / (ms * 1e-3)
    line = {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "elements/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded; BASELINE config distributions)",
        "config": {"workload": cfg[6] + f" (each step: a {ch}-channel slice on the host CPU)",
                   "batch": b, "dim": cfg[1], "sample_channels": ch, "seqlen": l, "dstate": cfg[3]},
        "cpu_baseline": {"value": value, "unit": "elements/s", "cores": cores, "kind": kind,
                         "sample": f"{args.steps} fwd+bwd passes of b={b} x {ch} channels x l={l} after "
                                   f"{args.warmup} warm-up, {cores} threads"},
        "e2e": {"value": value, "unit": "elements/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


C1 = dict(batch=1, dim=1536, seqlen=2048, dstate=16,
          desc="BASELINE config 1: selective_scan_fn forward only, fp32, b=1 d=1536 l=2048 n=16, softplus, no z / "
               "delta_bias (the reference README's direct-use shape)")


def c1_inputs(torch, dev):
    b, d, l, n = (C1[k] for k in ("batch", "dim", "seqlen", "dstate"))
    g = torch.Generator(device=dev).manual_seed(11)
    r = lambda *s: torch.randn(*s, generator=g, device=dev)  # noqa: E731
    return dict(u=r(b, d, l), delta=r(b, d, l), A=-torch.rand(d, n, generator=g, device=dev), B=r(b, 1, n, l),
                C=r(b, 1, n, l), D=r(d))


def c1_timing(args, ctx, peak, peak_kind):
    """Device-timed forward of BASELINE config 1 (inputs under L2: a 256 MiB write before each step)."""
    torch, dev = ctx["torch"], ctx["dev"]
    from mamba_cpu_b200 import _lib

    b, d, l, n = (C1[k] for k in ("batch", "dim", "seqlen", "dstate"))
    x = c1_inputs(torch, dev)
    ops = torch.ops.mamba_b200
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def fwd():
        return ops.selective_scan_fwd(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], None, None, True)
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for _ in range(3):
            fwd()
    torch.cuda.current_stream(dev).wait_stream(stream)
    launches = _lib.last_launch_count()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fwd()
    steps = max(args.steps, 20)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for _ in range(max(3, args.warmup)):
        flush.zero_()
        graph.replay()
    torch.cuda.synchronize(dev)
    with Clocks(ctx["local"]) as clk:
        for e0, e1 in evs:
            flush.zero_()
            e0.record()
            graph.replay()
            e1.record()
        torch.cuda.synchronize(dev)
    ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / steps
    del graph
    E = b * d * l
    fwd_bytes, _ = algorithmic_bytes(b, d, l, n, 4, 4, False)
    return {"workload": C1["desc"], "value": E / (ms * 1e-3), "unit": "elements/s", "ms_per_step": ms,
            "steps": steps, "l2": "flushed (256 MiB write) before every step",
            "roofline_fwd": roofline_block("forward", "scan_fwd_kernel", fwd_bytes, ms, peak, peak_kind, None, E),
            "gpu_launches": launches * steps, "clocks": clk.summary()}


def c1_cpu_baseline(budget_s):
    """The reference's forward kernel (oracle/_ref) on the whole config-1 problem, all host threads."""
    import torch

    import oracle
    from oracle import f64, ref_c

    cores = _host_cores()
    torch.set_num_threads(cores)
    b, d, l, n = (C1[k] for k in ("batch", "dim", "seqlen", "dstate"))
    x = c1_inputs(torch, torch.device("cpu"))
    Bk = x["B"].transpose(-1, -2).contiguous()  # (b, g, l, n): selective_scan_interface.py:131-135
    Ck = x["C"].transpose(-1, -2).contiguous()
    out, last = torch.empty(b, d, l), torch.empty(b, d, n)
    P = lambda t: t.data_ptr()  # noqa: E731
    if oracle.ref_available():
        kind = "reference"

        def step():
            ref_c.selective_scan_fwd_f32(P(x["u"]), P(x["delta"]), P(x["A"]), P(Bk), P(Ck), P(x["D"]), 0, 0, P(out),
                                         P(last), b, d, l, n, 1, True, cores)
    else:
        kind = "port"
        f64.set_num_threads(cores)

        def step():
            f64.scan_fwd(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], delta_softplus=True)
    t0 = time.perf_counter()
    step()
    first = time.perf_counter() - t0
    iters = max(1, min(20, int(budget_s / max(first, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(iters):
        step()
    dt = (time.perf_counter() - t0) / iters
    return {"value": b * d * l / dt, "unit": "elements/s", "cores": cores, "kind": kind,
            "sample": f"{iters} timed forward passes (after 1 warm-up) of the whole config-1 problem, {cores} threads, "
                      f"time.perf_counter", "ms_per_step": dt * 1e3}


SSD = dict(batch=2, seqlen=4096, nheads=80, headdim=64, ngroups=1, dstate=128,
           desc="Mamba-2 SSD chunk scan forward (mamba_chunk_scan_combined, a roadmap item of the reference) at the "
                "Mamba-2 2.7B layer shape: b=2, seqlen 4096, 80 heads x headdim 64 (d_inner 5120), dstate 128, "
                "ngroups 1; bf16 x/z/B/C, fp32 dt/A/D/dt_bias, softplus, z gate")


def ssd_inputs(torch, dev, b, l, h, p, g, n, seed=2000):
    gen = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    return dict(x=torch.randn(b, l, h, p, generator=gen).to(bf).to(dev),
                dt=(torch.randn(b, l, h, generator=gen) * 0.1 - 4.0).to(dev),
                A=(-(1.0 + 15.0 * torch.rand(h, generator=gen))).to(dev),
                B=torch.randn(b, l, g, n, generator=gen).to(bf).to(dev),
                C=torch.randn(b, l, g, n, generator=gen).to(bf).to(dev),
                D=torch.randn(h, generator=gen).to(dev),
                z=torch.randn(b, l, h, p, generator=gen).to(bf).to(dev),
                dt_bias=(torch.rand(h, generator=gen) * 0.5).to(dev))


def ssd_bytes(b, l, h, p, g, n):
    """Algorithmic bytes of one forward: x, z read and out written (bf16), dt read (fp32), B and C read
    (bf16), per-head parameters."""
    return b * l * h * p * 2 * 3 + b * l * h * 4 + 2 * b * l * g * n * 2 + 4 * 3 * h


def ssd_cpu_baseline(budget_s):
    """The reference has no SSD scan; its CPU path for this computation is its Mamba-1 kernel on the
    equivalent problem (channels = heads x headdim, A repeated over dstate, dt repeated over headdim),
    timed on a bounded slice of heads with all host threads."""
    import torch

    import oracle
    from oracle import f64, ref_c

    cores = _host_cores()
    torch.set_num_threads(cores)
    b, l, h, p, g, n = (SSD[k] for k in ("batch", "seqlen", "nheads", "headdim", "ngroups", "dstate"))
    hs = 2  # heads in the sample
    x = ssd_inputs(torch, torch.device("cpu"), b, l, hs, p, g, n)
    f = {k: v.float() for k, v in x.items()}
    d = hs * p
    u = f["x"].permute(0, 2, 3, 1).reshape(b, d, l).contiguous()
    z = f["z"].permute(0, 2, 3, 1).reshape(b, d, l).contiguous()
    dl = f["dt"].permute(0, 2, 1)[:, :, None, :].expand(b, hs, p, l).reshape(b, d, l).contiguous()
    A = f["A"][:, None, None].expand(hs, p, n).reshape(d, n).contiguous()
    D = f["D"][:, None].expand(hs, p).reshape(d).contiguous()
    bias = f["dt_bias"][:, None].expand(hs, p).reshape(d).contiguous()
    Bk, Ck = f["B"].reshape(b, l, g, n).permute(0, 2, 1, 3).contiguous(), f["C"].reshape(b, l, g, n).permute(
        0, 2, 1, 3).contiguous()
    out, last = torch.empty(b, d, l), torch.empty(b, d, n)
    P = lambda t: t.data_ptr()  # noqa: E731
    if oracle.ref_available():
        kind = "reference"

        def step():
            ref_c.selective_scan_fwd_f32(P(u), P(dl), P(A), P(Bk), P(Ck), P(D), P(z), P(bias), P(out), P(last),
                                         b, d, l, n, g, True, cores)
    else:
        kind = "port"
        f64.set_num_threads(cores)

        def step():
            f64.ssd_fwd(x["x"], x["dt"], x["A"], x["B"], x["C"], x["D"], x["z"], x["dt_bias"], dt_softplus=True)
    t0 = time.perf_counter()
    step()
    first = time.perf_counter() - t0
    iters = max(1, min(5, int(budget_s / max(first, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(iters):
        step()
    dt = (time.perf_counter() - t0) / iters
    return {"value": b * l * d / dt, "unit": "elements/s", "cores": cores, "kind": kind,
            "sample": f"{iters} timed forward passes (after 1 warm-up) of {hs} of the {h} heads (b={b}, l={l}, "
                      f"headdim {p}, dstate {n}) through the reference's selective_scan_fwd_f32 on the equivalent "
                      f"Mamba-1 problem ({d} channels), {cores} threads, time.perf_counter",
            "ms_per_step": dt * 1e3}


def ssd_timing(args, ctx, peak, peak_kind):
    """Device-timed Mamba-2 SSD forward at the SSD shape (one GPU)."""
    torch, dev = ctx["torch"], ctx["dev"]
    from mamba_cpu_b200 import _lib
    import mamba_cpu_b200 as mb

    b, l, h, p, g, n = (SSD[k] for k in ("batch", "seqlen", "nheads", "headdim", "ngroups", "dstate"))
    x = ssd_inputs(torch, dev, b, l, h, p, g, n)

    def run():
        return mb.mamba_chunk_scan_combined(x["x"], x["dt"], x["A"], x["B"], x["C"], 256, D=x["D"], z=x["z"],
                                            dt_bias=x["dt_bias"], dt_softplus=True)
    for _ in range(max(3, args.warmup)):
        run()
    launches = _lib.last_launch_count()
    torch.cuda.synchronize(dev)
    steps = max(args.steps, 20)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    stream = torch.cuda.current_stream(dev)
    with Clocks(ctx["local"]) as clk:
        for e0, e1 in evs:
            e0.record(stream)
            run()
            e1.record(stream)
        torch.cuda.synchronize(dev)
    ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / steps
    E = b * l * h * p
    nbytes = ssd_bytes(b, l, h, p, g, n)
    return {
        "workload": SSD["desc"], "value": E / (ms * 1e-3), "unit": "elements/s",
        "element": "(batch, timestep, head channel): b * seqlen * nheads * headdim",
        "tokens_per_s": b * l / (ms * 1e-3), "ms_per_step": ms, "steps": steps,
        "l2": "inputs larger than L2 (x, z, out 84 MB each): no flush between steps",
        "roofline": dict(roofline_block("ssd", "ssd_fwd_kernel", nbytes, ms, peak, peak_kind,
                                        load_traffic("ssd").get("fwd_bytes_per_element"), E),
                         traffic_source="profiles/roofline_traffic.txt: ncu dram__bytes_read.sum + "
                                        "dram__bytes_write.sum of ssd_fwd_kernel at this shape "
                                        "(profiles/ssd_chunk_scan_fwd.md) per element, times the elements"),
        "gpu_launches": launches * steps, "clocks": clk.summary(),
    }


def run_ours(args):
    import datetime

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        group = dist.group.WORLD
    ctx = dict(torch=torch, dist=dist, dev=dev, rank=rank, world=world, local=local, group=group)

    cfg = CONFIGS[args.config]
    b, D, l, n, dt_name, has_z, desc = cfg
    dtm = device_timing(cfg, args, ctx)
    e2e = None if args.no_e2e else e2e_timing(cfg, args, ctx, dtm["x"])
    dtm.pop("x")
    c2 = None
    if world == 1 and args.config != "c2" and not args.no_c2:
        c2 = device_timing(CONFIGS["c2"], args, ctx)
        c2.pop("x")
    models = {}
    if world == 1 and not args.no_models:
        for name in ("c3", "c4"):
            models[name] = model_timing(name, args, ctx)
    peak, peak_kind = load_peak()
    ssd = c1 = None
    if world == 1 and not args.no_ssd:
        ssd = ssd_timing(args, ctx, peak, peak_kind)
    if world == 1 and not args.no_c2:
        c1 = c1_timing(args, ctx, peak, peak_kind)
    if group is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    s = 4 if dt_name == "f32" else 2
    per = D // world
    E_rank = b * per * l
    E = b * D * l
    fwd_bytes, bwd_bytes = algorithmic_bytes(b, per, l, n, s, s, has_z)
    traffic = load_traffic(args.config)
    ms_step = dtm["ms_step"]
    line = {
        "metric": METRIC,
        "value": E / (ms_step * 1e-3),
        "unit": "elements/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": dt_name,
        "data": "synthetic (seeded; BASELINE config distributions)",
        "config": {
            "workload": desc + (f"; dim sharded over {world} ranks ({per} channels each)" if world > 1 else ""),
            "batch": b, "dim": D, "dim_per_rank": per, "seqlen": l, "dstate": n,
            "l2": dtm["l2"],
            "parallelism": f"dim-shard{world}" if world > 1 else "single",
            **({"dB_dC_exchange": exchange_kind(dtm.get("exchange_bytes", 0))} if world > 1 else {}),
        },
        "tokens_per_s": b * l / (ms_step * 1e-3),
        "ms_fwd": dtm["ms_fwd"],
        "ms_bwd": dtm["ms_bwd"],
        "hbm_frac_step": (fwd_bytes + bwd_bytes) / (ms_step * 1e-3) / 1e9 / peak,
        "roofline": roofline_block("backward", "the backward op, per rank: scan_bwd_kernel + scan_bwd_reduce_kernel "
                                   "(+ scan_piece_summary_kernel and piece_combine_kernel when rows are split "
                                   "into sequence pieces)",
                                   bwd_bytes, dtm["ms_bwd"], peak, peak_kind, traffic.get("bwd_bytes_per_element"),
                                   E_rank),
        "roofline_fwd": roofline_block("forward", "scan_fwd_kernel (per rank)", fwd_bytes, dtm["ms_fwd"], peak,
                                       peak_kind, traffic.get("fwd_bytes_per_element"), E_rank),
        "gpu_launches": dtm["launches"] * args.steps,
        "clocks": dtm["clocks"],
        "sustained": dict(dtm["sustained"], value=E / (dtm["sustained"]["ms_per_step"] * 1e-3)),
    }
    for k in ("exchange_check", "exchange_us_per_step", "exchange_bytes"):
        if k in dtm:
            line[k] = dtm[k]
    if e2e is not None:
        line["e2e"] = {"value": E / (e2e["ms"] * 1e-3), "unit": "elements/s", "ms_per_step": e2e["ms"],
                       "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"], "steps": e2e["steps"],
                       "timing": "CUDA events around K pipelined steps, pipeline fill and drain included "
                                 "(per rank: its shard's copies; max over ranks)",
                       "copy_only_ms_per_step": e2e["copy_floor_ms"]}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, args.cpu_budget)
    if c2 is not None:
        cb, cD, cl_, cn = CONFIGS["c2"][:4]
        cf, cbw = algorithmic_bytes(cb, cD, cl_, cn, 4, 4, True)
        cE = cb * cD * cl_
        ctr = load_traffic("c2")
        line["c2"] = {
            "workload": CONFIGS["c2"][6], "value": cE / (c2["ms_step"] * 1e-3), "unit": "elements/s",
            "ms_per_step": c2["ms_step"], "ms_fwd": c2["ms_fwd"], "ms_bwd": c2["ms_bwd"], "l2": c2["l2"],
            "hbm_frac_step": (cf + cbw) / (c2["ms_step"] * 1e-3) / 1e9 / peak,
            "roofline": roofline_block("backward", "scan_bwd_kernel + scan_bwd_reduce_kernel (the backward op)", cbw,
                                       c2["ms_bwd"], peak, peak_kind, ctr.get("bwd_bytes_per_element"), cE),
            "roofline_fwd": roofline_block("forward", "scan_fwd_kernel", cf, c2["ms_fwd"], peak, peak_kind,
                                           ctr.get("fwd_bytes_per_element"), cE),
            "clocks": c2["clocks"], "sustained": c2["sustained"],
        }
        if not args.no_cpu_baseline:
            line["c2"]["cpu_baseline"] = cpu_baseline(CONFIGS["c2"], args.cpu_budget)
    line.update(models)
    if c1 is not None:
        if not args.no_cpu_baseline:
            c1["cpu_baseline"] = c1_cpu_baseline(args.cpu_budget)
        line["c1"] = c1
    if ssd is not None:
        if not args.no_cpu_baseline:
            ssd["cpu_baseline"] = ssd_cpu_baseline(args.cpu_budget)
        line["ssd"] = ssd
    print(json.dumps(line), flush=True)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", default="c5", choices=sorted(CONFIGS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true", help="device timing only (for profiler runs)")
    p.add_argument("--no-c2", action="store_true", help="skip the config-1 and config-2 blocks of the N=1 line")
    p.add_argument("--no-models", action="store_true",
                   help="skip the model-level config-3 / config-4 blocks of the N=1 line")
    p.add_argument("--no-ssd", action="store_true", help="skip the Mamba-2 SSD block of the N=1 line")
    p.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU baseline work")
    args = p.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
