"""Benchmark: selective_scan fwd+bwd elements/s and % of HBM peak on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N

One step = one forward + backward selective scan over one batch of the configuration (default
fp32, batch 4, dim 1536, seqlen 1024, dstate 16, z, delta_bias, softplus).
With N GPUs every rank owns a 1536-channel shard of a dim = 1536*N problem (weak scaling): the
forward needs no communication and the backward sums the fp32 [dB | dC] partial sums over the ranks
in one exchange: a one-kernel sum read from the other GPUs' memory over NVLink (parallel.PeerReducer;
MAMBA_B200_PEER_REDUCE=0 selects one NCCL all_reduce instead). Inputs are resident in HBM when the timed region starts; L2 (126 MB) is flushed with a
256 MiB write before the forward and before the backward of every step. Kernel time is taken with
CUDA events on the launching stream (max over ranks); the step's kernels are replayed from CUDA
graphs so host launch latency is not measured.

`e2e` runs the public API (selective_scan_fn + autograd) with the step's inputs copied from pinned
host memory and every output and gradient copied back, all inside the timed region; consecutive
steps are pipelined (copies of neighbouring steps overlap the current step's kernels).

`--impl reference` times the reference's own CPU kernel (mamba-cpu csrc/selective_scan.cpp built
into oracle/_ref) with the reference's Python-side steps (B/C transpose to (b, g, l, n), zeroed
dB/dC, per-batch partial sums) on the host's cores.
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

CONFIGS = {
    # name: (batch, dim per rank, seqlen, dstate, dtype, has_z, description)
    "c2": (4, 1536, 1024, 16, "f32", True,
           "BASELINE config 2: selective_scan_fn fwd+bwd fp32, b=4 d=1536 l=1024 n=16, z, delta_bias, softplus"),
    "c5_4k": (2, 5120, 4096, 16, "bf16", True,
              "BASELINE config 5 (L=4096): fwd+bwd bf16 u/delta/B/C/z, fp32 A/D, b=2 d=5120 n=16"),
    "c5_16k": (2, 5120, 16384, 16, "bf16", True,
               "BASELINE config 5 (L=16384): fwd+bwd bf16 u/delta/B/C/z, fp32 A/D, b=2 d=5120 n=16"),
    "c5_64k": (2, 5120, 65536, 16, "bf16", True,
               "BASELINE config 5 (L=65536): fwd+bwd bf16 u/delta/B/C/z, fp32 A/D, b=2 d=5120 n=16"),
    "c4_layer": (8, 4096, 2048, 16, "bf16", True,
                 "BASELINE config 4 scan of one layer: fwd+bwd bf16, b=8 d_inner=4096 l=2048 n=16"),
}


def algorithmic_bytes(b, d, l, n, s, s_bc, has_z, ngroups=1):
    """Bytes a fwd+bwd pass must move at minimum (u/delta/z/out/grads + B/C + small params)."""
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
    """Per-element DRAM traffic of the dominant kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "roofline_traffic.txt")
    out = {}
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) == 3 and not line.startswith("#") and parts[0] == config:
                    out[parts[1]] = float(parts[2])
    except OSError:
        return None
    return out or None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
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
        sm = [float(p[1]) for p in self.samples if p[1].replace(".", "").isdigit()]
        mx = [float(p[2]) for p in self.samples if p[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for p in self.samples for i in range(4) if p[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def make_inputs(cfg, device, rank, torch):
    b, d, l, n, dt_name, has_z, _ = cfg
    dt = {"f32": torch.float32, "bf16": torch.bfloat16}[dt_name]
    g = torch.Generator().manual_seed(1000 + rank)  # per-shard channels
    gs = torch.Generator().manual_seed(7)  # B, C are replicated across shards
    u = torch.randn(b, d, l, generator=g).to(dt)
    delta = torch.randn(b, d, l, generator=g).to(dt)
    z = torch.randn(b, d, l, generator=g).to(dt) if has_z else None
    dout = torch.randn(b, d, l, generator=g).to(dt)
    B = torch.randn(b, 1, n, l, generator=gs).to(dt)
    C = torch.randn(b, 1, n, l, generator=gs).to(dt)
    D = torch.randn(d, generator=g)
    bias = torch.rand(d, generator=g) * 3 - 4
    if dt_name == "f32":
        A = -torch.arange(1, n + 1, dtype=torch.float32).repeat(d, 1)  # config 2: -exp(log(1..16))
    else:
        A = -(torch.rand(d, n, generator=g) * 15.5 + 0.5)  # config 5: -U(0.5, 16)
    host = dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z, delta_bias=bias, dout=dout)
    return host


def run_ours(args):
    import torch
    import torch.distributed as dist

    import mamba_cpu_b200 as mb
    from mamba_cpu_b200 import _lib
    from mamba_cpu_b200 import parallel

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        group = dist.group.WORLD

    cfg = CONFIGS[args.config]
    b, d, l, n, dt_name, has_z, desc = cfg
    host = make_inputs(cfg, dev, rank, torch)
    x = {k: (None if v is None else v.to(dev)) for k, v in host.items()}
    s = 4 if dt_name == "f32" else 2
    fwd_bytes, bwd_bytes = algorithmic_bytes(b, d, l, n, s, s, has_z)
    E = b * d * l
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    ops = torch.ops.mamba_b200
    launches = {}

    def fwd():
        r = ops.selective_scan_fwd(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"], x["delta_bias"], True)
        launches["fwd"] = _lib.last_launch_count()
        return r

    def bwd(chunk_states):
        r = ops.selective_scan_bwd(x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"], x["delta_bias"],
                                   True, x["dout"], None, chunk_states)
        launches["bwd"] = _lib.last_launch_count()
        if group is not None:
            parallel.all_reduce_bc(r[3], r[4], group)
        return r

    # warm up, then capture one graph per phase
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
    per_step_launches = launches["fwd"] + launches["bwd"]

    def step(events):
        flush.zero_()
        events[0].record()
        g_fwd.replay()
        events[1].record()
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
    with Clocks(local) as clk:
        for i in range(args.steps):
            step(evs[i])
        torch.cuda.synchronize(dev)
    if group is not None:
        dist.barrier()
    t_fwd = [e[0].elapsed_time(e[1]) for e in evs]
    t_bwd = [e[2].elapsed_time(e[3]) for e in evs]
    ms_fwd = sum(t_fwd) / len(t_fwd)
    ms_bwd = sum(t_bwd) / len(t_bwd)
    ms_step = ms_fwd + ms_bwd
    stat = torch.tensor([ms_step, ms_fwd, ms_bwd], dtype=torch.float64, device=dev)
    if group is not None:
        dist.all_reduce(stat, op=dist.ReduceOp.MAX)
    ms_step, ms_fwd, ms_bwd = stat.tolist()

    # ---- e2e through the public API: pinned H2D, fwd + autograd bwd, D2H of everything ----
    if args.no_e2e:
        del g_fwd, g_bwd
        if group is not None:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"ms_fwd": ms_fwd, "ms_bwd": ms_bwd, "ms_per_step": ms_step,
                              "value": E * world / (ms_step * 1e-3), "note": "--no-e2e run (profiling)"}))
        return
    # Steps are pipelined the way an input pipeline feeds a training loop: step i + 1's inputs
    # are copied host -> device on one stream and step i - 1's results device -> host on another
    # while step i runs on the compute stream, with two device input buffers. Every step still
    # moves all of its inputs and results across PCIe inside the timed region.
    pinned = {k: (None if v is None else v.pin_memory()) for k, v in host.items()}
    names_in = ["u", "delta", "A", "B", "C", "D", "z", "delta_bias"]
    nbuf = 2
    comp = torch.cuda.current_stream(dev)
    h2d_stream, d2h_stream = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    dbufs = [{k: (None if v is None else torch.empty(v.shape, dtype=v.dtype, device=dev))
              for k, v in pinned.items()} for _ in range(nbuf)]
    in_ready = [torch.cuda.Event() for _ in range(nbuf)]
    in_free = [torch.cuda.Event() for _ in range(nbuf)]
    out_ready = [torch.cuda.Event() for _ in range(nbuf)]
    for ev in in_free:
        ev.record(comp)
    outs_host = [[] for _ in range(nbuf)]

    def issue_h2d(i):
        b = i % nbuf
        h2d_stream.wait_event(in_free[b])
        with torch.cuda.stream(h2d_stream):
            for k, v in pinned.items():
                if v is not None:
                    dbufs[b][k].copy_(v, non_blocking=True)
        in_ready[b].record(h2d_stream)

    def compute(i):
        b = i % nbuf
        comp.wait_event(in_ready[b])
        dv = dbufs[b]
        leaves = {k: (None if dv[k] is None else dv[k].detach().requires_grad_()) for k in names_in}
        with parallel.channel_sharded(group):
            out = mb.selective_scan_fn(**leaves, delta_softplus=True)
        out.backward(dv["dout"])
        res = [out.detach()] + [leaves[k].grad for k in names_in if leaves[k] is not None]
        in_free[b].record(comp)
        out_ready[b].record(comp)
        return res

    def issue_d2h(i, res):
        b = i % nbuf
        if not outs_host[b]:
            outs_host[b] = [torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in res]
        d2h_stream.wait_event(out_ready[b])
        with torch.cuda.stream(d2h_stream):
            for hbuf, r in zip(outs_host[b], res):
                hbuf.copy_(r, non_blocking=True)
                r.record_stream(d2h_stream)

    def run_pipeline(n):
        issue_h2d(0)
        for i in range(n):
            if i + 1 < n:
                issue_h2d(i + 1)
            issue_d2h(i, compute(i))
        comp.wait_stream(d2h_stream)

    h2d = sum(v.numel() * v.element_size() for v in pinned.values() if v is not None)
    run_pipeline(max(args.warmup, 3))
    torch.cuda.synchronize(dev)
    d2h = sum(v.numel() * v.element_size() for v in outs_host[0])
    e2e_steps = max(3, args.steps)  # the same K steps as the device-timed region
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if group is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0.record(comp)
    h2d_stream.wait_event(e0)
    run_pipeline(e2e_steps)
    e1.record(comp)
    torch.cuda.synchronize(dev)
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / e2e_steps], dtype=torch.float64, device=dev)
    if group is not None:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())

    # The copy floor of that e2e step on this box right now: the same step's input bytes host ->
    # device and result bytes device -> host, both directions at once, without the compute.
    dev_in = dbufs[0]
    dev_out = [torch.empty_like(hb, device=dev) for hb in outs_host[0]]
    def copies_only():
        with torch.cuda.stream(h2d_stream):
            for k, v in pinned.items():
                if v is not None:
                    dev_in[k].copy_(v, non_blocking=True)
        with torch.cuda.stream(d2h_stream):
            for hb, dv in zip(outs_host[0], dev_out):
                hb.copy_(dv, non_blocking=True)
    for _ in range(2):
        copies_only()
    torch.cuda.synchronize(dev)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(comp)
    h2d_stream.wait_event(c0)
    d2h_stream.wait_event(c0)
    for _ in range(e2e_steps):
        copies_only()
    comp.wait_stream(h2d_stream)
    comp.wait_stream(d2h_stream)
    c1.record(comp)
    torch.cuda.synchronize(dev)
    copy_floor_ms = c0.elapsed_time(c1) / e2e_steps
    del dev_out

    del g_fwd, g_bwd
    torch.cuda.synchronize(dev)
    if group is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peak, peak_kind = load_peak()
    total_E = E * world
    value = total_E / (ms_step * 1e-3)
    achieved_bwd = bwd_bytes / (ms_bwd * 1e-3) / 1e9
    step_gbs = (fwd_bytes + bwd_bytes) / (ms_step * 1e-3) / 1e9
    traffic = load_traffic(args.config)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "elements/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": dt_name,
        "data": "synthetic (seeded; BASELINE config distributions)",
        "config": {
            "workload": desc + ("" if world == 1 else f"; dim sharded: {d} channels per rank, global dim {d * world}"),
            "batch": b, "dim_per_rank": d, "seqlen": l, "dstate": n, "global_dim": d * world,
            "l2": "flushed (256 MiB write) before the forward and before the backward of every step",
            "parallelism": f"dim-shard{world}" if world > 1 else "single",
            **({"dB_dC_exchange": "peer-memory one-shot sum (NVLink)"
                if os.environ.get("MAMBA_B200_PEER_REDUCE", "1") != "0" else "NCCL all_reduce"} if world > 1 else {}),
        },
        "tokens_per_s": b * l / (ms_step * 1e-3),
        "ms_fwd": ms_fwd,
        "ms_bwd": ms_bwd,
        "hbm_frac_step": step_gbs / peak,
        "step_algorithmic_gbs": step_gbs,
        "roofline": {
            "kernel": "scan_bwd_kernel + scan_bwd_reduce_kernel (the backward op)",
            "bound": "hbm",
            "achieved": achieved_bwd,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved_bwd / peak,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
            "traffic": None if traffic is None else traffic.get("bwd_bytes_per_element", 0) * E,
            "algorithmic_bytes_per_launch": bwd_bytes,
        },
        "e2e": {"value": total_E / (e2e_ms * 1e-3), "unit": "elements/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "timing": "CUDA events around K pipelined steps, pipeline fill and drain included",
                "copy_only_ms_per_step": copy_floor_ms},
        "gpu_launches": per_step_launches * args.steps,
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, args.cpu_budget)
    print(json.dumps(line), flush=True)


def _host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def reference_step_fn(cfg, torch):
    """One fwd+bwd of the reference CPU path on the config's shapes (kernel via oracle/_ref)."""
    import oracle
    from oracle import f64, ref_c

    b, d, l, n, dt_name, has_z, _ = cfg
    host = make_inputs(cfg, None, 0, torch)
    f32 = {k: (None if v is None else v.float().contiguous()) for k, v in host.items()}
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
    step, kind = reference_step_fn(cfg, torch)
    b, d, l = cfg[0], cfg[1], cfg[2]
    t0 = time.perf_counter()
    step()  # warmup (bench_selective_scan.py:16-22 method)
    first = time.perf_counter() - t0
    iters = max(1, min(5, int(budget_s / max(first, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(iters):
        step()
    dt = (time.perf_counter() - t0) / iters
    return {"value": b * d * l / dt, "unit": "elements/s", "cores": cores, "kind": kind,
            "sample": f"{iters} timed fwd+bwd passes (after 1 warm-up) of the full config "
                      f"b={b} d={d} l={l}, {cores} threads, time.perf_counter",
            "ms_per_step": dt * 1e3}


def run_reference(args):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    cores = _host_cores()
    torch.set_num_threads(cores)
    step, kind = reference_step_fn(cfg, torch)
    b, d, l = cfg[0], cfg[1], cfg[2]
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    value = b * d * l / (ms * 1e-3)
    line = {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "elements/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded; BASELINE config distributions)",
        "config": {"workload": CONFIGS[args.config][6] + " (one shard-sized step on the host CPU)",
                   "batch": b, "dim_per_rank": d, "seqlen": l, "dstate": cfg[3]},
        "cpu_baseline": {"value": value, "unit": "elements/s", "cores": cores, "kind": kind,
                         "sample": f"{args.steps} fwd+bwd passes of b={b} d={d} l={l} after {args.warmup} warm-up"},
        "e2e": {"value": value, "unit": "elements/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true", help="kernel timing only (for profiler runs)")
    p.add_argument("--cpu-budget", type=float, default=15.0, help="seconds of CPU baseline work")
    args = p.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
