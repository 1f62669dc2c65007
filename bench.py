"""Benchmark of the fused Mamba-3 recurrence hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg1|cfg2|cfg3|cfg4] [--no-box] [--reference-gpu]

One step is one pass of the hot path over one batch: at the default
``cfg1`` (B=16 clips, T=200, H=12, Hq=1, N=128, P=64, R=32) that is the
``fused_recurrence`` launch — C/B RMSNorm of the raw q/k rows, the fused
recurrence with its SiLU(z) gate, and the length mask (lengths ~ U{120..200}).

Timing: W untimed eager warm-up steps; then the K timed steps run as CUDA-graph
replays, each step on the next of S input sets whose total size exceeds the
126 MB L2 (so every step reads its inputs from HBM), bracketed by a barrier and
``torch.cuda.synchronize()`` and timed with CUDA events on the launching
stream; the max over ranks is reported. Under torchrun every rank runs its own
batch (weak scaling; no collective on the data path).

The default line also carries ``box``: the box-level sweep of the metric's
audio-seconds/s (1024 synthetic clips through ``InferenceEngine(graphs=True)``,
batches partitioned over the ranks, one logits all-gather; strong scaling), so a
run at N = 1, 2, 4, 8 GPUs measures both halves of the metric (``--no-box`` skips it).

``e2e`` runs the same call from pinned host buffers with the copies inside the
timed region (``RaggedHostPipeline``: only the rows before each clip's length
cross the host link; ``e2e.dense`` moves the whole padded tensors).

``--impl reference`` times the reference's arithmetic on the host CPU (the
oracle port under ``oracle/``, all host threads) on the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "trifusion-fp-kernel_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "fused_mamba tokens/s + HBM GB/s vs peak; audio-sec/s at 1/2/4/8 B200"
L2_BYTES = 126 * 2 ** 20
FALLBACK_HBM_GBS = 6650.0

STUDENT = dict(dim=384, depth=8, heads=6, ffn_dim=1536, state_dim=128)
WORKLOADS = {
    # recurrence steps: (B, T, H, lengths spec)
    "cfg1": dict(kind="recurrence", batch=16, time=200, heads=12, lengths=("uniform", 120, 200)),
    "cfg2": dict(kind="recurrence", batch=2, time=3600, heads=12, lengths=("fixed", [3600, 2871])),
    # whole student forward through InferenceEngine(graphs=True)
    "cfg3": dict(kind="model", batch=16, samples=64000, lengths=("uniform", 32000, 64000)),
    # box-level sweep: 1024 clips, length buckets, LPT partition over the GPUs
    # Up to 32 clips per batch and 480 padded audio-seconds per batch: a B200-sized budget
    # (the reference's planner takes it as a setting; its L4 default is 64 s on 24 GB).
    "cfg4": dict(kind="box", clips=1024, max_batch=32, padded_seconds=480),
}
AUDIO_METRIC_UNIT = "audio-sec/s"
# Reserved-memory bound of the benchmark engines: one graph per batch shape of up to 480
# padded audio-seconds needs more than the reference's 19.5 GiB default (sized for a 24 GB L4).
BENCH_RESERVED_GIB = 64.0
# Default timed steps: each bounded to well under a minute of GPU time.
DEFAULT_STEPS = {"cfg1": 20000, "cfg2": 20000, "cfg3": 200, "cfg4": 3}
# Sweeps timed by the box sub-record of the default line.
BOX_STEPS = 3


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default per workload: cfg1/cfg2 20000 launches, cfg3 200 forwards, "
                         "cfg4 3 sweeps of 1024 clips)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg1")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-box", action="store_true",
                    help="cfg1: skip the box-level audio-seconds/s sweep (cfg4) recorded under 'box'")
    ap.add_argument("--reference-gpu", action="store_true",
                    help="one GPU: also time the reference's own GPU path (installed in baseline/_ref) "
                         "on this GPU, as 'reference_gpu': its Triton fused_mamba for cfg1/cfg2, its "
                         "deployed InferenceEngine(graphs=True) for cfg3")
    ap.add_argument("--profile-eager", type=int, default=0, metavar="K",
                    help="model workloads: run K untimed eager forwards and exit (for ncu launch lists)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = DEFAULT_STEPS[args.workload]
    return args


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def make_lengths(spec, batch, seed=0):
    import torch
    from trifusion_b200.synthetic import lengths_uniform
    if spec[0] == "uniform":
        return lengths_uniform(batch, spec[1], spec[2], seed)
    return torch.tensor(spec[1], dtype=torch.int64)


def algorithmic_bytes(b, t, h, lengths, hq=1, n=128, p=64, r=32, trap_bytes=4):
    """Bytes the masked step must move: every input row t < lengths[b] read
    once (q/k once per group, angles once: head stride 0), every output row
    written once (zeros past the length), plus the per-head parameters."""
    rows = int(sum(min(int(x), t) for x in lengths))
    return (2 * rows * hq * n * 2          # q, k
            + 2 * rows * h * p * 2          # v, z
            + rows * h * (4 + 4 + trap_bytes)  # adt, dt, trap
            + rows * r * 2                  # raw angles (broadcast over heads)
            + b * t * h * p * 2             # out (all rows)
            + h * (2 * n + 1) * 4 + 2 * n * 4 + b * 8)  # qb, kb, d, norm weights, lengths


def input_sets(base, b, t, h):
    """(bytes of one input set incl. its output buffer, number of sets cycled so that
    every timed step reads its inputs from HBM: > 3x the L2)."""
    full_set_bytes = sum(x.numel() * x.element_size() for i, x in enumerate(base) if i != 8) + \
        b * t * 32 * 2 + b * t * h * 64 * 2  # + shared angles + the output buffer
    return full_set_bytes, max(2, math.ceil(3 * L2_BYTES / full_set_bytes))


def recurrence_config(workload, wl, base, lengths, world):
    """The ``config`` of a recurrence bench line; both arms print the same dict."""
    b, t, h = wl["batch"], wl["time"], wl["heads"]
    full_set_bytes, nsets = input_sets(base, b, t, h)
    return {"workload": workload, "B": b, "T": t, "H": h, "Hq": 1, "N": 128, "P": 64,
            "R": 32, "lengths": [int(x) for x in lengths],
            "step": "RMSNorm(q,k) + fused recurrence + SiLU(z) gate + length mask, one launch",
            "l2": f"inputs cycled over {nsets} sets ({nsets * full_set_bytes / 2**20:.0f} MiB > L2)",
            "parallelism": f"replicas x{world} (one batch per GPU)"}


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons in the background.

    One sampler per node, on rank 0, covers the GPUs of every local rank (indices
    0..world-1) at the profiling recipe's 200 ms interval; the other ranks sample
    nothing, so N ranks do not start N pollers of the driver while they are timed."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, rank=0, world=1):
        self.active = rank == 0
        self.ids = list(range(max(world, 1)))
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        if not self.active:
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--id=" + ",".join(str(i) for i in self.ids), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return

        def reader():
            for line in self.proc.stdout:
                self.samples.append((time.time(), line.strip()))

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self, t0, t1):
        """Median SM clock of the slowest sampled GPU, the union of throttle reasons and
        each GPU's median (None on ranks that do not sample)."""
        if not self.active:
            return None
        rows = [s for ts, s in self.samples if t0 <= ts <= t1]
        if len(rows) < len(self.ids):  # region shorter than the sampling interval: nearest samples
            rows = [s for ts, s in sorted(self.samples, key=lambda x: abs(x[0] - (t0 + t1) / 2))[:3 * len(self.ids)]]
        mhz, max_mhz, reasons = {}, None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in rows:
            f = [x.strip() for x in row.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.setdefault(int(f[0]), []).append(float(f[1]))
                max_mhz = float(f[2])
            except ValueError:
                continue
            for name, flag in zip(names, f[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        per_gpu = {i: statistics.median(v) for i, v in sorted(mhz.items())}
        return {"sm_mhz": min(per_gpu.values()) if per_gpu else None, "sm_max_mhz": max_mhz,
                "reasons": sorted(reasons), "samples": sum(len(v) for v in mhz.values()),
                "per_gpu_sm_mhz": per_gpu}


def cpu_port_time(workload, inputs_np, lengths_np, qw, kw, budget_s=12.0):
    """Time the oracle port of the step on the host (rank 0, N=1 only)."""
    import numpy as np
    from oracle import mamba_oracle as O

    def step():
        a = list(inputs_np)
        a[0] = O.rms(a[0], qw)
        a[1] = O.rms(a[1], kw)
        return O.mask_rows(O.fused_mamba(*a, dtype=np.float32), lengths_np)

    step()
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= 50:
            break
    return n, el


def _torch_threads():
    import torch

    return torch.get_num_threads()


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, wl):
    """`--impl reference`: the reference arithmetic (oracle port) on host CPU."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = host_threads()
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    import numpy as np
    import torch
    from trifusion_b200.synthetic import recurrence_inputs, norm_weight
    torch.set_num_threads(cores)
    b, t, h = wl["batch"], wl["time"], wl["heads"]
    base = recurrence_inputs(b, t, h, kind="baseline")
    inputs = [a.float().numpy() for a in base]
    lengths = make_lengths(wl["lengths"], b).numpy()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    qw, kw = norm_weight(128, 1).numpy(), norm_weight(128, 2).numpy()
    from oracle import mamba_oracle as O

    def step():
        a = list(inputs)
        a[0] = O.rms(a[0], qw)
        a[1] = O.rms(a[1], kw)
        return O.mask_rows(O.fused_mamba(*a, dtype=np.float32), lengths)

    for _ in range(max(args.warmup, 0)):
        step()
    steps = max(1, min(args.steps, 20))
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    el = time.perf_counter() - t0
    value = b * t * steps / el
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup, "ms_per_step": el / steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": recurrence_config(args.workload, wl, base, lengths, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "torch_threads": _torch_threads(), "kind": "port",
                         "sample": f"{steps} full {args.workload} batches (B={b}, T={t}, H={h}), numpy FP32"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference arm: the oracle port of the reference arithmetic (mamba_fused.py:72-152, "
                "native.py:8-39, masking.py:10-11) on the host cores; the reference itself is Triton "
                "for sm_89 and has no CPU implementation of this path",
    }
    if args.steps != steps:
        line["note"] += f"; steps capped at {steps} of {args.steps} to bound CPU time"
    print(json.dumps(line), flush=True)


def setup_dist():
    """(world, rank, local rank, device); NCCL process group when world > 1."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    return world, rank, local, dev


def max_over_ranks(value, world, dev):
    return max(per_rank(value, world, dev))


def per_rank(value, world, dev):
    """Every rank's value (all-gathered), in rank order."""
    if world == 1:
        return [value]
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], device=dev, dtype=torch.float64)
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


def main():
    args = parse()
    wl = WORKLOADS[args.workload]
    kind = wl["kind"]
    if args.impl == "reference":
        (run_reference if kind == "recurrence" else run_reference_model)(args, wl)
        return
    {"recurrence": run_recurrence, "model": run_model, "box": run_box}[kind](args, wl)


def run_recurrence(args, wl):
    import torch
    import torch.distributed as dist
    from trifusion_b200 import fused_recurrence
    from trifusion_b200.synthetic import recurrence_inputs, norm_weight

    world, rank, local, dev = setup_dist()

    b, t, h = wl["batch"], wl["time"], wl["heads"]
    # Weak scaling: every rank gets the same shape and lengths (the per-GPU work of the
    # printed config), its own input values.
    lengths_cpu = make_lengths(wl["lengths"], b, seed=0)
    base = recurrence_inputs(b, t, h, kind="baseline", seed=rank)
    qw_cpu, kw_cpu = norm_weight(128, 1), norm_weight(128, 2)
    qw, kw = qw_cpu.to(dev), kw_cpu.to(dev)
    step_bytes = algorithmic_bytes(b, t, h, lengths_cpu.tolist())
    full_set_bytes, nsets = input_sets(base, b, t, h)
    sets = []
    for s in range(nsets):
        dev_args = [x.to(dev) if i != 8 else None for i, x in enumerate(base)]
        ang_src = base[8][:, :, :1].contiguous().to(dev)  # [B,T,1,32]; heads share it
        dev_args[8] = ang_src.expand(b, t, h, 32)
        sets.append(dict(args=dev_args, ang=ang_src, lengths=lengths_cpu.to(dev),
                         out=torch.empty(b, t, h, 64, dtype=torch.bfloat16, device=dev)))

    def step(i):
        st = sets[i % nsets]
        fused_recurrence(*st["args"], q_norm=qw, k_norm=kw, lengths=st["lengths"], out=st["out"])

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 0)):
            step(i)
        torch.cuda.synchronize(dev)
        # Exactly K launches, all as graph replays: a graph over every input set,
        # replayed K // S times, then a graph over the first K % S sets, once.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(nsets):
                step(i)
        rest = args.steps % nsets
        tail = None
        if rest:
            tail = torch.cuda.CUDAGraph()
            with torch.cuda.graph(tail, stream=stream):
                for i in range(rest):
                    step(i)
            tail.replay()
        # load phase so clock samples reflect a busy GPU
        sampler = ClockSampler(rank, world)
        sampler.start()
        tl0 = time.time()
        while time.time() - tl0 < 0.6:
            graph.replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        tw0 = time.time()
        ev0.record(stream)
        for _ in range(args.steps // nsets):
            graph.replay()
        if tail is not None:
            tail.replay()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        tw1 = time.time()
        if world > 1:
            dist.barrier()
        sampler.stop()
    ms = ev0.elapsed_time(ev1)
    rank_ms = per_rank(ms / max(args.steps, 1), world, dev)
    # L2-warm reference figure (not the headline): the same launch repeated on one input set, which
    # then stays resident in the 126 MB L2. Timed after, and outside, the measured region.
    with torch.cuda.stream(stream):
        warm_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(warm_graph, stream=stream):
            for _ in range(nsets):
                step(0)
        warm_graph.replay()
        w0 = torch.cuda.Event(enable_timing=True)
        w1 = torch.cuda.Event(enable_timing=True)
        w0.record(stream)
        for _ in range(20):
            warm_graph.replay()
        w1.record(stream)
        torch.cuda.synchronize(dev)
        warm_ms_per_step = w0.elapsed_time(w1) / (20 * nsets)
    ms_per_step = max(rank_ms)
    value = world * b * t / (ms_per_step / 1e3)
    hbm_peak, peak_kind = peaks()
    achieved = step_bytes / (ms_per_step / 1e3) / 1e9

    # End to end through the public call with host buffers: every step copies its
    # inputs in from pinned host memory and its output back (HostPipeline: two
    # device buffer sets and copy-in / compute / copy-out streams, so one step's
    # copies overlap its neighbours' kernels). Timed from the first copy-in to
    # the last copy-out.
    from trifusion_b200.host_pipeline import HostPipeline

    host_in = [x.pin_memory() if i != 8 else x[:, :, :1].contiguous().pin_memory()
               for i, x in enumerate(base)] + [lengths_cpu.pin_memory()]
    host_outs = [torch.empty(b, t, h, 64, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    h2d = sum(x.numel() * x.element_size() for x in host_in)
    d2h = host_outs[0].numel() * 2

    def e2e_call(*xs, out):
        xs = list(xs)
        xs[8] = xs[8].expand(b, t, h, 32)  # [B,T,1,32] copied once; the heads share it
        fused_recurrence(*xs[:11], q_norm=qw, k_norm=kw, lengths=xs[11], out=out)

    # One pinned host block per step holding all inputs (filled once here), moved by one copy.
    pipe = HostPipeline(e2e_call, host_in, (b, t, h, 64), torch.bfloat16, device=dev, writes_out=True,
                        packed=True)
    host_block, views = pipe.host_block()
    for view, x in zip(views, host_in):
        view.copy_(x)
    h2d = host_block.numel()  # the bytes copied per step (inputs at 256-byte-aligned offsets)
    for i in range(16):
        pipe.submit(host_block, host_outs[i % 2])
    pipe.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(pipe.copy_in)
    for i in range(args.e2e_steps):
        pipe.submit(host_block, host_outs[i % 2])
    e1.record(pipe.copy_out)
    torch.cuda.synchronize(dev)
    e_ms = e0.elapsed_time(e1) / max(args.e2e_steps, 1)
    if world > 1:
        tt = torch.tensor([e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e_ms = float(tt.item())
    dense_e2e = {"value": world * b * t / (e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                 "d2h_bytes_per_step": d2h,
                 "pipeline": "HostPipeline depth 2, packed: whole padded tensors, one input copy per step"}

    # The same call with only the valid rows crossing the host link (RaggedHostPipeline:
    # lengths, per-head parameters and valid rows packed in one host block; the device
    # scatters them into the padded tensors, and only the output's valid rows come back).
    from trifusion_b200.host_pipeline import RaggedHostPipeline

    rag_in = [x if i != 8 else x[:, :, :1] for i, x in enumerate(host_in[:11])]
    rag_kinds = ["time_major", "time_major", "time_major", "time_minor", "time_minor", "time_minor",
                 None, None, "time_major", None, "time_major"]
    rpipe = RaggedHostPipeline(e2e_call, [x.contiguous() for x in rag_in], rag_kinds, (b, t, h, 64),
                               torch.bfloat16, device=dev, graphs=True)
    rblock, rout = rpipe.host_block(), rpipe.host_out()
    r_in = rpipe.pack(rblock, rag_in, lengths_cpu)
    r_out = rpipe.out_bytes(lengths_cpu.tolist())
    for i in range(16):  # graph captures on the first step of each buffer set, then a settled stream
        rpipe.submit(rblock, r_in, rout, r_out)
    rpipe.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(rpipe.copy_in)
    for i in range(args.e2e_steps):
        rpipe.submit(rblock, r_in, rout, r_out)
    e1.record(rpipe.copy_out)
    torch.cuda.synchronize(dev)
    r_ms = e0.elapsed_time(e1) / max(args.e2e_steps, 1)
    if world > 1:
        tt = torch.tensor([r_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        r_ms = float(tt.item())
    e2e_value = world * b * t / (r_ms / 1e3)
    h2d, d2h = r_in, r_out

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import numpy as np
        np_in = [x.float().numpy() for x in base]
        n, el = cpu_port_time(args.workload, np_in, lengths_cpu.numpy(), qw_cpu.numpy(), kw_cpu.numpy())
        cpu = {"value": b * t * n / el, "unit": "tokens/s", "cores": host_threads(), "torch_threads": _torch_threads(), "kind": "port",
               "sample": f"{n} full {args.workload} batches through the numpy oracle (FP32), {el:.1f} s"}

    ref_gpu = None
    if args.reference_gpu and world == 1:
        ref_gpu = reference_gpu_record(sets, qw, kw, dev, ms_per_step * 1e3)

    box = None
    if args.workload == "cfg1" and not args.no_box:
        # The box-level sweep of the metric's audio-seconds/s (cfg4), on the same ranks:
        # strong scaling over the ranks, one logits all-gather.
        del graph, tail, warm_graph
        box = box_sweep(WORKLOADS["cfg4"], BOX_STEPS, 1, world, rank, local, dev)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    clocks = sampler.summary(tl0, tw1)
    traffic = measured_traffic(args.workload)
    tensor_pct = measured_traffic(args.workload, column=3)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": recurrence_config(args.workload, wl, base, lengths_cpu.tolist(), world),
        "hbm_gbs": achieved,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": traffic,
                     "tensor_pipe_active_pct_ncu": tensor_pct,
                     "kernel_source_sha16": kernel_source_hash(),
                     "l2_warm": {"ms_per_step": warm_ms_per_step,
                                 "value": world * b * t / (warm_ms_per_step / 1e3)},
                     "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": step_bytes},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "pipeline": "RaggedHostPipeline depth 2: lengths, parameters and valid rows in one copy, valid "
                            "output rows back; copies overlap kernels; the device work of a step (row scatter, "
                            "fused_recurrence, row gather) replayed as a CUDA graph", "dense": dense_e2e},
        "gpu_launches": args.steps,
        "rank_ms_per_step": rank_ms,
        "clocks": clocks,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if ref_gpu is not None:
        line["reference_gpu"] = ref_gpu
    if box is not None:
        line["box"] = dict(workload="cfg4", scaling="strong", **box)
    print(json.dumps(line), flush=True)


def reference_gpu_record(sets, qw, kw, dev, ours_us):
    """The reference's own GPU path on the same inputs and GPU: its Triton RMSNorm on q
    and k, then its Triton ``fused_mamba`` (``mamba_fused.py:155-191``), timed the same
    way as our step (one CUDA graph over every input set, CUDA events). The reference
    has no length mask inside the recurrence (it masks afterwards, ``model.py:174``),
    so its step covers all T steps of every row. Also reports the relative L2 distance
    between the two outputs over the valid rows (the reference rounds its operands to
    BF16, ours to FP16 with exponents). Needs the reference installed under
    ``baseline/_ref`` (``pip install --no-index --no-deps --target baseline/_ref``)."""
    import torch

    ref_root = ROOT / "baseline" / "_ref"
    if not (ref_root / "trifusion_l4").is_dir():
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    sys.path.insert(0, str(ref_root))
    try:
        import trifusion_l4.mamba_fused as ref_fused
        import trifusion_l4.kernels.native as ref_native
    except Exception as exc:  # noqa: BLE001 - reported, not raised
        return {"unavailable": f"import of the reference failed: {exc!r}"[:200]}

    def ref_step(st):
        a = st["args"]
        return ref_fused.fused_mamba(ref_native.rms(a[0], qw), ref_native.rms(a[1], kw), *a[2:])

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        y_ref = ref_step(sets[0]).float()
        torch.cuda.synchronize(dev)
        y_our = sets[0]["out"].float()
        lengths = sets[0]["lengths"]
        valid = (torch.arange(y_ref.shape[1], device=dev)[None, :] < lengths[:, None])[:, :, None, None]
        diff = (y_ref - y_our) * valid
        rel = float(diff.norm() / (y_ref * valid).norm())
        for i in range(3):
            ref_step(sets[i % len(sets)])
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for st in sets:
                ref_step(st)
        graph.replay()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / (reps * len(sets))
    del graph
    return {"us_per_step": us, "ours_us_per_step": ours_us, "ours_speedup": us / ours_us,
            "rel_l2_vs_ours_valid_rows": rel,
            "what": "reference Triton RMSNorm(q), RMSNorm(k) + fused_mamba, graph replays over the same input sets"}


def _student(dev, tmpdir, optimized=True):
    from trifusion_b200 import load_student
    from trifusion_b200.synthetic import student_checkpoint

    path = student_checkpoint(Path(tmpdir) / "student.pt", STUDENT, seed=0)
    return load_student(path, optimized=optimized, device=dev)


def _l2_flush_buffer(dev):
    import torch

    return torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)


def run_model(args, wl):
    """cfg3: one step = one ``InferenceEngine(graphs=True)`` call on a [16, 1, 64000]
    batch (graph replay: input copies into the graph's buffers, the forward,
    the owned logits copy). Each timed step is bracketed by its own CUDA events
    with an L2 flush (a 252 MiB write) before it, outside the events."""
    import tempfile

    import torch
    import torch.distributed as dist
    from trifusion_b200 import InferenceEngine, configure_runtime
    from trifusion_b200.synthetic import synthetic_audio

    world, rank, local, dev = setup_dist()
    configure_runtime()
    b, n = wl["batch"], wl["samples"]
    lengths = make_lengths(wl["lengths"], b, seed=0)  # every rank: the config's lengths, its own audio
    audio, lengths, channels = synthetic_audio(b, n, lengths=lengths, seed=rank)
    with tempfile.TemporaryDirectory() as tmp:
        model = _student(dev, tmp)
        ref_model = None
        if args.reference_gpu and world == 1:
            ref_model = _reference_student(dev, tmp)
    inputs = tuple(x.to(dev) for x in (audio, lengths, channels))
    if args.profile_eager:
        eager = InferenceEngine(model, graphs=False)
        for _ in range(args.profile_eager):
            eager(*inputs)
        torch.cuda.synchronize(dev)
        return
    engine = InferenceEngine(model, graphs=True, max_graphs=1, max_reserved_gib=BENCH_RESERVED_GIB)
    flush = _l2_flush_buffer(dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 1)):
        engine(*inputs)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(rank, world)
    sampler.start()
    tl0 = time.time()
    while time.time() - tl0 < 0.6:
        engine(*inputs)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    for e0, e1 in events:
        flush.fill_(1)
        e0.record(stream)
        engine(*inputs)
        e1.record(stream)
    torch.cuda.synchronize(dev)
    tw1 = time.time()
    sampler.stop()
    ms = sum(e0.elapsed_time(e1) for e0, e1 in events)
    ms = max_over_ranks(ms, world, dev)
    ms_per_step = ms / max(args.steps, 1)
    audio_s = float(lengths.sum()) / 16000
    value = world * audio_s / (ms_per_step / 1e3)

    # End to end: pinned host audio in, logits back to pinned host memory, every
    # step, through HostPipeline (the copies of one batch overlap the forward of
    # its neighbours). The L2 flush runs inside each step here, so it is timed.
    from trifusion_b200.host_pipeline import HostPipeline

    host = [x.pin_memory() for x in (audio, lengths, channels)]
    host_outs = [torch.empty(b, 5).pin_memory() for _ in range(2)]
    h2d = sum(x.numel() * x.element_size() for x in host)

    def e2e_call(*xs):
        flush.fill_(1)
        return engine(*xs)

    pipe = HostPipeline(e2e_call, host, (b, 5), torch.float32, device=dev)
    for i in range(3):
        pipe.submit(host, host_outs[i % 2])
    pipe.synchronize()
    n_e2e = min(args.steps, args.e2e_steps)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(pipe.copy_in)
    for i in range(n_e2e):
        pipe.submit(host, host_outs[i % 2])
    e1.record(pipe.copy_out)
    torch.cuda.synchronize(dev)
    e_ms = e0.elapsed_time(e1) / max(n_e2e, 1)
    e_ms = max_over_ranks(e_ms, world, dev)
    ref_gpu = None
    if ref_model is not None:
        ref_gpu = reference_model_gpu_record(ref_model, engine, inputs, flush, args, audio_s, ms_per_step)
    if world > 1:
        dist.barrier()
        engine.clear()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": AUDIO_METRIC_UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 1), "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init student, PCM16-quantised noise)",
        "config": {"workload": args.workload, "student": STUDENT, "batch": b, "samples": n,
                   "channels": 1, "audio_seconds_per_step": audio_s,
                   "step": "InferenceEngine(graphs=True) replay incl. input/output copies",
                   "l2": "252 MiB write before every timed step (outside the events)",
                   "parallelism": f"replicas x{world} (one batch per GPU)"},
        "roofline": None,
        "e2e": {"value": world * audio_s / (e_ms / 1e3), "unit": AUDIO_METRIC_UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": b * 5 * 4,
                "pipeline": "HostPipeline depth 2 (copies overlap the forward; L2 flush timed)"},
        "clocks": sampler.summary(tl0, tw1),
    }
    if ref_gpu is not None:
        line["reference_gpu"] = ref_gpu
    print(json.dumps(line), flush=True)


def _reference_student(dev, tmpdir):
    """The reference's own deployed model (``baseline/_ref``) on the same synthetic
    checkpoint, or a string saying why it is unavailable."""
    from trifusion_b200.synthetic import student_checkpoint

    ref_root = ROOT / "baseline" / "_ref"
    if not (ref_root / "trifusion_l4").is_dir():
        return "the reference is not installed under baseline/_ref"
    sys.path.insert(0, str(ref_root))
    try:
        from trifusion_l4.runtime import load_student as ref_load
    except Exception as exc:  # noqa: BLE001 - reported, not raised
        return f"import of the reference failed: {exc!r}"[:200]
    path = student_checkpoint(Path(tmpdir) / "reference_student.pt", STUDENT, seed=0)
    return ref_load(path, optimized=True, device=dev)


def reference_model_gpu_record(ref_model, engine, inputs, flush, args, audio_s, ours_ms):
    """The reference's deployed path on the same GPU, batch and weights: its
    ``InferenceEngine(graphs=True)`` (fused Triton kernels, BF16 autocast, CUDA graph
    replay; ``runtime.py:67-138``), timed like our step (an L2 flush before every step,
    outside the CUDA events). Also the largest difference between the two engines'
    sigmoid probabilities on this batch."""
    import torch

    if isinstance(ref_model, str):
        return {"unavailable": ref_model}
    from trifusion_l4.runtime import InferenceEngine as RefEngine

    ref_engine = RefEngine(ref_model, graphs=True, max_graphs=1, max_reserved_gib=BENCH_RESERVED_GIB)
    dev = inputs[0].device
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 1)):
        ref_logits = ref_engine(*inputs)
    ours = engine(*inputs)
    torch.cuda.synchronize(dev)
    diff = float((ours.float().sigmoid() - ref_logits.float().sigmoid()).abs().max())
    steps = max(1, min(args.steps, 50))
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in events:
        flush.fill_(1)
        e0.record(stream)
        ref_engine(*inputs)
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = sum(e0.elapsed_time(e1) for e0, e1 in events) / steps
    ref_engine.clear()
    return {"ms_per_step": ms, "value": audio_s / (ms / 1e3), "unit": AUDIO_METRIC_UNIT, "steps": steps,
            "graph_hits": ref_engine.graph_hits, "disabled_shapes": len(ref_engine.disabled_shapes),
            "ours_ms_per_step": ours_ms, "ours_speedup": ms / ours_ms,
            "max_probability_difference_vs_ours": diff,
            "what": "reference load_student(optimized=True) + InferenceEngine(graphs=True) on the same "
                    "synthetic checkpoint and batch"}


def box_sweep(wl, steps, warmup, world, rank, local, dev):
    """The cfg4 box sweep on an initialised rank: 1024 clips bucketed by (channels,
    length) into batches of up to 32, partitioned over the ranks longest-processing-time
    first; one step = every rank runs all of its batches through its
    ``InferenceEngine(graphs=True)`` (one graph per batch shape, captured during
    warm-up) and the logits are all-gathered once. Returns the measurements (max over
    ranks); inputs are device-resident for ``value`` and copied from pinned host memory
    batch by batch for ``e2e``."""
    import tempfile

    import torch
    import torch.distributed as dist
    from trifusion_b200 import InferenceEngine, configure_runtime
    from trifusion_b200.audio import plan_batches
    from trifusion_b200.sharding import batch_cost, gather_logits, lpt_partition
    from trifusion_b200.synthetic import batch_audio, clip_set

    configure_runtime()
    records = clip_set(wl["clips"], seed=0)
    plan = plan_batches(records, padded_seconds=wl["padded_seconds"], max_batch=wl["max_batch"])
    parts = lpt_partition([batch_cost(lim, rows) for lim, rows in plan], world)
    mine = parts[rank]
    # Every rank computes the same partition, so the largest rank's clip count bounds
    # the gather: one all-gather of logits at the end.
    capacity = max(sum(len(plan[i][1]) for i in p) for p in parts)
    host = [tuple(x.pin_memory() for x in batch_audio(plan[i][0], plan[i][1], seed=0)) for i in mine]
    indices = torch.tensor([r.index for i in mine for r in plan[i][1]], dtype=torch.int64, device=dev)
    dev_in = [tuple(x.to(dev) for x in h) for h in host]
    shapes = {tuple(h[0].shape) for h in host}
    with tempfile.TemporaryDirectory() as tmp:
        model = _student(dev, tmp)
    engine = InferenceEngine(model, graphs=True, max_graphs=max(len(shapes), 1),
                             max_reserved_gib=BENCH_RESERVED_GIB)
    total_audio_s = sum(r.samples for r in records) / 16000
    stream = torch.cuda.current_stream(dev)

    def sweep(inputs):
        outs = [engine(*x) for x in inputs]
        local_logits = torch.cat(outs) if outs else torch.zeros(0, 5, device=dev)
        if world > 1:
            return gather_logits(indices, local_logits, capacity=capacity)
        return indices, local_logits

    for _ in range(max(warmup, 1)):
        sweep(dev_in)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(rank, world)
    sampler.start()
    tl0 = time.time()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
    for e0, e1 in events:
        e0.record(stream)
        idx, logits = sweep(dev_in)
        e1.record(stream)
    torch.cuda.synchronize(dev)
    tw1 = time.time()
    sampler.stop()
    rank_ms = per_rank(sum(a.elapsed_time(c) for a, c in events) / max(steps, 1), world, dev)
    ms_per_step = max(rank_ms)
    assert idx.numel() == len(records) and bool(torch.isfinite(logits).all())

    h2d = sum(x.numel() * x.element_size() for h in host for x in h)

    def e2e_sweep():
        staged = []
        for h, d in zip(host, dev_in):
            for src, dst in zip(h, d):
                dst.copy_(src, non_blocking=True)
            staged.append(d)
        idx_, logits_ = sweep(staged)
        return logits_.to("cpu", non_blocking=True)

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    e0.record(stream)
    e2e_sweep()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    if world > 1:
        dist.barrier()
    engine.clear()
    return {
        "value": total_audio_s / (ms_per_step / 1e3), "unit": AUDIO_METRIC_UNIT, "steps": steps,
        "warmup": max(warmup, 1), "ms_per_step": ms_per_step, "rank_ms_per_step": rank_ms,
        "config": {"student": STUDENT, "clips": len(records), "audio_seconds": total_audio_s,
                   "batches": len(plan), "batches_on_rank0": len(mine) if rank == 0 else None,
                   "graph_shapes_on_rank0": len(shapes) if rank == 0 else None,
                   "max_batch": wl["max_batch"], "padded_seconds_per_batch": wl["padded_seconds"],
                   "step": "all batches through InferenceEngine(graphs=True) + one logits all-gather",
                   "l2": "inputs larger than L2 (the sweep streams all batches)",
                   "parallelism": f"data-parallel x{world}, LPT partition by padded audio-seconds"},
        "e2e": {"value": total_audio_s / (e_ms / 1e3), "unit": AUDIO_METRIC_UNIT,
                "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": len(records) * 5 * 4},
        "clocks": sampler.summary(tl0, tw1),
    }


def run_box(args, wl):
    """cfg4 as its own bench line (see ``box_sweep``)."""
    import torch.distributed as dist

    world, rank, local, dev = setup_dist()
    res = box_sweep(wl, args.steps, args.warmup, world, rank, local, dev)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": res["value"], "unit": AUDIO_METRIC_UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": res["warmup"],
        "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init student, 1024 PCM16-quantised noise clips)",
        "config": dict(workload=args.workload, **res["config"]),
        "roofline": None, "e2e": res["e2e"], "clocks": res["clocks"],
    }
    print(json.dumps(line), flush=True)


def run_reference_model(args, wl):
    """`--impl reference` for cfg3/cfg4: the reference model's arithmetic on the
    host CPU (FP32, this package's host model with the reference formulas and
    the oracle recurrence), on a bounded sample of clips."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import tempfile

    import numpy as np
    import torch
    from oracle import mamba_oracle as O
    import trifusion_b200.mamba_fused as mf
    from trifusion_b200.synthetic import synthetic_audio

    cores = host_threads()
    torch.set_num_threads(cores)

    def oracle_recurrence(q, k, v, adt, dt, trap, qb, kb, angles, d, z, warps=8):
        a = [t.detach().float().numpy() for t in (q, k, v, adt, dt, trap, qb, kb, angles, d, z)]
        return torch.from_numpy(np.asarray(O.fused_mamba(*a, dtype=np.float32), np.float32))

    mf.fused_mamba = oracle_recurrence
    with tempfile.TemporaryDirectory() as tmp:
        model = _student("cpu", tmp, optimized=False)
    b, n = 2, 64000
    audio, lengths, channels = synthetic_audio(b, n, lengths=[64000, 48000], seed=0)
    with torch.inference_mode():
        model(audio, lengths, channels)
        steps = max(1, min(args.steps, 3))
        t0 = time.perf_counter()
        for _ in range(steps):
            model(audio, lengths, channels)
        el = time.perf_counter() - t0
    audio_s = float(lengths.sum()) / 16000
    value = audio_s * steps / el
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": AUDIO_METRIC_UNIT,
        "n_gpus": args.gpus, "steps": steps, "warmup": 1, "ms_per_step": el / steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": args.workload, "student": STUDENT},
        "cpu_baseline": {"value": value, "unit": AUDIO_METRIC_UNIT, "cores": cores, "torch_threads": _torch_threads(), "kind": "port",
                         "sample": f"{steps} forwards of 2 clips (4 s, 3 s) on the host, FP32"},
        "e2e": {"value": value, "unit": AUDIO_METRIC_UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


KERNEL_SOURCES = ("recurrence_persistent.cu", "recurrence.cuh", "sm100.cuh", "tf_common.cuh")


def kernel_source_hash():
    """First 16 hex digits of the SHA-256 over the recurrence kernel's source files."""
    import hashlib

    h = hashlib.sha256()
    for name in KERNEL_SOURCES:
        h.update((ROOT / "trifusion-fp-kernel_b200" / "csrc" / name).read_bytes())
    return h.hexdigest()[:16]


def measured_traffic(workload, column=2):
    """A figure of the committed ncu summary (column 2: DRAM bytes per launch; 3: tensor-pipe
    active %), or None when it is absent or was captured on other kernel sources (column 4
    holds the source hash of the capture)."""
    path = ROOT / "profiles" / "traffic.txt"
    if not path.exists():
        return None
    current = kernel_source_hash()
    for row in path.read_text().splitlines():
        f = row.split()
        if len(f) > 4 and f[0] == workload and f[4] == current:
            try:
                return float(f[column])
            except ValueError:
                return None
    return None


if __name__ == "__main__":
    main()
