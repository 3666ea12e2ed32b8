#!/usr/bin/env python
"""Learner-step throughput: samples/s of the fused fwd + bwd + loss + Adam step.

Workload (default): c3, actor + critic 27-512-512-512-{9,1}, global batch 1,048,576
rows split evenly over the ranks (strong scaling), one flat-gradient all-reduce per
step between the backward and the replicated Adam. Inputs are seeded synthetic
learner batches with the real inputs' shapes and distributions (tic-tac-toe boards,
Dirichlet(0.3) targets, N(0,1) old logits, 5-step returns).

Timed quantities (one JSON line on rank 0):
  value       samples/s with the batch already in HBM: K steps between CUDA events on
              the learner's stream, max over ranks
  e2e         the same through the public API with pinned HOST buffers: each step
              copies its batch host->device (HostFeed: the upload of step i+1 runs on a
              copy stream during step i) and reads the loss statistics back
  roofline    the dominant kernel (the hidden-layer GEMM) timed with CUDA events on the
              same stream with the step's shapes; algorithmic FLOPs / duration vs the
              measured peak
  cpu_baseline the CPU restatement (float32 numpy) on a bounded sample, rank 0, N = 1

L2: a workload whose inputs and activations exceed the 126 MB L2 (c2, c3, c4) is timed
over K back-to-back steps; one that fits (c0, c1) is timed one step at a time, with a
write of twice the L2 size between steps outside the timed events, and `value` is the
mean of those step times. --graph (one GPU) replays each step as one CUDA graph, which
the small, launch-latency-bound workloads want.

--impl reference times the reference's computation on the host CPU (the reference
is Mojo GPU code with no CPU path and no runnable toolchain here, so its algorithm is
run as the float32 numpy restatement), with all host threads.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c3] [--graph]
                  [--impl ours|reference]
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from spo_mojo_b200.workloads import WORKLOADS, init_params, make_batch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c3", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="budget of the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--engine", default="tensor", choices=["tensor", "cuda"],
                    help="tensor: tcgen05 3xTF32 for the hidden layers; cuda: fp32 FMA everywhere")
    ap.add_argument("--graph", action="store_true",
                    help="replay each learner step as one CUDA graph (one GPU; for the small, "
                         "launch-bound workloads)")
    ap.add_argument("--rows", type=int, default=0,
                    help="override the global batch (profiling of small cases only; not a bench line)")
    ap.add_argument("--roofline-only", type=int, default=0, metavar="ROWS",
                    help="launch only the roofline kernel at ROWS rows and print its line (for an ncu "
                         "capture of a small case; not a bench line)")
    ap.add_argument("--peaks", action="store_true",
                    help="measure the tcgen05 TF32 and FP32-FMA peaks of this GPU (not a bench line) and exit")
    return ap.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------- CPU arm
def cpu_learner_step(wl, params, batch, nets_state=None):
    from oracle import spo_oracle as O
    hp = dict(lr_actor=wl.lr, lr_critic=wl.lr, b1=wl.beta1, b2=wl.beta2, eps=wl.adam_eps,
              max_norm=wl.max_grad_norm, kl_eps=wl.kl_eps, dual=wl.dual, step=1)
    nets = {}
    for which in ("actor", "critic"):
        if which in params:
            p = params[which]
            nets[which] = {"params": p, "m": [(np.zeros_like(w), np.zeros_like(b)) for w, b in p],
                           "v": [(np.zeros_like(w), np.zeros_like(b)) for w, b in p]}
    b = dict(batch)
    if not wl.dual:
        b["logits_old"] = None
    return O.learner_step(b, actor=nets.get("actor"), critic=nets.get("critic"),
                          log_alpha=wl.log_alpha if wl.dual else None, hp=hp, dtype=np.float32)


def cpu_measure(wl, seconds, steps=None, warmup=0):
    """samples/s of the float32 CPU restatement on a bounded sample of the workload."""
    sample_rows = min(wl.batch, 8192)
    params = init_params(wl, seed=0)
    batch = make_batch(wl, sample_rows, seed=7)
    for _ in range(warmup):
        cpu_learner_step(wl, params, batch)
    times = []
    t_end = time.perf_counter() + seconds
    n = 0
    while (steps is None and (n == 0 or time.perf_counter() < t_end)) or (steps is not None and n < steps):
        t0 = time.perf_counter()
        cpu_learner_step(wl, params, batch)
        times.append(time.perf_counter() - t0)
        n += 1
    per_step = statistics.median(times)
    return sample_rows / per_step, sample_rows, len(times), per_step


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    cores = os.cpu_count()
    try:
        import threadpoolctl
        threadpoolctl.threadpool_limits(cores)
    except Exception:
        pass
    sps, rows, n, per_step = cpu_measure(wl, seconds=1e9, steps=args.steps, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": "learner samples/sec (fwd+bwd+loss+Adam)", "value": sps,
        "unit": "samples/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        # the time of the step that was timed: one sample of rows_timed rows of the workload
        "ms_per_step": per_step * 1e3, "rows_timed": rows, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl.describe(), "global_batch": wl.batch,
                   "sample_rows_per_step": rows},
        "cpu_baseline": {"value": sps, "unit": "samples/s", "cores": cores, "kind": "port",
                         "sample": f"{rows} rows of the workload per step, {n} steps; the reference "
                                   "is Mojo GPU-only, its algorithm runs as the float32 numpy restatement"},
        "e2e": {"value": sps, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling every 50 ms on a reader thread, each line time-stamped on
    arrival. start() waits (bounded) for the first line, so a short job is still covered;
    mark() and stop() bracket the timed region, whose samples are the ones reported (all
    samples since start() when the region was shorter than the interval)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    INTERVAL_MS = 50

    def __init__(self, gpu_indices):
        self.gpus = ",".join(str(g) for g in gpu_indices)
        self.proc = None
        self.lines = []
        self.t_mark = None
        self._reader = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line))

    def start(self, wait_s=5.0):
        import threading
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpus, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", str(self.INTERVAL_MS)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self._reader = threading.Thread(target=self._read, daemon=True)
        self._reader.start()
        t_end = time.perf_counter() + wait_s
        while not self.lines and time.perf_counter() < t_end and self.proc.poll() is None:
            time.sleep(0.01)

    def mark(self):
        """The start of the timed region."""
        self.t_mark = time.perf_counter()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        t_stop = time.perf_counter()
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self._reader is not None:
            self._reader.join(timeout=5)
        lines = list(self.lines)
        window = "timed region"
        if self.t_mark is not None:
            inside = [(t, ln) for t, ln in lines if self.t_mark <= t <= t_stop + self.INTERVAL_MS / 1e3]
            if inside:
                lines = inside
            else:
                window = "warm-up and timed region (the timed region was shorter than the interval)"
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for _, line in lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "window": window}


# ---------------------------------------------------------------- GPU arm
def roofline_hidden_gemm(args, rows, H, dev, stream, engine="tensor", reps=20):
    """Time the dominant kernel — the hidden x hidden forward GEMM with the step's shape —
    through the same C-ABI entry the learner uses, with CUDA events on the step's stream.
    achieved = algorithmic fp32 FLOPs (2 rows H^2) / average launch time."""
    import ctypes
    import torch
    from spo_mojo_b200 import ffi
    pk, kind = peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.rand(rows, H, device=dev, generator=g)
    w = torch.rand(H, H, device=dev, generator=g)
    bb = torch.zeros(H, device=dev)
    y = torch.empty(rows, H, device=dev)
    if engine == "tensor":
        # as the learner runs a hidden layer that feeds another: the activations and W^T as
        # TF32 hi/lo pairs, the output as a hi/lo pair with its packed ReLU mask
        xh, xl = torch.empty_like(x), torch.empty_like(x)
        ffi.call("spo_split_tf32", stream.cuda_stream, xh.data_ptr(), xl.data_ptr(), x.data_ptr(), x.numel(), 0)
        wh, wl = torch.empty_like(w), torch.empty_like(w)
        ffi.call("spo_split_tf32", stream.cuda_stream, wh.data_ptr(), wl.data_ptr(), w.data_ptr(), w.numel(), 0)
        del x
        yl = torch.empty_like(y)
        bits = torch.empty(rows, H // 32, dtype=torch.int32, device=dev)
        d = ffi.TcGemmDesc(kind=ffi.TC_FWD, a_hi=xh.data_ptr(), a_lo=xl.data_ptr(), b_hi=wh.data_ptr(),
                           b_lo=wl.data_ptr(), m=rows, n=H, k=H, bias=bb.data_ptr(), c_hi=y.data_ptr(),
                           c_lo=yl.data_ptr(), c_bits=bits.data_ptr())
        launch = lambda: ffi.call("spo_tc_gemm", stream.cuda_stream, ctypes.byref(d))  # noqa: E731
        name = "tc_gemm_kernel (tcgen05 3xTF32, hi/lo operands), hidden forward %dx%dx%d" % (rows, H, H)
    else:
        launch = lambda: ffi.call("spo_linear_fwd", stream.cuda_stream, y.data_ptr(), x.data_ptr(),  # noqa: E731
                                  w.data_ptr(), bb.data_ptr(), rows, H, H, 1)
        name = "gemm_simt_kernel (fp32 FMA), hidden forward %dx%dx%d" % (rows, H, H)
    for _ in range(3):
        launch()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    for _ in range(reps):
        launch()
    k1.record(stream)
    k1.synchronize()
    kms = k0.elapsed_time(k1) / reps
    flops = 2.0 * rows * H * H
    achieved = flops / (kms / 1e3) / 1e12
    # the kernel is timed alone (back-to-back launches of it): the burst peak applies
    peak = pk.get("bf16_tflops") or pk.get("bf16_tflops_sustained")
    traffic = TRAFFIC_PER_LAUNCH.get((engine, H), {}).get("bytes") if rows == 1048576 else None
    # the layer's fp32 essentials: A read once, C written once, its packed mask, W, bias (the
    # kernel moves A and C as TF32 hi/lo pairs: twice these activation bytes)
    fp32_bytes = 4.0 * (2 * rows * H + H * H + H) + rows * H / 8
    roof = {"bound": "tensor", "kernel": name, "achieved": achieved, "peak": peak,
            "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_kind": f"{kind} bf16 dense, burst (the kernel is timed alone)",
            "frac_of_sustained_peak": achieved / (pk.get("bf16_tflops_sustained") or peak),
            "ms_per_launch": kms,
            "traffic": traffic,
            "traffic_source": TRAFFIC_PER_LAUNCH.get((engine, H), {}).get("source"),
            "fp32_algorithmic_bytes": fp32_bytes,
            "traffic_vs_fp32_bytes": traffic / fp32_bytes if traffic else None}
    if engine == "tensor":
        # 3xTF32 issues three TF32 MMAs per fp32 product; TF32 runs at half the bf16 rate
        roof["tf32_mma_tflops"] = 3 * achieved
        roof["tf32_frac_of_half_bf16_peak"] = 3 * achieved / (peak / 2)
        # and against the TF32 MMA rate measured live on this GPU (spo_measure_peaks)
        t, f = ctypes.c_double(), ctypes.c_double()
        ffi.call("spo_measure_peaks", stream.cuda_stream, ctypes.byref(t), ctypes.byref(f))
        roof["tf32_mma_peak_measured_tflops"] = t.value / 1e12
        roof["frac_of_measured_3xtf32_ceiling"] = 3 * achieved / (t.value / 1e12)
    return roof


# DRAM bytes (read + write) of one launch of the roofline kernel at 1,048,576 rows, from an
# ncu capture of the same kernel at 262,144 rows scaled by the 4x rows (the kernel streams
# its activations once, so traffic grows with the rows): dram__bytes_read.sum 1,076,124,672
# + dram__bytes_write.sum 1,043,872,000 (profiles/roofline_tc_gemm_fwd_c3.md).
TRAFFIC_PER_LAUNCH = {
    ("tensor", 512): {"bytes": 4 * (1076124672 + 1043872000),
                      "source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of this kernel at 262,144 rows "
                                "(bench.py --roofline-only 262144), x4 rows"},
}


TC0_MIN_ROWS = 16384  # the library runs the input layer on tensor cores from this many rows


SMALL_MAX_ROWS = 8192  # batches up to this many rows run as one launch when the shapes fit


SMALL_MAX_SMEM_FLOATS = 220 * 1024 // 4  # the one-launch step's shared memory per CTA


def small_step_fits(wl, rows):
    """Whether the library runs this step as its one-launch small-batch step: every
    network's weights, biases and one 32-row block of activations fit in shared memory
    (the layout of small_step.cu)."""
    if rows < 1 or rows > SMALL_MAX_ROWS:
        return False
    pad4 = lambda v: (v + 3) // 4 * 4  # noqa: E731
    for net in (wl.actor, wl.critic):
        if net is None:
            continue
        d = list(net.dims)
        L = len(d) - 1
        if not (2 <= L <= 4 and d[0] <= 32 and d[-1] in (1, 9)):
            return False
        if any(h % 32 or h > 256 for h in d[1:-1]):
            return False
        if sum(d[i] * d[i + 1] + d[i + 1] for i in range(L)) > 65536:
            return False
        dmax = max([pad4(d[-1])] + d[1:-1])
        f = 32 * 32 + 32 * 28 + 8 * 8 + 32 * sum(d[1:-1]) + 2 * 32 * dmax
        f += 255  # to the 1024-byte boundary of the weight slabs
        f += sum((32 if i == 0 else d[i]) * d[i + 1] + pad4(d[i + 1]) for i in range(L))
        if f > SMALL_MAX_SMEM_FLOATS:
            return False
    return True


def count_launches(wl, clip, engine="tensor", rows=None, world=1):
    """libspo_cuda kernel launches of one learner step on `rows` rows (per rank)."""
    rows = wl.batch if rows is None else rows
    if small_step_fits(wl, rows):
        return 1 if world == 1 else 2    # the step; or backward, then Adam after the all-reduce
    n = 0
    for net in (wl.actor, wl.critic):
        if net is None:
            continue
        L = net.num_layers
        n += (L - 1) + 1 + (L - 1) + (L - 2)    # forward GEMMs, head, dW GEMMs, dX GEMMs
        hidden = net.dims[1:-1]
        if engine == "tensor" and L >= 3 and all(h % 128 == 0 and h <= 1024 for h in hidden):
            n += L - 2                           # per-step TF32 split of the hidden weights
            if net.dims[0] <= 32 and net.dims[1] % 128 == 0 and rows >= TC0_MIN_ROWS:
                n += 2                           # first layer on tensor cores: pad/split x and W0
    return n + 1 + 1 + (1 if clip else 0)      # reduce, adam, sum of squares


def run_ours(args):
    import torch
    import torch.distributed as dist
    from spo_mojo_b200 import ffi
    from spo_mojo_b200.learner import Comm, HostFeed, Learner, PackedHostBatch

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    wl = WORKLOADS[args.workload]
    if args.rows:
        import dataclasses
        wl = dataclasses.replace(wl, batch=args.rows, name=wl.name + f"@{args.rows}rows")
    B = wl.batch
    assert B % world == 0, "global batch must split evenly"
    rows = B // world
    params = init_params(wl, seed=0)
    batch_np = make_batch(wl, rows, seed=100 + rank)
    # the host batch: every field a view of one pinned buffer (one upload per step)
    host = PackedHostBatch.of(batch_np)
    batch = {k: v.to(dev) for k, v in host.items()}
    L = Learner.for_workload(wl, max_rows=rows, device=local, engine=args.engine)
    L.load(actor=params.get("actor"), critic=params.get("critic"), log_alpha=wl.log_alpha)
    comm = None
    if world > 1:
        obj = [Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = Comm(obj[0], world, rank)
    stream = torch.cuda.Stream(dev)
    scale = 1.0 / B

    def eager_step(b):
        if comm is None:             # one GPU: the public step (one launch for small batches)
            L.step(b, stream=stream)
            return
        L.backward(b, grad_scale=scale, stream=stream)
        comm.allreduce_(L.grads, stream=stream)
        L.apply(stream=stream)

    if args.graph and world > 1:
        raise SystemExit("--graph runs on one GPU")
    graphs = {}

    def capture(b):
        """One learner step on the batch tensors b recorded as a CUDA graph (the kernels
        neither allocate nor synchronise; the Adam step counter lives on the device)."""
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            eager_step(b)
        torch.cuda.synchronize(dev)
        return g

    def step(b):
        if not args.graph:
            eager_step(b)
            return
        key = id(b)
        if key not in graphs:
            graphs[key] = (capture(b), b)
        with torch.cuda.stream(stream):
            graphs[key][0].replay()

    # Clocks: rank 0 samples every GPU of the job with one nvidia-smi process, started
    # before the warm-up so that its start-up is not inside the timed region.
    def phys(i):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        return vis.split(",")[i] if vis else str(i)

    clocks = ClockSampler([phys(i) for i in range(world)]) if rank == 0 else None
    if clocks is not None:
        clocks.start()
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            eager_step(batch)  # first launches set kernel attributes, outside any capture
    if args.graph:
        step(batch)  # capture (the capture records, it does not run) and one replay, untimed
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()

    # A step whose inputs and activations fit in L2 is timed one step at a time, with a
    # write of twice the L2 size between steps (outside the timed events), so no step
    # reads what the previous one left in L2.
    in_bytes = sum(v.nbytes for v in batch_np.values())
    act_bytes = rows * sum(sum(n.dims[1:-1]) for n in (wl.actor, wl.critic) if n) * 4
    flush = in_bytes + act_bytes < L2_BYTES
    flush_buf = torch.empty(L2_BYTES // 2, dtype=torch.float32, device=dev) if flush else None

    def flushed_ms(one):
        """Average event-timed duration of one(i) over the steps, L2 flushed before each."""
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(stream):
            for i, (a, b) in enumerate(evs):
                flush_buf.fill_(float(i))
                a.record(stream)
                one(i)
                b.record(stream)
        evs[-1][1].synchronize()
        return sum(a.elapsed_time(b) for a, b in evs) / args.steps

    if clocks is not None:
        clocks.mark()
    launch_floor_us = None
    if flush:
        ms = flushed_ms(lambda i: step(batch))
    else:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        t0.record(stream)
        for _ in range(args.steps):
            step(batch)
        t1.record(stream)
        t1.synchronize()
        ms = t0.elapsed_time(t1) / args.steps
    clk = clocks.stop() if clocks is not None else None
    if flush:
        # the same timing applied to a graph of one one-element fill: what the launch, the
        # event records and the flush's aftermath cost a step that does no work
        tiny = torch.zeros(1, device=dev)
        torch.cuda.synchronize(dev)
        g_tiny = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_tiny, stream=stream):
            tiny.fill_(1.0)
        torch.cuda.synchronize(dev)
        launch_floor_us = 1e3 * flushed_ms(lambda i: g_tiny.replay())
        del g_tiny
    ms_max, ms_ranks = ms, [ms]
    if world > 1:
        tm = torch.tensor([ms], device=dev)
        every = [torch.zeros_like(tm) for _ in range(world)]
        dist.all_gather(every, tm)
        ms_ranks = [float(t.item()) for t in every]
        ms_max = max(ms_ranks)
    value = B / (ms_max / 1e3)
    stats = L.stats()

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        stats_host = torch.empty(ffi.NUM_STATS, dtype=torch.float32).pin_memory()
        h2d = int(host.flat.numel())  # the packed buffer, field padding included
        d2h = stats_host.numel() * 4
        if world > 1:
            dist.barrier()
        feed = HostFeed(host, dev, stream)
        if args.graph:
            for buf in feed.bufs:  # one graph per feed buffer, captured before the timed region
                graphs[id(buf)] = (capture(buf), buf)
        torch.cuda.synchronize(dev)
        w0 = time.perf_counter()
        if flush:
            # one step at a time: upload on the step's stream, the step, the read-back
            dbuf = feed.bufs[0]

            def e2e_step(i):
                feed.copy_into(0, host)
                step(dbuf)
                stats_host.copy_(L.stats_tensor(), non_blocking=True)

            ems = flushed_ms(e2e_step)
        else:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            feed.copy.wait_stream(stream)  # every upload starts inside the timed region
            with torch.cuda.stream(stream):
                j = feed.upload(host)
                for i in range(args.steps):
                    b = feed.take(j)
                    nxt = feed.upload(host) if i + 1 < args.steps else None  # overlaps step i
                    step(b)
                    feed.release(j)
                    stats_host.copy_(L.stats_tensor(), non_blocking=True)
                    j = nxt
            e1.record(stream)
            e1.synchronize()
            ems = e0.elapsed_time(e1) / args.steps
        torch.cuda.synchronize(dev)
        wall = (time.perf_counter() - w0) * 1e3 / args.steps
        if world > 1:
            tm = torch.tensor([ems], device=dev)
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
            ems = float(tm.item())
        e2e = {"value": B / (ems / 1e3), "unit": "samples/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": ems, "wall_ms_per_step": wall,
               "loss_read": float(stats_host[0])}

    # ---- the step's one collective alone: the all-reduce of the flat gradient buffer,
    # CUDA events on the learner's stream, averaged over 10 calls, max over ranks
    allreduce_ms = None
    if comm is not None:
        dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            comm.allreduce_(L.grads, stream=stream)
            a0.record(stream)
            for _ in range(10):
                comm.allreduce_(L.grads, stream=stream)
            a1.record(stream)
        a1.synchronize()
        tm = torch.tensor([a0.elapsed_time(a1) / 10], device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        allreduce_ms = float(tm.item())

    # ---- roofline of the dominant kernel: the hidden x hidden GEMM (forward shape)
    roof = None
    net = wl.actor or wl.critic
    H = net.dims[1]
    if rank == 0:
        roof = roofline_hidden_gemm(args, rows, H, dev, stream, engine=args.engine)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sps, srows, n, per = cpu_measure(wl, seconds=args.cpu_seconds)
        cpu = {"value": sps, "unit": "samples/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{srows} rows of {wl.name} per step, median of {n} steps "
                         "(float32 numpy restatement, all threads)"}

    if comm is not None:
        comm.close()
    if rank == 0:
        clip = wl.max_grad_norm > 0 and math.isfinite(wl.max_grad_norm)
        line = {
            "metric": "learner samples/sec (fwd+bwd+loss+Adam)",
            "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": wl.describe(), "global_batch": B, "rows_per_rank": rows,
                       "parallelism": f"dp{world}",
                       "launch": "CUDA graph per step" if args.graph else "stream launches",
                       "l2": ("working set per step < L2 (inputs %.2f MB, activations %.2f MB): "
                              "each step timed alone, a %d MB write between steps flushes L2"
                              % (in_bytes / 1e6, act_bytes / 1e6, 2 * L2_BYTES // 2**20)) if flush else
                             ("working set per step > L2 (inputs %.0f MB, activations %.1f GB); no flush"
                              % (in_bytes / 1e6, act_bytes / 1e9))},
            "e2e": e2e, "roofline": roof, "cpu_baseline": cpu, "clocks": clk,
            "ms_per_rank": ms_ranks,
            "launch_floor_us": launch_floor_us,
            "allreduce_ms": allreduce_ms,
            "allreduce_bytes": int(L.grads.numel() * 4) if world > 1 else 0,
            # the whole step's arithmetic (forward, dW, dX: 2 flop per multiply-add, fp32
            # products) over its measured time
            "step_tflops_fp32": wl.flops_per_sample() * B / (ms_max / 1e3) / 1e12,
            "gpu_launches": count_launches(wl, clip, args.engine, rows, world) * args.steps,
            "engine": args.engine,
            "stats": stats,
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_peaks():
    """The compute peaks the learner's two arithmetic paths run against (spo_measure_peaks),
    next to the driver-measured HBM and bf16 figures."""
    import ctypes
    import torch
    from spo_mojo_b200 import ffi
    torch.cuda.set_device(0)
    tf32, fp32 = ctypes.c_double(), ctypes.c_double()
    rows = []
    clocks = ClockSampler([0])
    clocks.start()
    for _ in range(3):
        ffi.call("spo_measure_peaks", torch.cuda.current_stream().cuda_stream, ctypes.byref(tf32), ctypes.byref(fp32))
        rows.append((tf32.value, fp32.value))
    clk = clocks.stop()
    pk, kind = peaks()
    print(json.dumps({"peaks": {
        "tf32_tcgen05_tflops": max(r[0] for r in rows) / 1e12,
        "fp32_ffma2_tflops": max(r[1] for r in rows) / 1e12,
        "three_tf32_fp32_equivalent_tflops": max(r[0] for r in rows) / 3e12,
        "hbm_gbs": pk.get("hbm_gbs"), "bf16_tflops": pk.get("bf16_tflops"),
        "bf16_tflops_sustained": pk.get("bf16_tflops_sustained"), "peaks_source": kind,
        "clocks": clk}}))
    return 0


def main():
    args = parse()
    if args.peaks:
        return run_peaks()
    if args.roofline_only:
        import torch
        wl = WORKLOADS[args.workload]
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        stream = torch.cuda.Stream(dev)
        H = (wl.actor or wl.critic).dims[1]
        print(json.dumps(roofline_hidden_gemm(args, args.roofline_only, H, dev, stream, engine=args.engine,
                                              reps=2)))
        return 0
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
