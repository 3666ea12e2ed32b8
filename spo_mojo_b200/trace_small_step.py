"""Phase trace of the one-launch small-batch learner step (small_step.cu).

The trace build of the library (`python -m spo_mojo_b200.build --trace`, which compiles
the kernel's phase marks in: thread 0 of every CTA records %globaltimer at each phase
boundary, and clock64 at the first and last mark) is loaded in place of the product
library; a workload's learner steps are run back to back and the marks of the last step
are printed as one JSON line per workload: per mark, the earliest / median / latest CTA,
in microseconds from the earliest CTA's start, and the SM clock over the kernel.

    python -m spo_mojo_b200.trace_small_step c0 c1 [--steps 300] [--flush]

--flush writes a 256 MB buffer (twice the L2) before every step, so that the traced step
starts with the weights, moments and partials out of L2, as the bench's steps do; the
back-to-back time is then not measured.

Marks: 0 start, 13 weight copies issued and the first block's input rows loaded, 1 the
block's loss inputs in shared memory, 2 forward done (each layer waits for its own
weights first), 3 loss done, 9 + l layer l's backward done, 12 layer 1's dW done (a
barrier is added there in the trace build), 4 last row block done, 5 rows phase done, 6
after the grid barrier, 7 reduction and Adam done, 8 exit.
"""

import argparse
import ctypes
import json
import os

import numpy as np

MARKS = 16


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("workloads", nargs="+")
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--flush", action="store_true", help="evict L2 before every step")
    args = ap.parse_args()

    from . import build, ffi
    if not os.path.exists(build.TRACE_LIB):
        build.build(trace=True)
    ffi.LIB_PATH = build.TRACE_LIB  # before the first call loads a library
    import torch
    from .learner import Learner
    from .workloads import WORKLOADS, init_params, make_batch

    lib = ffi.lib()
    read = lib.spo_small_trace_read
    read.restype = ctypes.c_int
    read.argtypes = [ctypes.c_void_p, ctypes.c_int]
    for name in args.workloads:
        wl = WORKLOADS[name]
        rows = wl.batch
        L = Learner.for_workload(wl, max_rows=rows)
        p = init_params(wl, seed=0)
        L.load(actor=p.get("actor"), critic=p.get("critic"), log_alpha=wl.log_alpha)
        b = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in make_batch(wl, rows, seed=1).items()}
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        scratch = torch.empty(64 << 20, dtype=torch.float32, device="cuda") if args.flush else None
        for i in range(args.steps):
            if i == args.steps // 2:
                s0.record()
            if scratch is not None:
                scratch.fill_(float(i))
            L.step(b)
        s1.record()
        torch.cuda.synchronize()
        # back-to-back steps (no L2 flush between them), CUDA events: kernel + launch gaps
        back_to_back_us = None if args.flush else s0.elapsed_time(s1) * 1e3 / (args.steps - args.steps // 2)
        buf = (ctypes.c_ulonglong * (1024 * MARKS))()
        if read(buf, 1024 * MARKS) != 0:
            raise RuntimeError("spo_small_trace_read failed")
        grid = torch.cuda.get_device_properties(0).multi_processor_count
        a = np.frombuffer(buf, dtype=np.uint64).reshape(1024, MARKS)[:grid].astype(np.int64)
        t0 = a[:, 0].min()
        rel = (a - t0) / 1000.0
        rel[a == 0] = np.nan
        clk, ns = a[:, 15] - a[:, 14], a[:, 8] - a[:, 0]
        out = {"workload": name, "rows": rows, "steps": args.steps,
               "sm_mhz": float(np.median(clk[ns > 0] * 1000.0 / ns[ns > 0])),
               "l2_flushed": bool(args.flush),
               "back_to_back_us_per_step": None if back_to_back_us is None else round(back_to_back_us, 2)}
        for m in range(14):
            col = rel[:, m]
            if np.any(~np.isnan(col)):
                out[str(m)] = [round(float(np.nanmin(col)), 3), round(float(np.nanmedian(col)), 3),
                               round(float(np.nanmax(col)), 3)]
        print(json.dumps(out))


if __name__ == "__main__":
    main()
