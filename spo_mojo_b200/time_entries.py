"""Launch times of the standalone C-ABI entry points around the learner step.

Times, through libspo_cuda on cuda:0, the entries a caller that runs its own networks uses
(the reference's step-by-step composition), on seeded synthetic tic-tac-toe-shaped rows:

* actor_loss   spo_actor_loss_fwd_bwd on logits [rows x 9] with mask, q, pi_old logits and
               log_alpha (the eq-11 loss, the alpha*KL term, dz, statistics, the dual
               gradient); algorithmic bytes: logits, mask, q, pi_old logits in, dz out
* softmax      spo_softmax_rows on [rows x 9] (about 30 % of the logits masked to -inf);
               bytes: in and out
* actor_head   spo_actor_head_fwd_bwd: the fused last layer, loss and last-layer backward
               from activations [rows x 512] (fp32 dX out); bytes: activations, mask, q,
               pi_old logits in, dX out

Each entry: 3 warm-up launches, then the best of 3 runs of 20 back-to-back launches timed
with CUDA events on the launching stream. One JSON line per entry.

    python -m spo_mojo_b200.time_entries [--rows 1048576] [entries ...]
"""

import argparse
import json

import torch

from . import ffi

A = 9
H = 512


def _inputs(rows, g):
    mask = (torch.rand(rows, A, device="cuda", generator=g) < 0.6).float()
    mask[:, 0] = 1.0
    q = torch.rand(rows, A, device="cuda", generator=g) * mask
    q = q / q.sum(1, keepdim=True)
    zold = torch.randn(rows, A, device="cuda", generator=g)
    return mask, q, zold


def _time(run, stream):
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(20):
            run()
        e1.record(stream)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1) / 20)
    return best


def actor_loss(rows, s, g):
    z = torch.randn(rows, A, device="cuda", generator=g)
    mask, q, zold = _inputs(rows, g)
    la = torch.zeros(1, device="cuda")
    dz = torch.empty(rows, A, device="cuda")
    stats = torch.empty(ffi.NUM_STATS, device="cuda")
    dla = torch.empty(1, device="cuda")
    ws = torch.empty(int(ffi.lib().spo_loss_workspace_size()), dtype=torch.uint8, device="cuda")

    def run():
        ffi.call("spo_actor_loss_fwd_bwd", s.cuda_stream, z.data_ptr(), mask.data_ptr(), q.data_ptr(),
                 zold.data_ptr(), la.data_ptr(), 0.01, rows, A, 1.0 / rows, dz.data_ptr(), stats.data_ptr(),
                 dla.data_ptr(), ws.data_ptr(), ws.numel())
    return run, rows * A * 4 * 5


def softmax(rows, s, g):
    z = torch.randn(rows, A, device="cuda", generator=g)
    z[torch.rand(rows, A, device="cuda", generator=g) < 0.3] = float("-inf")
    z[:, 0] = torch.randn(rows, device="cuda", generator=g)
    out = torch.empty(rows, A, device="cuda")

    def run():
        ffi.call("spo_softmax_rows", s.cuda_stream, out.data_ptr(), z.data_ptr(), rows, A)
    return run, rows * A * 4 * 2


def actor_head(rows, s, g):
    act = torch.randn(rows, H, device="cuda", generator=g).relu_()
    w = torch.randn(H, A, device="cuda", generator=g) / H ** 0.5
    b = torch.randn(A, device="cuda", generator=g) * 0.1
    mask, q, zold = _inputs(rows, g)
    la = torch.zeros(1, device="cuda")
    dact = torch.empty(rows, H, device="cuda")
    dw, db, dbact = torch.empty(H, A, device="cuda"), torch.empty(A, device="cuda"), torch.empty(H, device="cuda")
    stats = torch.empty(ffi.NUM_STATS, device="cuda")
    ws = torch.empty(int(ffi.lib().spo_head_workspace_size(rows, H, A)), dtype=torch.uint8, device="cuda")

    def run():
        ffi.call("spo_actor_head_fwd_bwd", s.cuda_stream, act.data_ptr(), w.data_ptr(), b.data_ptr(), rows, H, A,
                 mask.data_ptr(), q.data_ptr(), zold.data_ptr(), la.data_ptr(), 1.0 / rows, None, None, None,
                 dact.data_ptr(), dw.data_ptr(), db.data_ptr(), dbact.data_ptr(), stats.data_ptr(), ws.data_ptr(),
                 ws.numel())
    return run, rows * (2 * H + 3 * A) * 4


ENTRIES = {"actor_loss": actor_loss, "softmax": softmax, "actor_head": actor_head}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("entries", nargs="*", default=list(ENTRIES))
    ap.add_argument("--rows", type=int, default=1048576)
    args = ap.parse_args()
    assert torch.cuda.is_available(), "needs a CUDA device"
    s = torch.cuda.current_stream()
    for name in args.entries:
        g = torch.Generator(device="cuda").manual_seed(0)
        run, nbytes = ENTRIES[name](args.rows, s, g)
        ms = _time(run, s)
        print(json.dumps({"entry": name, "rows": args.rows, "ms_per_launch": round(ms, 4),
                          "algorithmic_bytes": nbytes, "gb_per_s": round(nbytes / ms / 1e6, 1)}))
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
