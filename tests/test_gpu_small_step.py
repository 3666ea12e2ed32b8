"""The one-launch learner step of small batches (small_step.cu) against the multi-launch
path of the same library and against the float64 oracle: gradients within rel 1e-5 of max
of each other (both fp32, different summation orders), losses rel 1e-5, post-Adam
parameters rel 1e-4 / abs 1e-6 where the update is determined (as in test_gpu_learner),
three consecutive steps, the backward-only form used by data parallelism, board-cell
inputs, a biting global-norm clip, 1-3 hidden layers, both networks and each alone."""

import numpy as np
import pytest
import torch

from oracle import spo_oracle as O
from spo_mojo_b200.workloads import WORKLOADS, NetSpec, Workload, init_params, make_batch, cells_of

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def dev(batch):
    return {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in batch.items()}


def rel_of_max(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.max(np.abs(got - want))) / max(float(np.max(np.abs(want))), 1e-30)


def learner(wl, rows, small, **kw):
    from spo_mojo_b200.learner import Learner
    L = Learner.for_workload(wl, max_rows=rows, **kw)
    L.set_small_rows(rows if small else 0)
    params = init_params(wl, seed=0)
    L.load(actor=params.get("actor"), critic=params.get("critic"), log_alpha=wl.log_alpha)
    return L, params


WLS = {
    "c0": WORKLOADS["c0"],
    "c1": WORKLOADS["c1"],
    "a1": Workload("a1", actor=NetSpec((27, 64, 9)), batch=300),
    "ac3": Workload("ac3", actor=NetSpec((27, 96, 160, 64, 9)), critic=NetSpec((27, 96, 160, 64, 1)),
                    batch=1000),
    "clip": Workload("clip", actor=NetSpec((27, 128, 128, 9)), critic=NetSpec((27, 128, 128, 1)),
                     batch=512, max_grad_norm=0.05),
}


@pytest.mark.parametrize("name,rows", [("c0", 256), ("c1", 4096), ("a1", 300), ("ac3", 1000), ("clip", 512),
                                       ("c0", 1), ("c0", 37), ("c1", 8192)])
def test_small_step_matches_the_multi_launch_step(name, rows):
    wl = WLS[name]
    batch = dev(make_batch(wl, rows, seed=5))
    out = []
    for small in (True, False):
        L, _ = learner(wl, rows, small)
        L.backward(batch)                  # gradients at the initial parameters
        g = L.grads.clone()
        s = L.stats()
        L.apply()
        for _ in range(2):
            L.step(batch)
        torch.cuda.synchronize()
        assert L.device_status() == 0
        out.append((g, s, L.params.clone(), int(L.step_counter.item()), L))
    (g1, s1, p1, t1, L1), (g0, s0, p0, t0, L0) = out
    assert t1 == t0 == 3
    for which in ("actor", "critic"):
        if getattr(wl, which) is None:
            continue
        for a, b in zip(L1.tensors(which, g1), L0.tensors(which, g0)):
            for x, y in zip(a, b):
                assert rel_of_max(x.cpu().numpy(), y.cpu().numpy()) <= 1e-5
        for a, b in zip(L1.tensors(which, p1), L0.tensors(which, p0)):
            for x, y in zip(a, b):
                # three Adam steps on gradients that agree to 1e-5 of max: elements whose
                # gradient is within that of zero may move in opposite directions (lr a step)
                x, y = x.cpu().numpy(), y.cpu().numpy()
                d = np.abs(x - y)
                assert np.mean(d > 1e-6 + 1e-4 * np.abs(y)) <= 0.03
                assert np.max(d) <= 6 * wl.lr + 1e-6
    for k in s0:
        assert abs(s1[k] - s0[k]) <= 1e-5 * max(abs(s0[k]), 1e-3), k


@pytest.mark.parametrize("name,rows", [("c0", 256), ("ac3", 1000)])
def test_small_step_matches_oracle(name, rows):
    wl = WLS[name]
    batch = make_batch(wl, rows, seed=9)
    L, params = learner(wl, rows, True)
    L.backward(dev(batch))
    torch.cuda.synchronize()
    st = L.stats()
    x = batch["obs"]
    for which in ("actor", "critic"):
        if which not in params:
            continue
        acts, z = O.mlp_forward(params[which], x)
        if which == "actor":
            lo = O.actor_loss(z, batch["mask"], batch["q"], batch["logits_old"], wl.log_alpha, wl.kl_eps, 1.0 / rows)
            assert abs(st["actor_loss"] - lo["loss"]) <= 1e-5 * abs(lo["loss"])
            dout = lo["dz"]
        else:
            lo = O.value_loss(z, batch["target"], 1.0 / rows)
            assert abs(st["critic_loss"] - lo["loss"]) <= 1e-5 * abs(lo["loss"])
            dout = lo["dv"]
        ours = [a.cpu().numpy() for a in L.activations(which, rows)]
        for a_g, a_o in zip(ours, acts):
            assert rel_of_max(a_g, a_o) <= 1e-5
        og = O.mlp_backward(params[which], x, acts, dout, masks=[a > 0 for a in ours])
        for (gw, gb), (ow, ob) in zip(L.tensors(which, L.grads), og):
            assert rel_of_max(gw.cpu().numpy(), ow) <= 1e-4
            assert rel_of_max(gb.cpu().numpy(), ob) <= 1e-4


def test_small_step_from_board_cells():
    wl = WLS["c0"]
    rows = 256
    batch = make_batch(wl, rows, seed=3)
    cells = {"cells": cells_of(batch["obs"]), "q": batch["q"], "logits_old": batch["logits_old"]}
    L1, _ = learner(wl, rows, True)
    L1.step(dev(cells))
    L0, _ = learner(wl, rows, True)
    L0.step(dev(batch))
    torch.cuda.synchronize()
    assert torch.equal(L1.grads, L0.grads) and torch.equal(L1.params, L0.params)


def test_small_backward_then_apply_equals_the_small_step():
    """The data-parallel form: backward alone (one launch), then apply (Adam kernel)."""
    wl = WLS["ac3"]
    rows = 1000
    batch = dev(make_batch(wl, rows, seed=4))
    L1, _ = learner(wl, rows, True)
    L1.backward(batch)
    L1.apply()
    L0, _ = learner(wl, rows, True)
    L0.step(batch)
    torch.cuda.synchronize()
    assert torch.equal(L1.grads, L0.grads)
    assert torch.allclose(L1.params, L0.params, rtol=0, atol=1e-7)


def test_small_rows_are_refused_for_wide_networks():
    from spo_mojo_b200 import ffi
    wl = WORKLOADS["c3"]
    from spo_mojo_b200.learner import Learner
    L = Learner.for_workload(wl, max_rows=64)
    with pytest.raises(ffi.SpoError, match="one-launch step"):
        L.set_small_rows(64)
    L.set_small_rows(0)


def test_bounded_barrier_wait_runs_out_and_the_next_step_is_exact():
    """The one-launch step's bounded grid-barrier waits, made to run out without a fault:
    the first CTA withholds its arrival at the first barrier and every wait is limited to
    2 ms (spo_learner_step_withheld). The launch must end by itself with a nonzero code in
    the learner's error word and change no parameter, moment or step counter; the next
    normal step must then match a fresh learner's step exactly (barrier words reset)."""
    import ctypes
    import time
    from spo_mojo_b200 import ffi
    wl = WLS["c0"]
    rows = 256
    batch = dev(make_batch(wl, rows, seed=5))
    L, _ = learner(wl, rows, True)
    assert L.device_status() == 0
    p0, m0, v0 = L.params.clone(), L.adam_m.clone(), L.adam_v.clone()
    b = L._batch(batch)
    torch.cuda.synchronize()
    t0 = time.time()
    ffi.call("spo_learner_step_withheld", L._h, None, ctypes.byref(b), ctypes.byref(L._state), 2000)
    torch.cuda.synchronize()
    assert time.time() - t0 < 10.0
    assert L.device_status() == 16          # a grid-barrier wait ran out
    assert torch.equal(L.params, p0) and torch.equal(L.adam_m, m0) and torch.equal(L.adam_v, v0)
    assert L.report_dict()["step"] == 0 and int(L.step_counter.item()) == 0
    with pytest.raises(ffi.SpoError, match="one-launch step"):
        big = dev(make_batch(wl, rows, seed=5))
        L.set_small_rows(128)
        ffi.call("spo_learner_step_withheld", L._h, None, ctypes.byref(L._batch(big)), ctypes.byref(L._state), 2000)
    L.set_small_rows(rows)
    L.step(batch)
    R, _ = learner(wl, rows, True)
    R.step(batch)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    assert torch.equal(L.params, R.params) and torch.equal(L.grads, R.grads)
