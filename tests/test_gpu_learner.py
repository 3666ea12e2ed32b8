"""The fused learner step (libspo_cuda through spo_learner_*) against the float64
CPU oracle, on seeded synthetic inputs of the five learner workloads.

Tolerances (the parity bar of this path): losses rel 1e-5; gradients rel 1e-4 of
max |want| per tensor (the reference's gradient metric,
tests/test_actor_backward.mojo:59-71); post-Adam parameters rel 1e-4 / abs 1e-6.
"""

import json
import math
import os

import numpy as np
import pytest
import torch

from oracle import spo_oracle as O
from spo_mojo_b200.workloads import WORKLOADS, make_batch, init_params, Workload, NetSpec

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-5
FWD_RTOL = 1e-5
GRAD_RTOL = 1e-4
PARAM_RTOL, PARAM_ATOL = 1e-4, 1e-6


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def to_dev(batch):
    return {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in batch.items()}


def oracle_run(wl, params, batch, steps=1, max_norm=None):
    hp = dict(lr_actor=wl.lr, lr_critic=wl.lr, b1=wl.beta1, b2=wl.beta2, eps=wl.adam_eps,
              max_norm=wl.max_grad_norm if max_norm is None else max_norm,
              kl_eps=wl.kl_eps, dual=wl.dual)
    nets = {}
    for which in ("actor", "critic"):
        if which in params:
            p = [(w.astype(np.float64), b.astype(np.float64)) for w, b in params[which]]
            nets[which] = {"params": p, "m": [(np.zeros_like(w), np.zeros_like(b)) for w, b in p],
                           "v": [(np.zeros_like(w), np.zeros_like(b)) for w, b in p]}
    la, am, av = wl.log_alpha, 0.0, 0.0
    first = None
    for step in range(1, steps + 1):
        hp.update(step=step, alpha_m=am, alpha_v=av)
        b = dict(batch)
        if not wl.dual:
            b["logits_old"] = None
        out = O.learner_step(b, actor=nets.get("actor"), critic=nets.get("critic"),
                             log_alpha=la if wl.dual else None, hp=hp)
        if first is None:
            first = out
        for which in nets:
            nets[which]["params"] = out[which]["new_params"]
            nets[which]["m"] = out[which]["new_m"]
            nets[which]["v"] = out[which]["new_v"]
        if "log_alpha" in out:
            la, am, av = out["log_alpha"]["value"], out["log_alpha"]["m"], out["log_alpha"]["v"]
    return first, nets, la


def run_learner(wl, params, batch_dev, steps=1, max_norm=None, rows=None, engine="tensor"):
    from spo_mojo_b200.learner import Learner
    kw = {} if max_norm is None else {"max_grad_norm": max_norm}
    L = Learner.for_workload(wl, max_rows=rows or batch_dev["obs"].shape[0], engine=engine, **kw)
    L.load(actor=params.get("actor"), critic=params.get("critic"), log_alpha=wl.log_alpha)
    grads0 = stats0 = rep0 = None
    for i in range(steps):
        L.step(batch_dev)
        if i == 0:
            grads0 = L.grads.clone()
            stats0 = L.stats()
            rep0 = L.report_dict()
    torch.cuda.synchronize()
    assert L.device_status() == 0, "a bounded wait of a tensor-core kernel gave up"
    return L, grads0, stats0, rep0


def rel_of_max(got, want):
    want = np.asarray(want, np.float64)
    return float(np.max(np.abs(np.asarray(got, np.float64) - want))) / max(float(np.max(np.abs(want))), 1e-30)


def check_against_oracle(wl, L, grads0, stats0, rep0, ora, nets, la, params, batch):
    """Losses vs the oracle; hidden activations within FWD_RTOL of max; ReLU decisions
    that differ from float64 (activations within fp32 rounding of zero) at most
    max(2, 1e-5 of the activations); gradients vs the oracle's backward taken through
    this library's ReLU decisions (the same branch of the piecewise-linear network);
    post-Adam parameters as check_adam describes."""
    # losses
    if wl.actor is not None:
        al = ora["actor"]["loss"]
        assert abs(stats0["actor_loss"] - al["loss"]) <= LOSS_RTOL * abs(al["loss"])
        assert abs(stats0["ce"] - al["ce_mean"]) <= LOSS_RTOL * abs(al["ce_mean"])
        assert abs(stats0["entropy"] - al["entropy_mean"]) <= LOSS_RTOL * abs(al["entropy_mean"]) + 1e-7
        assert abs(stats0["kl_q"] - al["kl_q_mean"]) <= LOSS_RTOL * abs(al["ce_mean"])
        assert abs(stats0["kl_old"] - al["kl_old_mean"]) <= LOSS_RTOL * abs(al["loss"])
    if wl.critic is not None:
        cl = ora["critic"]["loss"]
        assert abs(stats0["critic_loss"] - cl) <= LOSS_RTOL * abs(cl)
    # forward activations, ReLU decisions, then gradients per tensor
    x = batch["obs"]
    rows = x.shape[0]
    for which in ("actor", "critic"):
        if which not in ora:
            continue
        acts_o, out_o = O.mlp_forward(params[which], x)
        ours = [a.cpu().numpy() for a in L.activations(which, rows)]
        flips = 0
        for i, (a_g, a_o) in enumerate(zip(ours, acts_o)):
            assert rel_of_max(a_g, a_o) <= FWD_RTOL, f"{which} activation {i + 1}"
            flips += int(((a_g > 0) != (a_o > 0)).sum())
        assert flips <= max(2, 1e-5 * sum(a.size for a in acts_o)), f"{which}: {flips} ReLU flips"
        if which == "actor":
            dout = ora["actor"]["loss"]["dz"]
        else:
            dout = O.value_loss(out_o, batch["target"], 1.0 / rows)["dv"]
        og = O.mlp_backward(params[which], x, acts_o, dout, masks=[a > 0 for a in ours])
        for i, ((gw, gb), (ow, ob)) in enumerate(zip(L.tensors(which, grads0), og)):
            assert rel_of_max(gw.cpu().numpy(), ow) <= GRAD_RTOL, f"{which} dW{i + 1}"
            assert rel_of_max(gb.cpu().numpy(), ob) <= GRAD_RTOL, f"{which} db{i + 1}"
        clip_o = O.global_clip_scale(O.global_norm([t for pair in og for t in pair]), wl.max_grad_norm)
        want = [(O.adam_step(w, gw_, np.zeros_like(gw_), np.zeros_like(gw_), 1, wl.lr, wl.beta1,
                             wl.beta2, wl.adam_eps, clip_o)[0],
                 O.adam_step(b, gb_, np.zeros_like(gb_), np.zeros_like(gb_), 1, wl.lr, wl.beta1,
                             wl.beta2, wl.adam_eps, clip_o)[0])
                for (w, b), (gw_, gb_) in zip(params[which], og)]
        excluded = {}
        check_adam(wl, L, which, grads0, og, want, params[which], rep0[f"clip_{which}"], excluded)
        n_out = sum(e for e, _ in excluded.values())
        n_all = sum(t for _, t in excluded.values())
        _record_excluded(wl, rows, which, excluded)
        # the undetermined updates are the gradients within the fp32 error of zero: few
        assert n_out <= 0.05 * n_all, (which, excluded)
    if wl.actor is not None and wl.dual:
        want = ora["log_alpha"]["grad"]
        assert abs(rep0["dlog_alpha"] - want) <= 1e-4 * abs(want) + 1e-7
        assert abs(float(L.log_alpha) - la) <= PARAM_RTOL * abs(la) + PARAM_ATOL


def _record_excluded(wl, rows, which, excluded):
    """Appends the per-tensor counts of post-Adam elements checked only against the 2 lr
    bound to the JSON-lines file named by SPO_PARITY_REPORT (when set)."""
    path = os.environ.get("SPO_PARITY_REPORT")
    if not path:
        return
    with open(path, "a") as f:
        f.write(json.dumps({"workload": wl.name, "rows": rows, "net": which,
                            "excluded": {k: list(v) for k, v in excluded.items()}}) + "\n")


def adam_determined(g_or, g_gpu, lr, eps):
    """Elements whose first Adam step lr * g / (|g| + eps) the fp32 gradient determines to
    within PARAM_ATOL / 2: a gradient that is exactly zero in both (a unit no row
    activates: the parameter does not move), or one whose magnitude is at least ten times
    the tensor's largest gradient error d (so the sign is right) and large enough that the
    step's sensitivity lr * eps * d / (|g| - d)^2 stays below PARAM_ATOL / 2."""
    d = float(np.max(np.abs(g_gpu - g_or))) if g_or.size else 0.0
    a = np.abs(g_or)
    both_zero = (g_or == 0) & (g_gpu == 0)
    big = (a >= 10 * d) & ((a - d) ** 2 * (0.5 * PARAM_ATOL) >= lr * eps * d)
    return both_zero | big


def check_adam(wl, L, which, grads_gpu, grads_ora, params_ora, p0, clip, report=None):
    """Post-Adam parameters, rel 1e-4 / abs 1e-6, on every element, checked two ways.

    Adam's first step moves a parameter by lr * g / (|g| + eps): for a gradient within the
    gradient error of zero its sign, hence the update, is not determined by the fp32 inputs
    at all. So (1) the update is checked exactly as the optimiser defines it, by applying
    the oracle's Adam (float64) to this library's own gradients, on every element; (2)
    against the full oracle on every element whose update the gradient determines
    (adam_determined), and on the others (reported in `report`: a few tenths of a percent
    of the elements, the gradients within the fp32 error of zero) to within the largest
    step Adam can take, 2 lr.
    """
    for i, ((pw, pb), (gw, gb), (ogw, ogb), (ow, ob), (w0, b0)) in enumerate(
            zip(L.tensors(which), L.tensors(which, grads_gpu), grads_ora, params_ora, p0)):
        for got, g_gpu, g_or, want, start, nm in ((pw, gw, ogw, ow, w0, "W"), (pb, gb, ogb, ob, b0, "b")):
            got = got.cpu().numpy()
            g_gpu = g_gpu.cpu().numpy().astype(np.float64)
            mine, _, _ = O.adam_step(start, g_gpu, np.zeros_like(g_gpu), np.zeros_like(g_gpu), 1,
                                     wl.lr, wl.beta1, wl.beta2, wl.adam_eps, clip)
            np.testing.assert_allclose(got, mine, rtol=PARAM_RTOL, atol=PARAM_ATOL,
                                       err_msg=f"{which} {nm}{i + 1}: Adam on our gradients")
            clear = adam_determined(np.asarray(g_or, np.float64) * clip, g_gpu * clip, wl.lr, wl.adam_eps)
            np.testing.assert_allclose(got[clear], want[clear], rtol=PARAM_RTOL, atol=PARAM_ATOL,
                                       err_msg=f"{which} {nm}{i + 1}: oracle Adam")
            assert np.all(np.abs(got[~clear] - want[~clear]) <= 2 * wl.lr * (1 + 1e-3) + PARAM_ATOL)
            if report is not None:
                report[f"{which} {nm}{i + 1}"] = (int((~clear).sum()), int(clear.size))


@pytest.mark.parametrize("engine", ["tensor", "cuda"])
@pytest.mark.parametrize("name,rows", [("c0", 256), ("c1", 4096), ("c2", 4096), ("c3", 2048), ("c4", 1024)])
def test_workload_step_matches_oracle(name, rows, engine):
    wl = WORKLOADS[name]
    params = init_params(wl, seed=0)
    batch = make_batch(wl, rows, seed=1)
    L, g0, s0, r0 = run_learner(wl, params, to_dev(batch), engine=engine)
    ora, nets, la = oracle_run(wl, params, batch)
    check_against_oracle(wl, L, g0, s0, r0, ora, nets, la, params, batch)


def test_c2_full_batch_matches_oracle():
    """c2 at its full 65,536 rows (the oracle still finishes in seconds)."""
    wl = WORKLOADS["c2"]
    params = init_params(wl, seed=0)
    batch = make_batch(wl, wl.batch, seed=2)
    L, g0, s0, r0 = run_learner(wl, params, to_dev(batch))
    ora, nets, la = oracle_run(wl, params, batch)
    check_against_oracle(wl, L, g0, s0, r0, ora, nets, la, params, batch)


@pytest.mark.parametrize("engine", ["tensor", "cuda"])
def test_three_steps_bias_correction(engine):
    """Three consecutive steps (Adam bias corrections 1/(1-b^t), t = 1, 2, 3, from the
    device step counter): each step's loss matches the float64 oracle run over the same
    three steps, and the parameters match the oracle's Adam applied step by step to this
    library's own gradients (moments carried across steps)."""
    from spo_mojo_b200.learner import Learner
    wl = WORKLOADS["c0"]
    params = init_params(wl, seed=3)
    batch = make_batch(wl, 256, seed=4)
    dev = to_dev(batch)
    L = Learner.for_workload(wl, max_rows=256, engine=engine)
    L.load(actor=params["actor"], log_alpha=wl.log_alpha)
    p = [(w.astype(np.float64), b.astype(np.float64)) for w, b in params["actor"]]
    m = [(np.zeros_like(w), np.zeros_like(b)) for w, b in p]
    v = [(np.zeros_like(w), np.zeros_like(b)) for w, b in p]
    la, am, av = wl.log_alpha, 0.0, 0.0
    hp = dict(lr_actor=wl.lr, lr_critic=wl.lr, b1=wl.beta1, b2=wl.beta2, eps=wl.adam_eps,
              max_norm=wl.max_grad_norm, kl_eps=wl.kl_eps, dual=True)
    full = {"params": [(w.astype(np.float64), b.astype(np.float64)) for w, b in params["actor"]],
            "m": [(np.zeros_like(a), np.zeros_like(b)) for a, b in p],
            "v": [(np.zeros_like(a), np.zeros_like(b)) for a, b in p]}
    fla, fam, fav = la, 0.0, 0.0
    for t in (1, 2, 3):
        L.backward(dev)
        L.apply()
        torch.cuda.synchronize()
        st = L.stats()
        hp.update(step=t, alpha_m=fam, alpha_v=fav)
        out = O.learner_step(batch, actor=full, log_alpha=fla, hp=hp)
        assert abs(st["actor_loss"] - out["actor"]["loss"]["loss"]) <= LOSS_RTOL * abs(out["actor"]["loss"]["loss"])
        full = {"params": out["actor"]["new_params"], "m": out["actor"]["new_m"], "v": out["actor"]["new_v"]}
        fla, fam, fav = out["log_alpha"]["value"], out["log_alpha"]["m"], out["log_alpha"]["v"]
        # the oracle's Adam on our gradients, moments carried
        g = [(gw.cpu().numpy().astype(np.float64), gb.cpu().numpy().astype(np.float64))
             for gw, gb in L.tensors("actor", L.grads)]
        for i in range(len(p)):
            pw, mw, vw = O.adam_step(p[i][0], g[i][0], m[i][0], v[i][0], t, wl.lr, wl.beta1, wl.beta2, wl.adam_eps)
            pb, mb, vb = O.adam_step(p[i][1], g[i][1], m[i][1], v[i][1], t, wl.lr, wl.beta1, wl.beta2, wl.adam_eps)
            p[i], m[i], v[i] = (pw, pb), (mw, mb), (vw, vb)
        gla = float(L.grads[L.layout.alpha_index])
        lap, am, av = O.adam_step(np.array([la]), np.array([gla]), np.array([am]), np.array([av]), t,
                                  wl.lr, wl.beta1, wl.beta2, wl.adam_eps)
        la, am, av = float(lap[0]), float(am[0]), float(av[0])
        for (pw, pb), (ow, ob) in zip(L.tensors("actor"), p):
            np.testing.assert_allclose(pw.cpu().numpy(), ow, rtol=PARAM_RTOL, atol=PARAM_ATOL)
            np.testing.assert_allclose(pb.cpu().numpy(), ob, rtol=PARAM_RTOL, atol=PARAM_ATOL)
        assert abs(float(L.log_alpha) - la) <= PARAM_RTOL * abs(la) + PARAM_ATOL
    assert int(L.step_counter.item()) == 3
    assert L.device_status() == 0


def test_global_norm_clip_bites():
    """max_grad_norm small enough that the reference's clip (networks/optim.mojo:133-142)
    scales both networks' updates."""
    wl = Workload("clip", actor=NetSpec((27, 64, 64, 9)), critic=NetSpec((27, 64, 64, 1)),
                  batch=512, max_grad_norm=1e-3)
    params = init_params(wl, seed=5)
    batch = make_batch(wl, 512, seed=6)
    L, g0, s0, r0 = run_learner(wl, params, to_dev(batch))
    ora, nets, la = oracle_run(wl, params, batch)
    assert r0["clip_actor"] < 1.0 and r0["clip_critic"] < 1.0
    assert abs(r0["norm_actor"] - ora["actor"]["norm"]) <= 1e-4 * ora["actor"]["norm"]
    assert abs(r0["norm_critic"] - ora["critic"]["norm"]) <= 1e-4 * ora["critic"]["norm"]
    check_against_oracle(wl, L, g0, s0, r0, ora, nets, la, params, batch)


@pytest.mark.parametrize("rows", [1, 3, 129, 1000])
def test_ragged_row_counts(rows):
    wl = WORKLOADS["c2"]
    params = init_params(wl, seed=7)
    batch = make_batch(wl, rows, seed=8)
    L, g0, s0, r0 = run_learner(wl, params, to_dev(batch), rows=4096)
    ora, nets, la = oracle_run(wl, params, batch)
    check_against_oracle(wl, L, g0, s0, r0, ora, nets, la, params, batch)


def test_degenerate_rows():
    """A fully masked row (a finished board: uniform pi, zero dz, no NaN —
    networks/actor.mojo:57-62) and q with zeros on legal cells (the q == 0 skip of
    networks/actor_loss.mojo:48-56)."""
    wl = WORKLOADS["c0"]
    params = init_params(wl, seed=9)
    batch = make_batch(wl, 64, seed=10)
    batch["mask"][0] = 0.0
    batch["q"][0] = 0.0
    batch["logits_old"][0] = O.NEG_INF
    legal = np.flatnonzero(batch["mask"][1])
    batch["q"][1] = 0.0
    batch["q"][1, legal[0]] = 1.0
    L, g0, s0, r0 = run_learner(wl, params, to_dev(batch))
    assert all(math.isfinite(v) for v in s0.values())
    assert torch.isfinite(g0).all()
    ora, nets, la = oracle_run(wl, params, batch)
    check_against_oracle(wl, L, g0, s0, r0, ora, nets, la, params, batch)
    logits, pi = L.forward("actor", to_dev(batch)["obs"], to_dev(batch)["mask"])
    assert torch.allclose(pi[0], torch.full((9,), 1.0 / 9, device="cuda"))


def test_zero_rows_leave_zero_gradients():
    wl = WORKLOADS["c0"]
    from spo_mojo_b200.learner import Learner
    L = Learner.for_workload(wl, max_rows=16)
    L.load(actor=init_params(wl)["actor"])
    L.grads.fill_(7.0)
    b = to_dev(make_batch(wl, 1, seed=0))
    b = {k: v[:0] for k, v in b.items()}
    L.backward(b, grad_scale=1.0)
    torch.cuda.synchronize()
    lay = L.layout
    assert torch.count_nonzero(L.grads[:lay.stats_offset + 8]) == 0


def test_rows_beyond_capacity_raise():
    from spo_mojo_b200 import ffi
    from spo_mojo_b200.learner import Learner
    wl = WORKLOADS["c0"]
    L = Learner.for_workload(wl, max_rows=8)
    with pytest.raises(ffi.SpoError) as e:
        L.backward(to_dev(make_batch(wl, 9, seed=0)))
    assert "max_rows" in str(e.value)


@pytest.mark.parametrize("engine", ["tensor", "cuda"])
def test_deterministic(engine):
    wl = WORKLOADS["c2"]
    params = init_params(wl, seed=0)
    batch = to_dev(make_batch(wl, 8192, seed=11))
    _, g1, _, _ = run_learner(wl, params, batch, engine=engine)
    _, g2, _, _ = run_learner(wl, params, batch, engine=engine)
    assert torch.equal(g1, g2)


@pytest.mark.parametrize("name,engine", [("c3", "tensor"), ("c3", "cuda"), ("c4", "tensor"), ("c4", "cuda")])
def test_full_batch_vs_float64(name, engine):
    """c3 at its full 1,048,576 rows (actor + critic 27-512x3-{9,1}) and c4 at its full
    262,144 rows (actor 27-1024x4-9, the deepest products: 32 k-blocks each) against a
    float64 restatement run on the GPU.

    Forward: every hidden activation within 1e-5 of max, losses within 1e-5 relative.
    ReLU decisions of activations within fp32 noise of zero can differ from float64
    (at most 1e-5 of the activations may); the backward is therefore compared with the
    float64 backward taken through this library's own ReLU decisions, at rel 1e-4 of max.
    """
    import fp64_reference as R
    from spo_mojo_b200.learner import Learner
    wl = WORKLOADS[name]
    B = wl.batch
    params = init_params(wl, seed=0)
    batch = to_dev(make_batch(wl, B, seed=13))
    L = Learner.for_workload(wl, max_rows=B, engine=engine)
    L.load(actor=params.get("actor"), critic=params.get("critic"), log_alpha=wl.log_alpha)
    L.backward(batch)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    st = L.stats()
    x = batch["obs"].double()
    for which in [w for w in ("actor", "critic") if w in params]:
        p64 = [(torch.from_numpy(w).cuda().double(), torch.from_numpy(b).cuda().double())
               for w, b in params[which]]
        acts, out = R.mlp_forward(p64, x)
        ours = L.activations(which, B)
        flips = 0
        for a64, a32 in zip(acts, ours):
            err = (a32.double() - a64).abs().max() / a64.abs().max()
            assert float(err) <= 1e-5
            flips += int(((a32 > 0) != (a64 > 0)).sum())
        assert flips <= 1e-5 * sum(a.numel() for a in acts)
        if which == "actor":
            lo = R.actor_loss(out, batch["mask"].double(), batch["q"].double(),
                              batch["logits_old"].double(), wl.log_alpha, 1.0 / B)
            assert abs(st["actor_loss"] - lo["loss"]) <= LOSS_RTOL * abs(lo["loss"])
            assert abs(st["kl_old"] - lo["kl_old"]) <= LOSS_RTOL * abs(lo["loss"])
            dout = lo["dz"]
        else:
            lo = R.value_loss(out, batch["target"].double(), 1.0 / B)
            assert abs(st["critic_loss"] - lo["loss"]) <= LOSS_RTOL * abs(lo["loss"])
            dout = lo["dv"]
        grads = R.mlp_backward(p64, x, acts, dout, masks=[a > 0 for a in ours])
        for i, ((gw, gb), (rw, rb)) in enumerate(zip(L.tensors(which, L.grads), grads)):
            assert rel_of_max(gw.cpu().numpy(), rw.cpu().numpy()) <= GRAD_RTOL, f"{which} dW{i + 1}"
            assert rel_of_max(gb.cpu().numpy(), rb.cpu().numpy()) <= GRAD_RTOL, f"{which} db{i + 1}"
        del acts, ours, grads


def test_c3_full_batch_additivity_and_forward():
    """c3 at its full 1,048,576 rows. The float64 oracle cannot run this size in
    seconds, so: (1) the gradient over the batch equals the sum of the gradients over
    its two halves with the same 1/B scale (the backward is linear in the per-row
    terms); (2) the forward of 2,000 sampled rows matches the oracle."""
    from spo_mojo_b200.learner import Learner
    wl = WORKLOADS["c3"]
    params = init_params(wl, seed=0)
    batch = to_dev(make_batch(wl, wl.batch, seed=12))
    B = wl.batch
    L = Learner.for_workload(wl, max_rows=B)
    L.load(actor=params["actor"], critic=params["critic"])
    L.backward(batch, grad_scale=1.0 / B)
    full = L.grads.clone()
    h = B // 2
    L.backward({k: v[:h] for k, v in batch.items()}, grad_scale=1.0 / B)
    part = L.grads.clone()
    L.backward({k: v[h:] for k, v in batch.items()}, grad_scale=1.0 / B)
    part += L.grads
    torch.cuda.synchronize()
    assert torch.isfinite(full).all()
    for which in ("actor", "critic"):
        for (fw, fb), (pw, pb) in zip(L.tensors(which, full), L.tensors(which, part)):
            assert rel_of_max(fw.cpu().numpy(), pw.cpu().numpy()) <= GRAD_RTOL
            assert rel_of_max(fb.cpu().numpy(), pb.cpu().numpy()) <= GRAD_RTOL
    idx = np.random.default_rng(0).choice(B, 2000, replace=False)
    obs = batch["obs"][torch.from_numpy(idx).cuda()].contiguous()
    mask = batch["mask"][torch.from_numpy(idx).cuda()].contiguous()
    logits, pi = L.forward("actor", obs, mask)
    _, z = O.mlp_forward(params["actor"], obs.cpu().numpy())
    zm = O.masked_logits(z, mask.cpu().numpy())
    np.testing.assert_allclose(pi.cpu().numpy(), O.softmax_rows(zm), atol=2e-5)
    v, _ = L.forward("critic", obs)
    _, vo = O.mlp_forward(params["critic"], obs.cpu().numpy())
    np.testing.assert_allclose(v.cpu().numpy(), vo, rtol=1e-4, atol=3e-5 * math.sqrt(512))
