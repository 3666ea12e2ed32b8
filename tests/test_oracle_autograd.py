"""A second, independent pin for the parts of the oracle no reference golden covers: the
alpha*KL(pi_old||pi) term, the log_alpha dual gradient, the 27-wide three-plane input,
more than two hidden layers, and Adam with eps = 1e-8.

The reference produces its goldens by automatic differentiation (JAX at highest matmul
precision, tests/golden/gen/gen_actor_backward.py). Here the same role is played by
PyTorch autograd in float64 over the loss written directly from its definition:

    actor:  mean_rows[ -sum_{q>0} q log pi + alpha * sum_{pi_old>0} pi_old (log pi_old - log pi) ],
            pi = softmax(logits masked with the most negative finite float32),
            alpha = softplus(log_alpha), a constant for the policy loss
    dual:   softplus(log_alpha) * (eps_kl - stopgrad(mean KL(pi_old || pi)))
    critic: mean_rows 0.5 (V - target)^2

and torch.optim.Adam for the update. The oracle's hand-derived backward and its Adam
must agree with both to float64 rounding. CPU only."""

import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle import spo_oracle as O  # noqa: E402
from spo_mojo_b200.workloads import Workload, NetSpec, init_params, make_batch  # noqa: E402

NEG = float(np.finfo(np.float32).min)
ROWS = 48
WL = Workload("autograd", actor=NetSpec((27, 64, 64, 64, 9)), critic=NetSpec((27, 64, 64, 64, 1)),
              batch=ROWS)
HP = dict(lr_actor=3e-4, lr_critic=3e-4, b1=0.9, b2=0.999, eps=1e-8, max_norm=float("inf"),
          kl_eps=0.01, dual=True)


def _mlp(params, x):
    h = x
    for i, (w, b) in enumerate(params):
        h = h @ w + b
        if i + 1 < len(params):
            h = torch.relu(h)
    return h


def _actor_loss(z, mask, q, z_old, alpha):
    zm = torch.where(mask > 0, z, torch.full_like(z, NEG))
    log_pi = torch.log_softmax(zm, dim=1)
    zo = torch.where(mask > 0, z_old, torch.full_like(z_old, NEG))
    log_pi_old = torch.log_softmax(zo, dim=1)
    pi_old = torch.exp(log_pi_old)
    ce = -torch.where(q > 0, q * log_pi, torch.zeros_like(q)).sum(1)
    kl = torch.where(pi_old > 0, pi_old * (log_pi_old - log_pi), torch.zeros_like(q)).sum(1)
    return (ce + alpha * kl).mean(), kl.mean()


def _tensors(params):
    return [(torch.tensor(w, dtype=torch.float64, requires_grad=True),
             torch.tensor(b, dtype=torch.float64, requires_grad=True)) for w, b in params]


@pytest.fixture(scope="module")
def setup():
    params = init_params(WL, seed=5)
    # non-zero biases, so that the bias gradients and updates are exercised too
    rng = np.random.default_rng(6)
    for net in ("actor", "critic"):
        params[net] = [(w, (0.05 * rng.standard_normal(b.shape)).astype(np.float32)) for w, b in params[net]]
    batch = {k: v.astype(np.float64) for k, v in make_batch(WL, ROWS, seed=7).items()}
    # q sums to 1 in float32 only; the hand-derived dz = pi - q (the reference's
    # logits_grad_kernel, networks/actor_loss.mojo:168-191) is the exact derivative when it
    # sums to 1, so both sides get q renormalised in float64
    batch["q"] = batch["q"] / batch["q"].sum(axis=1, keepdims=True)
    return params, batch


def test_gradients_and_dual_match_autograd(setup):
    params, batch = setup
    la = 0.3
    t = {k: torch.tensor(v, dtype=torch.float64) for k, v in batch.items()}
    pa, pc = _tensors(params["actor"]), _tensors(params["critic"])
    alpha = torch.nn.functional.softplus(torch.tensor(la, dtype=torch.float64))
    loss_a, kl_mean = _actor_loss(_mlp(pa, t["obs"]), t["mask"], t["q"], t["logits_old"], alpha)
    loss_a.backward()
    v = _mlp(pc, t["obs"])
    loss_c = (0.5 * (v - t["target"]) ** 2).mean()
    loss_c.backward()
    log_alpha = torch.tensor(la, dtype=torch.float64, requires_grad=True)
    dual = torch.nn.functional.softplus(log_alpha) * (HP["kl_eps"] - kl_mean.detach())
    dual.backward()

    nets = {n: {"params": params[n], "m": [(np.zeros_like(w), np.zeros_like(b)) for w, b in params[n]],
                "v": [(np.zeros_like(w), np.zeros_like(b)) for w, b in params[n]]} for n in ("actor", "critic")}
    out = O.learner_step(batch, actor=nets["actor"], critic=nets["critic"], log_alpha=la, hp=dict(HP, step=1))

    assert abs(out["actor"]["loss"]["loss"] - loss_a.item()) <= 1e-12 * abs(loss_a.item())
    assert abs(out["critic"]["loss"] - loss_c.item()) <= 1e-12 * abs(loss_c.item())
    for net, tp in (("actor", pa), ("critic", pc)):
        for (gw, gb), (tw, tb) in zip(out[net]["grads"], tp):
            for got, want in ((gw, tw.grad.numpy()), (gb, tb.grad.numpy())):
                err = np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-300)
                assert err <= 1e-10, (net, err)
    assert abs(out["log_alpha"]["grad"] - log_alpha.grad.item()) <= 1e-12


def test_three_adam_steps_match_torch_adam(setup):
    """Three learner steps with eps = 1e-8 for both networks and log_alpha: autograd gives
    each step's gradients at the current weights, torch.optim.Adam and the oracle's Adam
    apply the same gradients, and parameters and moments must agree to float64 rounding."""
    params, batch = setup
    la0 = 0.3
    t = {k: torch.tensor(v, dtype=torch.float64) for k, v in batch.items()}
    pa, pc = _tensors(params["actor"]), _tensors(params["critic"])
    log_alpha = torch.tensor(la0, dtype=torch.float64, requires_grad=True)
    leaves = [p for pair in pa + pc for p in pair] + [log_alpha]
    opt = torch.optim.Adam(leaves, lr=3e-4, betas=(0.9, 0.999), eps=1e-8)
    mine = [(p.detach().numpy().copy(), np.zeros(p.shape), np.zeros(p.shape)) for p in leaves]
    for step in (1, 2, 3):
        opt.zero_grad()
        alpha = torch.nn.functional.softplus(log_alpha.detach())
        loss_a, kl_mean = _actor_loss(_mlp(pa, t["obs"]), t["mask"], t["q"], t["logits_old"], alpha)
        loss_a.backward()
        (0.5 * (_mlp(pc, t["obs"]) - t["target"]) ** 2).mean().backward()
        (torch.nn.functional.softplus(log_alpha) * (HP["kl_eps"] - kl_mean.detach())).backward()
        grads = [p.grad.numpy().copy() for p in leaves]
        opt.step()
        mine = [O.adam_step(p, g, m, v, step, 3e-4, 0.9, 0.999, 1e-8) for (p, m, v), g in zip(mine, grads)]
    for (p, m, v), leaf in zip(mine, leaves):
        st = opt.state[leaf]
        moved = np.max(np.abs(leaf.detach().numpy() - p)) / 9e-4  # three steps move a weight by <= 9e-4
        assert moved <= 1e-9, moved
        assert np.allclose(m, st["exp_avg"].numpy(), rtol=1e-12, atol=0)
        assert np.allclose(v, st["exp_avg_sq"].numpy(), rtol=1e-12, atol=0)
