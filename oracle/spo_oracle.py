"""CPU oracle of the SPO learner step. TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import it;
the library (``spo_mojo_b200`` over ``libspo_cuda.so``) never calls it and has no
CPU fallback.

It restates, in numpy, what the reference's ``networks/`` layer computes
(josedanielchg/spo-mojo, Mojo 1.0.0b1). Every function cites the reference
file:line it follows. Arithmetic is float64 by default (``dtype`` argument), so that
the oracle is more precise than the fp32 kernels it checks; the CPU baseline runs the
same code in float32.

Pinning. The restatement is checked against the reference's own committed golden
tensors (copied unchanged into ``tests/golden/ref``; produced by the reference's
JAX/optax/Stoix generators at highest matmul precision) in
``tests/test_oracle_golden.py``: linear forward/backward, critic MLP forward and
gradients, actor masked softmax, actor loss + dz + gradients, CE/H/KL rows, softmax
family, Adam with global-norm clip, EMA and truncated GAE.

Parity unpinned (no reference code or golden covers these; they rest on this
restatement and on the algebra written beside each): the alpha*KL(pi_old||pi) term,
the log_alpha dual gradient, the 27-wide three-plane input, more than two hidden
layers, and Adam eps = 1e-8 (the reference hard-codes 1e-5). Their algebra is
cross-checked (tests/test_oracle_autograd.py) against float64 automatic
differentiation of the loss written from its definition and against torch.optim.Adam,
the role JAX autodiff and optax play for the reference's own goldens.
"""

import numpy as np

# ops/common.mojo:19-23 — the masking constant is the most negative FINITE float32,
# not -inf, so a fully masked row degenerates to uniform instead of NaN.
NEG_INF = float(np.finfo(np.float32).min)


# ---------------------------------------------------------------------------
# Linear layer and MLP
# ---------------------------------------------------------------------------

def linear_forward(x, w, b, dtype=np.float64):
    """y = x @ W + b with W stored [in, out] row-major (networks/linear.mojo:37-84)."""
    return x.astype(dtype, copy=False) @ w.astype(dtype, copy=False) + b.astype(dtype, copy=False)


def relu(a):
    """In-place ReLU max(a, 0) (networks/mlp.mojo:34-46)."""
    return np.maximum(a, 0)


def linear_backward(x, w, dy, dtype=np.float64):
    """The three gradients of y = xW + b (networks/linear.mojo:99-167).

    dW = x^T dy  (linear_grad_w_kernel, :120-131)
    db = sum over rows of dy  (linear_grad_b_kernel, :134-149)
    dx = dy W^T  (linear_grad_x_kernel, :152-167)
    """
    x = x.astype(dtype, copy=False)
    w = w.astype(dtype, copy=False)
    dy = dy.astype(dtype, copy=False)
    return x.T @ dy, dy.sum(axis=0), dy @ w.T


def mlp_forward(params, x, dtype=np.float64):
    """MLP forward with ReLU between layers and none after the last.

    networks/mlp.mojo:105-123 (critic_forward) generalised from three Linear layers
    to L. ``params`` is a list of (W [d_i, d_{i+1}], b [d_{i+1}]). Returns the list
    of post-ReLU hidden activations (the CriticCache a1, a2, ...) and the output.
    """
    acts = []
    h = x.astype(dtype, copy=False)
    last = len(params) - 1
    for i, (w, b) in enumerate(params):
        y = linear_forward(h, w, b, dtype)
        if i < last:
            y = relu(y)
            acts.append(y)
        h = y
    return acts, h


def mlp_backward(params, x, acts, dout, dtype=np.float64, masks=None):
    """Gradients of all layers from dL/d(output) (networks/mlp.mojo:236-275).

    backward_from_dvalue: walk the layers top-down; each linear_backward hands dx to
    the layer below, which passes through relu_backward_kernel
    (networks/mlp.mojo:155-166): the gradient is zeroed where the STORED post-ReLU
    activation is <= 0. Returns a list of (dW, db) in layer order.

    ``masks`` (optional, one boolean array per hidden layer) replaces the ReLU decisions
    acts > 0: a checker uses it to differentiate through the same branch of the
    piecewise-linear network as an fp32 computation whose activations sit within
    rounding distance of zero.
    """
    grads = [None] * len(params)
    d = dout.astype(dtype, copy=False)
    for i in range(len(params) - 1, -1, -1):
        inp = x if i == 0 else acts[i - 1]
        dw, db, dx = linear_backward(inp, params[i][0], d, dtype)
        grads[i] = (dw, db)
        if i > 0:
            keep = acts[i - 1] > 0 if masks is None else masks[i - 1]
            d = np.where(keep, dx, 0.0)
    return grads


# ---------------------------------------------------------------------------
# Softmax family (ops/softmax.mojo) and actor masking (networks/actor.mojo)
# ---------------------------------------------------------------------------

def masked_logits(z, mask, dtype=np.float64):
    """logits[mask == 0] = NEG_INF (mask_logits_kernel, networks/actor.mojo:50-71)."""
    return np.where(mask == 0, NEG_INF, z.astype(dtype, copy=False))


def logsumexp_rows(a, dtype=np.float64):
    """m + log(sum exp(a - m)) per row (ops/softmax.mojo:81-98)."""
    a = a.astype(dtype, copy=False)
    m = a.max(axis=1, keepdims=True)
    return (m + np.log(np.exp(a - m).sum(axis=1, keepdims=True)))[:, 0]


def softmax_rows(a, dtype=np.float64):
    """Stable softmax per row, max subtracted first (ops/softmax.mojo:58-78)."""
    a = a.astype(dtype, copy=False)
    e = np.exp(a - a.max(axis=1, keepdims=True))
    return e / e.sum(axis=1, keepdims=True)


def log_softmax_rows(a, dtype=np.float64):
    """a - logsumexp(a) per row, without going through the softmax (ops/softmax.mojo:101-135)."""
    a = a.astype(dtype, copy=False)
    return a - logsumexp_rows(a, dtype)[:, None]


# ---------------------------------------------------------------------------
# Losses
# ---------------------------------------------------------------------------

def cross_entropy_rows(q, log_pi):
    """-sum_a q log pi, skipping q == 0 terms (networks/actor_loss.mojo:40-65)."""
    return -np.where(q != 0, q * np.where(q != 0, log_pi, 0.0), 0.0).sum(axis=1)


def entropy_rows(q):
    """H(q) = -sum_{q > 0} q log q (networks/actor_loss.mojo:105-116)."""
    safe = np.where(q > 0, q, 1.0)
    return -np.where(q > 0, q * np.log(safe), 0.0).sum(axis=1)


def kl_rows(ce, h):
    """KL(q || pi) = CE - H(q) (networks/actor_loss.mojo:119-124)."""
    return ce - h


def softplus(x):
    return np.log1p(np.exp(-abs(x))) + max(x, 0.0)


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def actor_loss(z, mask, q, z_old, log_alpha, eps_kl, scale, dtype=np.float64):
    """See ``_actor_loss``; ``z_old=None`` drops the KL term (alpha = 0), which is
    exactly the reference's eq-11 loss."""
    return _actor_loss(z, mask, q, z_old, log_alpha, eps_kl, scale, dtype)


def _actor_loss(z, mask, q, z_old, log_alpha, eps_kl, scale, dtype):
    """Equation-11 actor loss with the alpha*KL(pi_old || pi) term, and its gradient.

    Reference part (networks/actor.mojo:50-122, networks/actor_loss.mojo:40-191,
    tests/golden/gen/gen_actor_backward.py:93-106):
        z_m = mask(z); log pi = log_softmax(z_m); pi = softmax(z_m)
        ce_row = -sum_{q != 0} q log pi
        dz = (pi - q) * scale, forced to 0 on illegal cells
    Extension (no reference code; parity unpinned, stated here):
        log pi_old = log_softmax(mask(z_old)); pi_old = softmax(mask(z_old))
        kl_old_row = sum_{pi_old > 0} pi_old (log pi_old - log pi)
        alpha = softplus(log_alpha)   (a constant for the policy loss)
        loss_row = ce_row + alpha * kl_old_row
        dz += alpha * (pi - pi_old) * scale      (d/dz of -sum pi_old log pi,
                                                  with sum pi_old = 1)
        dual: L_dual = alpha * (eps_kl - stopgrad(mean kl_old)),
              dL_dual/dlog_alpha = sigmoid(log_alpha) * (eps_kl - mean kl_old),
              with mean kl_old = scale * sum kl_old_row.
    Returns a dict with per-row arrays, the scaled sums and dz.
    """
    zm = masked_logits(z, mask, dtype)
    log_pi = log_softmax_rows(zm, dtype)
    pi = softmax_rows(zm, dtype)
    ce = cross_entropy_rows(q.astype(dtype), log_pi)
    h = entropy_rows(q.astype(dtype))
    if z_old is None:
        pi_old = np.zeros_like(pi)
        kl_old = np.zeros_like(ce)
        alpha = 0.0
        log_alpha = 0.0
    else:
        zo = masked_logits(z_old, mask, dtype)
        log_pi_old = log_softmax_rows(zo, dtype)
        pi_old = softmax_rows(zo, dtype)
        kl_old = np.where(pi_old > 0, pi_old * (np.where(pi_old > 0, log_pi_old, 0.0)
                                                - np.where(pi_old > 0, log_pi, 0.0)),
                          0.0).sum(axis=1)
        alpha = softplus(float(log_alpha))
    per_row = ce + alpha * kl_old
    dz = np.where(mask == 0, 0.0, ((pi - q) + alpha * (pi - pi_old)) * scale)
    kl_mean = scale * kl_old.sum()
    return {
        "log_pi": log_pi, "pi": pi, "ce": ce, "entropy": h, "kl_q": kl_rows(ce, h),
        "kl_old": kl_old, "per_row": per_row, "dz": dz,
        "loss": scale * per_row.sum(), "ce_mean": scale * ce.sum(),
        "entropy_mean": scale * h.sum(), "kl_q_mean": scale * (ce - h).sum(),
        "kl_old_mean": kl_mean, "alpha": alpha,
        "dlog_alpha": sigmoid(float(log_alpha)) * (eps_kl - kl_mean),
    }


def value_loss(v, target, scale, dtype=np.float64):
    """L = scale * sum 0.5 (V - t)^2 and dV = (V - t) * scale.

    value_loss_grad_kernel (networks/mlp.mojo:141-152) with scale = 1/n, and the host
    loss sum of demos/train_critic.mojo:317-327.
    """
    d = v.astype(dtype) - target.astype(dtype)
    return {"loss": scale * (0.5 * d * d).sum(), "dv": d * scale}


# ---------------------------------------------------------------------------
# Optimiser (networks/optim.mojo)
# ---------------------------------------------------------------------------

def global_norm(grads):
    """sqrt of the sum of squares over ALL tensors (sum_squares, networks/optim.mojo:48-73,115-130)."""
    return float(np.sqrt(sum(float((np.asarray(g, np.float64) ** 2).sum()) for g in grads)))


def global_clip_scale(norm, max_norm):
    """1 if norm <= max_norm else max_norm / norm (networks/optim.mojo:133-142)."""
    if not np.isfinite(max_norm) or max_norm <= 0 or norm <= max_norm:
        return 1.0
    return max_norm / norm


def adam_step(p, g, m, v, step, lr, b1=0.9, b2=0.999, eps=1e-5, grad_scale=1.0,
              dtype=np.float64):
    """One Adam step, elementwise (adam_step_kernel networks/optim.mojo:75-99; host
    bias corrections :172-187). eps sits OUTSIDE the sqrt, as in optax. Returns new
    (p, m, v)."""
    g = g.astype(dtype) * grad_scale
    m = b1 * m.astype(dtype) + (1 - b1) * g
    v = b2 * v.astype(dtype) + (1 - b2) * g * g
    bc1 = 1.0 / (1.0 - b1 ** step)
    bc2 = 1.0 / (1.0 - b2 ** step)
    p = p.astype(dtype) - lr * (m * bc1) / (np.sqrt(v * bc2) + eps)
    return p, m, v


def ema_update(target, online, tau, dtype=np.float64):
    """target <- tau*online + (1 - tau)*target (ema_kernel, networks/optim.mojo:145-160)."""
    return tau * online.astype(dtype) + (1 - tau) * target.astype(dtype)


def truncated_gae(reward, discount, v_tm1, v_t, trunc, lam, dtype=np.float64):
    """Stoix truncated GAE walked backwards in time, batch-major [B, T]
    (gae_kernel, rl_utils/multistep.mojo:40-69). Returns (adv, targets)."""
    reward, discount, v_tm1, v_t, trunc = (a.astype(dtype) for a in
                                           (reward, discount, v_tm1, v_t, trunc))
    b, t = reward.shape
    adv = np.zeros((b, t), dtype)
    acc = np.zeros(b, dtype)
    for i in range(t - 1, -1, -1):
        delta = reward[:, i] + discount[:, i] * v_t[:, i] - v_tm1[:, i]
        acc = delta + discount[:, i] * lam * acc * (1 - trunc[:, i])
        adv[:, i] = acc
    return adv, v_tm1 + adv


# ---------------------------------------------------------------------------
# The whole learner step (demos/train_spo.mojo:417-554 composition)
# ---------------------------------------------------------------------------

def learner_step(batch, actor=None, critic=None, log_alpha=0.0, hp=None,
                 dtype=np.float64, scale=None):
    """One learner step: critic block then actor block, each with its own global clip
    and Adam (demos/train_spo.mojo:417-554; separate optimisers per network as in
    :17-21), plus the log_alpha dual update when ``hp['dual']``.

    ``actor``/``critic``: dict(params=[(W, b)...], m=[(mW, mb)...], v=[...], step=int)
    or None. ``batch``: dict(obs, mask, q, logits_old, target). ``hp``: lr_actor,
    lr_critic, b1, b2, eps, max_norm, kl_eps, dual, alpha_m, alpha_v.
    Returns a dict with grads, updated params/moments, and the loss statistics.
    """
    out = {}
    x = batch["obs"]
    rows = x.shape[0]
    scale = 1.0 / rows if scale is None else scale
    step = hp.get("step", 1)
    if critic is not None:
        acts, v = mlp_forward(critic["params"], x, dtype)
        vl = value_loss(v, batch["target"].reshape(v.shape), scale, dtype)
        grads = mlp_backward(critic["params"], x, acts, vl["dv"], dtype)
        flat = [t for pair in grads for t in pair]
        norm = global_norm(flat)
        cs = global_clip_scale(norm, hp["max_norm"])
        new = _adam_net(critic, grads, step, hp["lr_critic"], hp, cs, dtype)
        out["critic"] = {"grads": grads, "loss": vl["loss"], "norm": norm, "acts": acts,
                         "out": v, **new}
    if actor is not None:
        acts, z = mlp_forward(actor["params"], x, dtype)
        al = actor_loss(z, batch["mask"], batch["q"], batch["logits_old"], log_alpha,
                        hp["kl_eps"], scale, dtype)
        grads = mlp_backward(actor["params"], x, acts, al["dz"], dtype)
        flat = [t for pair in grads for t in pair]
        norm = global_norm(flat)
        cs = global_clip_scale(norm, hp["max_norm"])
        new = _adam_net(actor, grads, step, hp["lr_actor"], hp, cs, dtype)
        out["actor"] = {"grads": grads, "loss": al, "norm": norm, "acts": acts, "out": z,
                        **new}
        if hp.get("dual", False):
            g = np.array([al["dlog_alpha"]], dtype)
            p, m, v = adam_step(np.array([log_alpha], dtype), g,
                                np.array([hp.get("alpha_m", 0.0)], dtype),
                                np.array([hp.get("alpha_v", 0.0)], dtype), step,
                                hp["lr_actor"], hp["b1"], hp["b2"], hp["eps"], 1.0, dtype)
            out["log_alpha"] = {"grad": float(g[0]), "value": float(p[0]),
                                "m": float(m[0]), "v": float(v[0])}
    return out


def _adam_net(net, grads, step, lr, hp, clip, dtype):
    params, ms, vs = [], [], []
    for (w, b), (dw, db), (mw, mb), (vw, vb) in zip(net["params"], grads, net["m"], net["v"]):
        pw, mw2, vw2 = adam_step(w, dw, mw, vw, step, lr, hp["b1"], hp["b2"], hp["eps"], clip, dtype)
        pb, mb2, vb2 = adam_step(b, db, mb, vb, step, lr, hp["b1"], hp["b2"], hp["eps"], clip, dtype)
        params.append((pw, pb))
        ms.append((mw2, mb2))
        vs.append((vw2, vb2))
    return {"new_params": params, "new_m": ms, "new_v": vs, "clip": clip}
