"""Pin the CPU oracle against the reference's own golden tensors (CPU only).

Each test mirrors one reference test file and uses that file's tolerance, so that
the oracle the GPU parity tests lean on is itself checked against what the
reference's JAX/optax/Stoix generators produced.
"""

import math

import numpy as np
import pytest

from golden_io import read_f32, max_abs, max_rel_of_max
from oracle import spo_oracle as O


def _params(prefix, dims):
    out = []
    for i in range(len(dims) - 1):
        w = read_f32(f"{prefix}w{i + 1}", (dims[i], dims[i + 1]))
        b = read_f32(f"{prefix}b{i + 1}", (dims[i + 1],))
        out.append((w, b))
    return out


@pytest.mark.parametrize("case,m,k,n", [(0, 4, 18, 64), (1, 64, 64, 64), (2, 7, 5, 3)])
def test_linear_forward(case, m, k, n):
    # tests/test_linear.mojo:49 — tol 1e-5 * sqrt(K)
    x = read_f32(f"linear{case}_x", (m, k))
    w = read_f32(f"linear{case}_w", (k, n))
    b = read_f32(f"linear{case}_b", (n,))
    y = read_f32(f"linear{case}_y", (m, n))
    assert max_abs(O.linear_forward(x, w, b), y) <= 1e-5 * math.sqrt(k)


@pytest.mark.parametrize("case,m,k,n", [(0, 3, 4, 8), (1, 20, 18, 64), (2, 64, 64, 64), (3, 1, 1, 1)])
def test_linear_backward(case, m, k, n):
    # tests/test_linear_backward.mojo:287-292 — dW, db 1e-5*sqrt(M); dx 1e-5*sqrt(N)
    x = read_f32(f"linbwd{case}_x", (m, k))
    w = read_f32(f"linbwd{case}_w", (k, n))
    dy = read_f32(f"linbwd{case}_dy", (m, n))
    dw, db, dx = O.linear_backward(x, w, dy)
    assert max_abs(dw, read_f32(f"linbwd{case}_dw", (k, n))) <= 1e-5 * math.sqrt(m)
    assert max_abs(db, read_f32(f"linbwd{case}_db", (n,))) <= 1e-5 * math.sqrt(m)
    assert max_abs(dx, read_f32(f"linbwd{case}_dx", (m, k))) <= 1e-5 * math.sqrt(n)


@pytest.mark.parametrize("hidden", [32, 64, 256])
@pytest.mark.parametrize("m", [5, 64])
def test_critic_forward(hidden, m):
    # tests/test_critic_mlp.mojo:83-90 — per-layer tolerance grows with depth
    p = _params(f"critic_h{hidden}_", (18, hidden, hidden, 1))
    x = read_f32(f"critic_h{hidden}_x{m}", (m, 18))
    acts, v = O.mlp_forward(p, x)
    assert max_abs(acts[0], read_f32(f"critic_h{hidden}_a1_{m}", (m, hidden))) <= 1e-5 * math.sqrt(18)
    assert max_abs(acts[1], read_f32(f"critic_h{hidden}_a2_{m}", (m, hidden))) <= 2e-5 * math.sqrt(hidden)
    assert max_abs(v, read_f32(f"critic_h{hidden}_v{m}", (m, 1))) <= 3e-5 * math.sqrt(hidden)


@pytest.mark.parametrize("hidden,m", [(32, 20), (64, 64)])
def test_critic_backward(hidden, m):
    # tests/test_critic_backward.mojo:80-105 — grads 1e-6*sqrt(m*H)
    t = f"cbwd_h{hidden}_m{m}_"
    p = _params(t, (18, hidden, hidden, 1))
    x = read_f32(t + "x", (m, 18))
    target = read_f32(t + "target", (m, 1))
    acts, v = O.mlp_forward(p, x)
    assert max_abs(v, read_f32(t + "v", (m, 1))) <= 1e-5 * math.sqrt(hidden)
    vl = O.value_loss(v, target, 1.0 / m)
    grads = O.mlp_backward(p, x, acts, vl["dv"])
    tol = 1e-6 * math.sqrt(m * hidden)
    dims = (18, hidden, hidden, 1)
    for i, (dw, db) in enumerate(grads):
        assert max_abs(dw, read_f32(f"{t}dw{i + 1}", (dims[i], dims[i + 1]))) <= tol
        assert max_abs(db, read_f32(f"{t}db{i + 1}", (dims[i + 1],))) <= tol


@pytest.mark.parametrize("hidden", [32, 64, 256])
@pytest.mark.parametrize("m", [5, 64])
def test_actor_forward(hidden, m):
    # tests/test_actor.mojo:27,82-84 — TOL 2e-5
    t = f"actor_h{hidden}_"
    p = _params(t, (18, hidden, hidden, 9))
    x = read_f32(f"{t}x{m}", (m, 18))
    mask = read_f32(f"{t}mask{m}", (m, 9))
    _, z = O.mlp_forward(p, x)
    assert max_abs(z, read_f32(f"{t}raw{m}", (m, 9))) <= 2e-5
    zm = O.masked_logits(z, mask)
    want_masked = read_f32(f"{t}masked{m}", (m, 9))
    legal = mask != 0
    assert max_abs(zm[legal], want_masked[legal]) <= 2e-5
    assert np.all(want_masked[~legal] == np.float32(O.NEG_INF))
    assert np.all(zm[~legal] == O.NEG_INF)
    assert max_abs(O.softmax_rows(zm), read_f32(f"{t}probs{m}", (m, 9))) <= 2e-5


@pytest.mark.parametrize("name,batch,hidden", [("bw_small", 5, 32), ("bw_big", 40, 64)])
def test_actor_backward(name, batch, hidden):
    # tests/test_actor_backward.mojo:95-163 — pi 2e-5, loss 2e-5, dz 2e-6 and exactly
    # 0 on masked cells, gradients rel 1e-4 of max|want|
    t = name + "_"
    p = _params(t, (18, hidden, hidden, 9))
    x = read_f32(t + "x", (batch, 18))
    mask = read_f32(t + "mask", (batch, 9))
    q = read_f32(t + "q", (batch, 9))
    acts, z = O.mlp_forward(p, x)
    assert max_abs(z, read_f32(t + "z", (batch, 9))) <= 2e-5
    al = O.actor_loss(z, mask, q, None, None, 0.0, 1.0 / batch)
    assert max_abs(al["pi"], read_f32(t + "pi", (batch, 9))) <= 2e-5
    assert abs(al["loss"] - float(read_f32(t + "loss")[0])) <= 2e-5
    want_dz = read_f32(t + "dz", (batch, 9))
    assert max_abs(al["dz"], want_dz) <= 2e-6
    assert np.all(al["dz"][mask == 0] == 0.0)
    grads = O.mlp_backward(p, x, acts, al["dz"])
    dims = (18, hidden, hidden, 9)
    for i, (dw, db) in enumerate(grads):
        assert max_rel_of_max(dw, read_f32(f"{t}dw{i + 1}", (dims[i], dims[i + 1]))) <= 1e-4
        assert max_rel_of_max(db, read_f32(f"{t}db{i + 1}", (dims[i + 1],))) <= 1e-4


@pytest.mark.parametrize("case,batch", [("small", 3), ("mid", 7), ("big", 32), ("multiblock", 70)])
def test_cross_entropy_rows(case, batch):
    # tests/test_actor_loss.mojo:26 — TOL 2e-5
    t = f"ce_{case}_"
    logits = read_f32(t + "logits", (batch, 9))
    q = read_f32(t + "q", (batch, 9))
    log_pi = O.log_softmax_rows(logits)
    want_lp = read_f32(t + "logpi", (batch, 9))
    legal = read_f32(t + "mask", (batch, 9)) != 0
    assert max_abs(log_pi[legal], want_lp[legal]) <= 2e-5
    ce = O.cross_entropy_rows(q, log_pi)
    h = O.entropy_rows(q)
    assert max_abs(ce, read_f32(t + "per_state")) <= 2e-5
    assert max_abs(h, read_f32(t + "entropy")) <= 2e-5
    assert max_abs(O.kl_rows(ce, h), read_f32(t + "kl")) <= 2e-5
    assert abs(ce.mean() - float(read_f32(t + "loss")[0])) <= 2e-5


def test_known_answers():
    # tests/test_actor_loss.mojo:158 and :265 — ln 3 and H(0.5, 0.3, 0.2)
    q = np.array([[1 / 3, 1 / 3, 1 / 3, 0, 0, 0, 0, 0, 0]])
    assert abs(O.entropy_rows(q)[0] - 1.0986123) < 1e-6
    q = np.array([[0.5, 0.3, 0.2, 0, 0, 0, 0, 0, 0]])
    assert abs(O.entropy_rows(q)[0] - 1.0296531) < 1e-6
    # tests/test_optim.mojo:131-158 — (3, 4, 12) has norm 13; clip 6.5 gives 0.5
    n = O.global_norm([np.array([3.0]), np.array([4.0]), np.array([12.0])])
    assert abs(n - 13.0) < 1e-9
    assert abs(O.global_clip_scale(n, 6.5) - 0.5) < 1e-12


@pytest.mark.parametrize("prefix,rows,cols", [("", 6, 16), ("wide_", 4, 100)])
def test_softmax_family(prefix, rows, cols):
    # tests/test_softmax.mojo — stable softmax, logsumexp, log_softmax
    a = read_f32(("softmax_in" if not prefix else "wide_in"), (rows, cols))
    sm = read_f32("softmax_out" if not prefix else "wide_softmax", (rows, cols))
    lse = read_f32("logsumexp_out" if not prefix else "wide_logsumexp", (rows,))
    lsm = read_f32("logsoftmax_out" if not prefix else "wide_logsoftmax", (rows, cols))
    assert max_abs(O.softmax_rows(a), sm) <= 1e-6
    # tests/test_softmax.mojo:80-88 — logsumexp compared relatively (the +1000 row)
    got = O.logsumexp_rows(a)
    assert np.max(np.abs(got - lse) / np.maximum(np.abs(lse), 1.0)) <= 1e-6
    assert max_abs(O.log_softmax_rows(a), lsm) <= 1e-4


@pytest.mark.parametrize("case", [0, 1])
def test_adam_with_global_clip(case):
    # tests/test_optim.mojo:35 — TOL 2e-6 absolute; optax chain(clip 0.5, adam eps 1e-5)
    shapes = [("w1", (4, 5)), ("b1", (5,)), ("w2", (5, 5)), ("b2", (5,)), ("w3", (5, 1)), ("b3", (1,))]
    p = {n: read_f32(f"adam{case}_{n}_p0", s).astype(np.float64) for n, s in shapes}
    g = {n: read_f32(f"adam{case}_{n}_g", s) for n, s in shapes}
    m = {n: np.zeros(s) for n, s in shapes}
    v = {n: np.zeros(s) for n, s in shapes}
    scale = O.global_clip_scale(O.global_norm(list(g.values())), 0.5)
    assert (scale < 1.0) == (case == 1)
    for step in (1, 2, 3):
        for n, s in shapes:
            p[n], m[n], v[n] = O.adam_step(p[n], g[n], m[n], v[n], step, 3e-4, 0.9, 0.999, 1e-5, scale)
            assert max_abs(p[n], read_f32(f"adam{case}_{n}_p{step}", s)) <= 2e-6


def test_ema():
    # tests/test_ema.mojo — optax.incremental_update, tau 0.005, 10 steps
    # optax runs the chain in float32; the oracle is run in float32 here so that the
    # ten rounding steps match (in float64 it drifts ~1e-6 from the golden by step 8).
    t = read_f32("ema_target0")
    online = read_f32("ema_online")
    for k in range(1, 11):
        t = O.ema_update(t, online, np.float32(0.005), np.float32).astype(np.float32)
        assert max_abs(t, read_f32(f"ema_target{k}")) <= 1e-6


@pytest.mark.parametrize("case,b,t", [(0, 4, 16), (1, 4, 16), (2, 8, 32)])
def test_truncated_gae(case, b, t):
    # tests/test_gae.mojo — Stoix batch_truncated_generalized_advantage_estimation
    r = {n: read_f32(f"gae{case}_{n}", (b, t)) for n in
         ("r", "discount", "v_tm1", "v_t", "trunc", "adv", "targets")}
    adv, targets = O.truncated_gae(r["r"], r["discount"], r["v_tm1"], r["v_t"], r["trunc"], 0.95)
    assert max_abs(adv, r["adv"]) <= 1e-5
    assert max_abs(targets, r["targets"]) <= 1e-5


def test_kl_extension_algebra():
    """The alpha*KL(pi_old||pi) gradient (no reference golden): check dz against a
    central finite difference of the oracle's own loss, in float64."""
    rng = np.random.default_rng(3)
    b, a = 6, 9
    mask = (rng.random((b, a)) < 0.6).astype(np.float32)
    mask[:, 0] = 1
    z = rng.normal(size=(b, a))
    q = rng.gamma(0.3, size=(b, a)) * mask
    q /= q.sum(1, keepdims=True)
    z_old = rng.normal(size=(b, a))
    la = 0.3
    base = O.actor_loss(z, mask, q, z_old, la, 0.01, 1.0 / b)
    h = 1e-6
    for i in range(b):
        for j in range(a):
            zp = z.copy()
            zm = z.copy()
            zp[i, j] += h
            zm[i, j] -= h
            num = (O.actor_loss(zp, mask, q, z_old, la, 0.01, 1.0 / b)["loss"]
                   - O.actor_loss(zm, mask, q, z_old, la, 0.01, 1.0 / b)["loss"]) / (2 * h)
            # q sums to 1 over legal cells, so (pi - q) is the exact derivative
            assert abs(num - base["dz"][i, j]) < 1e-7
    # dual: d/dlog_alpha of softplus(la) * (eps - KL) = sigmoid(la) * (eps - KL)
    kl = base["kl_old_mean"]
    num = (O.softplus(la + h) - O.softplus(la - h)) / (2 * h) * (0.01 - kl)
    assert abs(num - base["dlog_alpha"]) < 1e-8
