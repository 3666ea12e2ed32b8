"""The reference's own golden tensors through libspo_cuda (GPU).

Each test follows one reference test file (tests/test_*.mojo of spo-mojo), calls the
same-named function of spo_mojo_b200.networks (which enqueues libspo_cuda kernels
through the C ABI) and uses that file's tolerance.
"""

import math

import numpy as np
import pytest
import torch

from golden_io import read_f32, max_abs, max_rel_of_max

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def N():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from spo_mojo_b200 import networks
    return networks


@pytest.fixture(scope="module")
def ctx(N):
    return N.DeviceContext(0)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def _params(prefix, dims):
    return [(read_f32(f"{prefix}w{i + 1}", (dims[i], dims[i + 1])), read_f32(f"{prefix}b{i + 1}", (dims[i + 1],)))
            for i in range(len(dims) - 1)]


@pytest.mark.parametrize("case,m,k,n", [(0, 4, 18, 64), (1, 64, 64, 64), (2, 7, 5, 3)])
def test_linear(N, ctx, case, m, k, n):
    # tests/test_linear.mojo:49 — tol 1e-5 * sqrt(K)
    x, w, b = (dev(read_f32(f"linear{case}_{s}")) for s in "xwb")
    y = N.zero_buffer(ctx, m * n)
    N.linear_forward(ctx, y, x, w, b, m, k, n)
    assert max_abs(host(y), read_f32(f"linear{case}_y")) <= 1e-5 * math.sqrt(k)


@pytest.mark.parametrize("case,m,k,n", [(0, 3, 4, 8), (1, 20, 18, 64), (2, 64, 64, 64), (3, 1, 1, 1)])
def test_linear_backward(N, ctx, case, m, k, n):
    # tests/test_linear_backward.mojo:287-292
    x, w, dy = (dev(read_f32(f"linbwd{case}_{s}")) for s in ("x", "w", "dy"))
    dw, db, dx = N.zero_buffer(ctx, k * n), N.zero_buffer(ctx, n), N.zero_buffer(ctx, m * k)
    N.linear_backward(ctx, dw, db, dx, x, w, dy, m, k, n)
    assert max_abs(host(dw), read_f32(f"linbwd{case}_dw")) <= 1e-5 * math.sqrt(m)
    assert max_abs(host(db), read_f32(f"linbwd{case}_db")) <= 1e-5 * math.sqrt(m)
    assert max_abs(host(dx), read_f32(f"linbwd{case}_dx")) <= 1e-5 * math.sqrt(n)


@pytest.mark.parametrize("hidden", [32, 64, 256])
@pytest.mark.parametrize("m", [5, 64])
def test_critic_forward(N, ctx, hidden, m):
    # tests/test_critic_mlp.mojo:83-90
    dims = (18, hidden, hidden, 1)
    t = f"critic_h{hidden}_"
    p = N.zero_critic_params(ctx, 18, hidden, 1)
    p.load(_params(t, dims))
    cache = N.CriticCache(ctx, m, dims)
    N.critic_forward(ctx, p, cache, dev(read_f32(f"{t}x{m}")), m)
    assert max_abs(host(cache.act(0, m)), read_f32(f"{t}a1_{m}", (m, hidden))) <= 1e-5 * math.sqrt(18)
    assert max_abs(host(cache.act(1, m)), read_f32(f"{t}a2_{m}", (m, hidden))) <= 2e-5 * math.sqrt(hidden)
    assert max_abs(host(cache.value), read_f32(f"{t}v{m}")) <= 3e-5 * math.sqrt(hidden)


@pytest.mark.parametrize("hidden,m", [(32, 20), (64, 64)])
def test_critic_backward(N, ctx, hidden, m):
    # tests/test_critic_backward.mojo:80-105 — tol 1e-6 * sqrt(m * H)
    dims = (18, hidden, hidden, 1)
    t = f"cbwd_h{hidden}_m{m}_"
    p = N.zero_critic_params(ctx, 18, hidden, 1)
    p.load(_params(t, dims))
    cache = N.CriticCache(ctx, m, dims)
    grads = N.CriticGrads(ctx, dims)
    scratch = N.CriticScratch(ctx, m, dims)
    x = dev(read_f32(t + "x"))
    N.critic_forward(ctx, p, cache, x, m)
    N.critic_backward(ctx, p, cache, grads, scratch, x, dev(read_f32(t + "target")), m)
    tol = 1e-6 * math.sqrt(m * hidden)
    for i in range(3):
        assert max_abs(host(grads.p.w[i]), read_f32(f"{t}dw{i + 1}", (dims[i], dims[i + 1]))) <= tol
        assert max_abs(host(grads.p.b[i]), read_f32(f"{t}db{i + 1}")) <= tol


@pytest.mark.parametrize("hidden", [32, 64, 256])
@pytest.mark.parametrize("m", [5, 64])
def test_actor_probs(N, ctx, hidden, m):
    # tests/test_actor.mojo:27,82-84 — TOL 2e-5
    t = f"actor_h{hidden}_"
    actor = N.Actor(ctx, m, hidden, in_dim=18)
    actor.params.load(_params(t, (18, hidden, hidden, 9)))
    actor.forward(ctx, dev(read_f32(f"{t}x{m}")), dev(read_f32(f"{t}mask{m}")), m)
    mask = read_f32(f"{t}mask{m}", (m, 9))
    got = host(actor.cache.value).reshape(m, 9)
    want = read_f32(f"{t}masked{m}", (m, 9))
    assert max_abs(got[mask != 0], want[mask != 0]) <= 2e-5
    assert np.all(got[mask == 0] == want[mask == 0])          # exactly -FLT_MAX
    assert max_abs(host(actor.probs).reshape(m, 9), read_f32(f"{t}probs{m}", (m, 9))) <= 2e-5


@pytest.mark.parametrize("name,batch,hidden", [("bw_small", 5, 32), ("bw_big", 40, 64)])
def test_actor_backward_stepwise(N, ctx, name, batch, hidden):
    # tests/test_actor_backward.mojo:95-163 through the reference's step-by-step chain
    t = name + "_"
    dims = (18, hidden, hidden, 9)
    actor = N.Actor(ctx, batch, hidden, in_dim=18)
    actor.params.load(_params(t, dims))
    x, mask, q = dev(read_f32(t + "x")), dev(read_f32(t + "mask")), dev(read_f32(t + "q"))
    actor.forward(ctx, x, mask, batch)
    assert max_abs(host(actor.probs), read_f32(t + "pi")) <= 2e-5
    grads = N.CriticGrads(ctx, dims)
    scratch = N.CriticScratch(ctx, batch, dims)
    N.actor_backward(ctx, actor.params, actor.cache, grads, scratch, x, actor.probs, q, mask, batch)
    dz = host(scratch.dvalue).reshape(batch, 9)
    assert max_abs(dz, read_f32(t + "dz", (batch, 9))) <= 2e-6
    assert np.all(dz[read_f32(t + "mask", (batch, 9)) == 0] == 0.0)
    for i in range(3):
        assert max_rel_of_max(host(grads.p.w[i]), read_f32(f"{t}dw{i + 1}", (dims[i], dims[i + 1]))) <= 1e-4
        assert max_rel_of_max(host(grads.p.b[i]), read_f32(f"{t}db{i + 1}")) <= 1e-4


@pytest.mark.parametrize("name,batch,hidden", [("bw_small", 5, 32), ("bw_big", 40, 64)])
def test_actor_backward_fused_learner(ctx, name, batch, hidden):
    """Same goldens through the fused learner step (one head kernel, no KL)."""
    from spo_mojo_b200.learner import Learner
    t = name + "_"
    dims = (18, hidden, hidden, 9)
    L = Learner(actor_dims=dims, max_rows=batch, use_kl=False, dual=False)
    L.load(actor=_params(t, dims))
    L.backward({"obs": dev(read_f32(t + "x", (batch, 18))), "mask": dev(read_f32(t + "mask", (batch, 9))),
                "q": dev(read_f32(t + "q", (batch, 9)))})
    st = L.stats()
    assert abs(st["actor_loss"] - float(read_f32(t + "loss")[0])) <= 2e-5
    for i, (dw, db) in enumerate(L.tensors("actor", L.grads)):
        assert max_rel_of_max(host(dw), read_f32(f"{t}dw{i + 1}", (dims[i], dims[i + 1]))) <= 1e-4
        assert max_rel_of_max(host(db), read_f32(f"{t}db{i + 1}")) <= 1e-4


@pytest.mark.parametrize("case,batch", [("small", 3), ("mid", 7), ("big", 32), ("multiblock", 70)])
def test_cross_entropy_rows(N, ctx, case, batch):
    # tests/test_actor_loss.mojo:26 — TOL 2e-5
    t = f"ce_{case}_"
    logits, q = dev(read_f32(t + "logits")), dev(read_f32(t + "q"))
    lp, ce, h, kl = (N.zero_buffer(ctx, n) for n in (batch * 9, batch, batch, batch))
    N.log_softmax_rows(ctx, lp, logits, batch, 9)
    N.cross_entropy_rows(ctx, ce, q, lp, batch, 9)
    N.entropy_rows(ctx, h, q, batch, 9)
    N.kl_rows(ctx, kl, ce, h, batch)
    legal = read_f32(t + "mask", (batch, 9)) != 0
    assert max_abs(host(lp).reshape(batch, 9)[legal], read_f32(t + "logpi", (batch, 9))[legal]) <= 2e-5
    assert max_abs(host(ce), read_f32(t + "per_state")) <= 2e-5
    assert max_abs(host(h), read_f32(t + "entropy")) <= 2e-5
    assert max_abs(host(kl), read_f32(t + "kl")) <= 2e-5


@pytest.mark.parametrize("inp,sm,lse,lsm,rows,cols", [
    ("softmax_in", "softmax_out", "logsumexp_out", "logsoftmax_out", 6, 16),
    ("wide_in", "wide_softmax", "wide_logsumexp", "wide_logsoftmax", 4, 100)])
def test_softmax_family(N, ctx, inp, sm, lse, lsm, rows, cols):
    # tests/test_softmax.mojo:31,80-88
    a = dev(read_f32(inp))
    o1, o2, o3 = N.zero_buffer(ctx, rows * cols), N.zero_buffer(ctx, rows), N.zero_buffer(ctx, rows * cols)
    N.softmax_rows(ctx, o1, a, rows, cols)
    N.logsumexp_rows(ctx, o2, a, rows, cols)
    N.log_softmax_rows(ctx, o3, a, rows, cols)
    assert max_abs(host(o1), read_f32(sm)) <= 1e-6
    want = read_f32(lse)
    assert np.max(np.abs(host(o2) - want) / np.maximum(np.abs(want), 1.0)) <= 1e-6
    assert max_abs(host(o3), read_f32(lsm)) <= 1e-4


@pytest.mark.parametrize("case", [0, 1])
def test_adam_with_global_clip(N, ctx, case):
    # tests/test_optim.mojo:35 — TOL 2e-6; one flat buffer for the six tensors (61 floats,
    # so the kernel's scalar tail runs too)
    names = ["w1", "b1", "w2", "b2", "w3", "b3"]
    p0 = np.concatenate([read_f32(f"adam{case}_{n}_p0") for n in names])
    g = np.concatenate([read_f32(f"adam{case}_{n}_g") for n in names])
    p, gd = dev(p0), dev(g)
    state = N.AdamState(ctx, p0.size)
    scale = N.global_clip_scale(N.sum_squares(ctx, gd, g.size), 0.5)
    assert (scale < 1.0) == (case == 1)
    for step in (1, 2, 3):
        N.adam_step(ctx, p, gd, state, p0.size, 3e-4, scale, step)
        want = np.concatenate([read_f32(f"adam{case}_{n}_p{step}") for n in names])
        assert max_abs(host(p), want) <= 2e-6


def test_ema(N, ctx):
    # tests/test_ema.mojo:122 — 1e-6 over 10 steps
    t = dev(read_f32("ema_target0"))
    online = dev(read_f32("ema_online"))
    for k in range(1, 11):
        N.ema_update(ctx, t, online, t.numel(), 0.005)
        assert max_abs(host(t), read_f32(f"ema_target{k}")) <= 1e-6


@pytest.mark.parametrize("case,b,t", [(0, 4, 16), (1, 4, 16), (2, 8, 32)])
def test_truncated_gae(N, ctx, case, b, t):
    # tests/test_gae.mojo:29 — TOL 1e-5
    arrs = {n: dev(read_f32(f"gae{case}_{n}")) for n in ("r", "discount", "v_tm1", "v_t", "trunc")}
    adv, tgt = N.zero_buffer(ctx, b * t), N.zero_buffer(ctx, b * t)
    N.truncated_gae(ctx, adv, tgt, arrs["r"], arrs["discount"], arrs["v_tm1"], arrs["v_t"],
                    arrs["trunc"], b, t, 0.95)
    assert max_abs(host(adv), read_f32(f"gae{case}_adv")) <= 1e-5
    assert max_abs(host(tgt), read_f32(f"gae{case}_targets")) <= 1e-5
