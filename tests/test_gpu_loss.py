"""The losses on caller-held outputs (spo_actor_loss_fwd_bwd, spo_value_loss_fwd_bwd)
through the C ABI: the reference's actor-backward and cross-entropy goldens at the
reference tests' tolerances, and the alpha*KL(pi_old || pi) term, its dual gradient and the
value loss against the oracle (losses rel 1e-5, gradients rel 1e-4 of max)."""

import numpy as np
import pytest
import torch

from golden_io import max_abs, max_rel_of_max, read_f32
from oracle import spo_oracle as O

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


@pytest.mark.parametrize("name,batch", [("bw_small", 5), ("bw_big", 40)])
def test_actor_loss_on_reference_logits(N, ctx, name, batch):
    # tests/test_actor_backward.mojo:95-163 of the reference: dz within 2e-6, loss 2e-5
    t = name + "_"
    z, mask, q = (dev(read_f32(t + s, (batch, 9))) for s in ("z", "mask", "q"))
    dz, stats = N.zero_buffer(ctx, batch * 9), N.zero_buffer(ctx, 8)
    N.actor_loss_fwd_bwd(ctx, dz, stats, z, mask, q, batch)
    got = host(dz).reshape(batch, 9)
    assert max_abs(got, read_f32(t + "dz", (batch, 9))) <= 2e-6
    assert np.all(got[read_f32(t + "mask", (batch, 9)) == 0] == 0.0)
    st = host(stats)
    assert abs(st[0] - float(read_f32(t + "loss")[0])) <= 2e-5
    assert abs(st[1] - st[0]) <= 1e-7 and st[4] == 0.0   # no KL term: loss = CE


@pytest.mark.parametrize("case,batch", [("small", 3), ("mid", 7), ("big", 32), ("multiblock", 70)])
def test_actor_loss_statistics_on_ce_goldens(N, ctx, case, batch):
    # tests/test_actor_loss.mojo:26 of the reference — TOL 2e-5 on the per-state values;
    # here their batch means
    t = f"ce_{case}_"
    z, q, mask = (dev(read_f32(t + s, (batch, 9))) for s in ("logits", "q", "mask"))
    dz, stats = N.zero_buffer(ctx, batch * 9), N.zero_buffer(ctx, 8)
    N.actor_loss_fwd_bwd(ctx, dz, stats, z, mask, q, batch)
    st = host(stats)
    assert abs(st[1] - read_f32(t + "per_state").mean()) <= 2e-5
    assert abs(st[2] - read_f32(t + "entropy").mean()) <= 2e-5
    assert abs(st[3] - read_f32(t + "kl").mean()) <= 2e-5


def _actor_case(rows, seed, fully_masked=0, q_zeros=True):
    rng = np.random.default_rng(seed)
    z = rng.normal(0, 2, (rows, 9)).astype(np.float32)
    zo = rng.normal(0, 1, (rows, 9)).astype(np.float32)
    mask = (rng.random((rows, 9)) < 0.6).astype(np.float32)
    mask[np.arange(rows), rng.integers(0, 9, rows)] = 1.0
    if fully_masked:
        mask[:fully_masked] = 0.0
    q = rng.dirichlet(np.full(9, 0.3), rows).astype(np.float32) * mask
    q = q / np.maximum(q.sum(axis=1, keepdims=True), 1e-30)
    if q_zeros:
        q[q < 1e-3] = 0.0
    return z, zo, mask, q.astype(np.float32)


@pytest.mark.parametrize("rows", [1, 3, 129, 1000, 65536])
@pytest.mark.parametrize("log_alpha", [0.0, -1.3])
def test_actor_loss_with_kl_and_dual_vs_oracle(N, ctx, rows, log_alpha):
    z, zo, mask, q = _actor_case(rows, 11 + rows, fully_masked=1 if rows > 2 else 0)
    eps_kl = 0.01
    la = dev(np.array([log_alpha]))
    dz, stats, dla = N.zero_buffer(ctx, rows * 9), N.zero_buffer(ctx, 8), N.zero_buffer(ctx, 1)
    N.actor_loss_fwd_bwd(ctx, dz, stats, dev(z), dev(mask), dev(q), rows, logits_old=dev(zo), log_alpha=la,
                         eps_kl=eps_kl, dlog_alpha=dla)
    ora = O.actor_loss(z, mask, q, zo, log_alpha, eps_kl, 1.0 / rows)
    assert max_rel_of_max(host(dz).reshape(rows, 9), ora["dz"]) <= 1e-4
    st = host(stats)
    for slot, key in ((0, "loss"), (1, "ce_mean"), (2, "entropy_mean"), (3, "kl_q_mean"), (4, "kl_old_mean")):
        assert abs(st[slot] - ora[key]) <= 1e-5 * max(abs(ora[key]), 1e-3), (slot, st[slot], ora[key])
    assert abs(host(dla)[0] - ora["dlog_alpha"]) <= 1e-5 * max(abs(ora["dlog_alpha"]), 1e-3)


def test_actor_loss_scale_and_untouched_slots(N, ctx):
    rows = 257
    z, zo, mask, q = _actor_case(rows, 5)
    dz, stats = N.zero_buffer(ctx, rows * 9), N.zero_buffer(ctx, 8)
    stats.fill_(7.0)
    N.actor_loss_fwd_bwd(ctx, dz, stats, dev(z), None, dev(q), rows, scale=1.0 / 4096)
    ora = O.actor_loss(z, np.ones_like(mask), q, None, 0.0, 0.01, 1.0 / 4096)
    st = host(stats)
    assert abs(st[0] - ora["loss"]) <= 1e-5 * abs(ora["loss"])
    assert np.all(st[5:] == 7.0)                         # the critic's slots are not written
    assert max_rel_of_max(host(dz).reshape(rows, 9), ora["dz"]) <= 1e-4


def test_actor_loss_zero_rows(N, ctx):
    stats = N.zero_buffer(ctx, 8)
    stats.fill_(3.0)
    empty = N.zero_buffer(ctx, 0)
    N.actor_loss_fwd_bwd(ctx, empty, stats, empty, None, empty, 0)
    assert np.all(host(stats)[:5] == 0.0) and np.all(host(stats)[5:] == 3.0)


def test_actor_loss_rejects_bad_arguments(N, ctx):
    from spo_mojo_b200 import ffi
    dz, stats = N.zero_buffer(ctx, 9), N.zero_buffer(ctx, 8)
    with pytest.raises(ffi.SpoError, match="SPO_ERR_SHAPE"):
        N.actor_loss_fwd_bwd(ctx, dz, stats, dz, None, dz, 1, num_actions=33)
    with pytest.raises(ffi.SpoError, match="SPO_ERR_ARG"):
        N.actor_loss_fwd_bwd(ctx, dz, stats, dz, None, dz, 1, logits_old=dz)   # no log_alpha


@pytest.mark.parametrize("n", [1, 1000, 262144])
def test_value_loss_vs_oracle(N, ctx, n):
    rng = np.random.default_rng(n)
    v = rng.normal(0, 1, n).astype(np.float32)
    t = rng.uniform(-2, 2, n).astype(np.float32)
    dv, stats = N.zero_buffer(ctx, n), N.zero_buffer(ctx, 8)
    stats.fill_(5.0)
    N.value_loss_fwd_bwd(ctx, dv, stats, dev(v), dev(t), n)
    ora = O.value_loss(v, t, 1.0 / n)
    st = host(stats)
    assert abs(st[5] - ora["loss"]) <= 1e-5 * abs(ora["loss"])
    assert np.all(np.delete(st, 5) == 5.0)
    assert max_rel_of_max(host(dv), ora["dv"]) <= 1e-6
