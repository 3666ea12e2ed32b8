"""The seeded synthetic learner inputs and initial weights against the workload
definitions: tic-tac-toe boards with each cell uniform over {empty, X, O}, one-hot
encoded as three planes [empty | X | O], at least one legal cell per row, legal mask =
empty plane, q ~ Dirichlet(0.3) over the legal cells, pi_old logits N(0, 1) masked with
the most negative finite float, critic targets sum_{k<5} 0.99^k r_k + 0.99^5 v_boot with
r in {-1, 0, 1} and v_boot ~ U[-1, 1], Glorot-uniform weights and zero biases. Also the
per-sample work counts the roofline figures are built on."""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from spo_mojo_b200.workloads import (NEG_INF, WORKLOADS, cells_of, init_params,  # noqa: E402
                                     make_batch)

ROWS = 20000


@pytest.fixture(scope="module")
def batch():
    return make_batch(WORKLOADS["c2"], ROWS, seed=3)


def test_boards_are_one_hot_with_a_legal_cell(batch):
    obs, mask = batch["obs"], batch["mask"]
    assert obs.shape == (ROWS, 27) and obs.dtype == np.float32
    assert set(np.unique(obs)) <= {0.0, 1.0}
    planes = obs.reshape(ROWS, 3, 9)
    assert np.all(planes.sum(axis=1) == 1.0)          # every cell in exactly one plane
    assert np.array_equal(mask, planes[:, 0, :])      # legal = empty
    assert np.all(mask.sum(axis=1) >= 1)


def test_cells_are_uniform_over_three_states(batch):
    planes = batch["obs"].reshape(ROWS, 3, 9)
    freq = planes.mean(axis=(0, 2))
    # uniform over three states, slightly tilted towards empty by resampling full boards
    # (a full board has probability (2/3)^9 = 2.6 %)
    assert np.all(np.abs(freq - 1 / 3) < 0.02), freq
    assert freq[0] > freq[1] and freq[0] > freq[2]


def test_cells_round_trip(batch):
    c = cells_of(batch["obs"])
    assert set(np.unique(c)) <= {-1.0, 0.0, 1.0}
    assert np.array_equal(c == 0, batch["mask"] > 0)


def test_q_is_a_distribution_over_legal_cells(batch):
    q, mask = batch["q"], batch["mask"]
    assert np.all(q >= 0)
    assert np.all(q[mask == 0] == 0)
    assert np.allclose(q.sum(axis=1), 1.0, atol=1e-5)
    # Dirichlet(0.3) over n legal cells: E[q_i] = 1 / n, and the mass concentrates on few
    # cells (E[max q] is well above the uniform 1 / n)
    n = mask.sum(axis=1)
    rows9 = n == 9
    assert abs(float(q[rows9].mean()) - 1 / 9) < 1e-3
    assert float(q[rows9].max(axis=1).mean()) > 0.4


def test_old_logits_masked(batch):
    z, mask = batch["logits_old"], batch["mask"]
    assert np.all(z[mask == 0] == NEG_INF)
    legal = z[mask > 0]
    assert abs(float(legal.mean())) < 0.02 and abs(float(legal.std()) - 1.0) < 0.02


def test_critic_targets_are_five_step_returns(batch):
    t = batch["target"]
    assert t.shape == (ROWS, 1)
    disc = 0.99 ** np.arange(5)
    bound = disc.sum() + 0.99 ** 5
    assert np.all(np.abs(t) <= bound + 1e-5)
    assert abs(float(t.mean())) < 0.05
    # Var = sum_k 0.99^{2k} Var(r) + 0.99^10 Var(U[-1,1]), Var(r) = 2/3
    var = (0.99 ** (2 * np.arange(5))).sum() * (2 / 3) + 0.99 ** 10 / 3
    assert abs(float(t.var()) - var) < 0.05 * var


def test_glorot_weights_and_zero_biases():
    p = init_params(WORKLOADS["c3"], seed=0)
    for which, dims in (("actor", (27, 512, 512, 512, 9)), ("critic", (27, 512, 512, 512, 1))):
        for i, (w, b) in enumerate(p[which]):
            lim = np.sqrt(6.0 / (dims[i] + dims[i + 1]))
            assert w.shape == (dims[i], dims[i + 1]) and w.dtype == np.float32
            assert np.all(np.abs(w) <= lim) and float(np.abs(w).max()) > 0.95 * lim
            assert np.all(b == 0)
    # seeded: the same seed gives the same weights, another seed different ones
    q = init_params(WORKLOADS["c3"], seed=0)
    assert np.array_equal(p["actor"][1][0], q["actor"][1][0])
    assert not np.array_equal(p["actor"][1][0], init_params(WORKLOADS["c3"], seed=1)["actor"][1][0])


def test_per_sample_work():
    # forward + dW + dX (no dX for the input layer), 2 flops per multiply-add
    assert WORKLOADS["c0"].flops_per_sample() == 119040
    assert WORKLOADS["c1"].flops_per_sample() == 112896
    assert WORKLOADS["c2"].flops_per_sample() == 1643520
    assert WORKLOADS["c3"].flops_per_sample() == 6432768
    assert WORKLOADS["c4"].flops_per_sample() == 19040256
    assert WORKLOADS["c3"].input_bytes_per_sample() == 108 + 3 * 36 + 4
    assert WORKLOADS["c0"].param_count() == 21257 + 1   # + log_alpha
    assert WORKLOADS["c3"].param_count() == 1084426 + 1


def test_search_head_sync_shape_check():
    """The search models copy a network only into one of the same shape, and say which
    shape they were given (envs/tictactoe_actor.mojo:121-140)."""
    from spo_mojo_b200.networks import check_sync_shape
    check_sync_shape((27, 128, 128, 9), [27, 128, 128, 9], "actor being copied")
    with pytest.raises(ValueError, match=r"the actor being copied does not have the model's shape: 27x64x64x9"):
        check_sync_shape((27, 64, 64, 9), (27, 128, 128, 9), "actor being copied")
    with pytest.raises(ValueError, match="critic"):
        check_sync_shape((27, 128, 128, 128, 1), (27, 128, 128, 1), "critic")
