"""A learner step captured as a CUDA graph (Learner.capture_step) and replayed gives the
same parameters, moments and statistics as the same number of eager steps (bit-exact: the
same kernels in the same order)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("engine", ["tensor", "cuda"])
def test_graph_replays_equal_eager_steps(engine):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from spo_mojo_b200.learner import Learner
    from spo_mojo_b200.workloads import WORKLOADS, init_params, make_batch
    wl = WORKLOADS["c2"]
    rows = 4096
    params = init_params(wl, seed=2)
    batch = {k: torch.from_numpy(v).cuda() for k, v in make_batch(wl, rows, seed=4).items()}

    def fresh():
        L = Learner.for_workload(wl, max_rows=rows, engine=engine)
        L.load(actor=params["actor"], critic=params["critic"], log_alpha=wl.log_alpha)
        return L

    eager = fresh()
    for _ in range(4):
        eager.step(batch)
    g_learner = fresh()
    graph = g_learner.capture_step(batch, warmup=1)   # warm-up step counts: 1 eager + 3 replays
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(g_learner.params, eager.params)
    assert torch.equal(g_learner.adam_m, eager.adam_m) and torch.equal(g_learner.adam_v, eager.adam_v)
    assert torch.equal(g_learner.step_counter, eager.step_counter)
    assert torch.equal(g_learner.stats_tensor(), eager.stats_tensor())
    assert g_learner.device_status() == 0
