"""A learner step captured as a CUDA graph (Learner.capture_step) and replayed gives the
same parameters, moments and statistics as the same number of eager steps (bit-exact: the
same kernels in the same order)."""

import warnings

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


def test_first_small_step_under_capture_is_refused_then_captures():
    """The one-launch step's first call on a parameter buffer copies the weights' tensor
    maps into the workspace (stream-ordered); recorded by a stream capture, that call is
    refused before anything is enqueued. After one eager step the capture records, and its
    replays match eager steps bit for bit."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from spo_mojo_b200 import ffi
    from spo_mojo_b200.learner import Learner
    from spo_mojo_b200.workloads import WORKLOADS, init_params, make_batch
    wl = WORKLOADS["c0"]
    params = init_params(wl, seed=5)
    batch = {k: torch.from_numpy(v).cuda() for k, v in make_batch(wl, wl.batch, seed=6).items()}

    def fresh():
        L = Learner.for_workload(wl, max_rows=wl.batch)
        L.load(actor=params["actor"], log_alpha=wl.log_alpha)
        return L

    L, twin = fresh(), fresh()
    g = torch.cuda.CUDAGraph()
    with pytest.raises(ffi.SpoError) as err, warnings.catch_warnings():
        warnings.simplefilter("ignore")   # the refused capture leaves an empty graph
        with torch.cuda.graph(g):
            L.step(batch)
    assert ffi.ERRORS[err.value.code] == "SPO_ERR_UNSUPPORTED"
    torch.cuda.synchronize()
    assert torch.equal(L.params, twin.params)   # nothing ran
    graph = L.capture_step(batch, warmup=1)
    for _ in range(2):
        graph.replay()
    for _ in range(3):
        twin.step(batch)
    torch.cuda.synchronize()
    assert torch.equal(L.params, twin.params)
    assert torch.equal(L.adam_m, twin.adam_m) and torch.equal(L.adam_v, twin.adam_v)
    assert L.device_status() == 0 and twin.device_status() == 0
