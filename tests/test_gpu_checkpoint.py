"""Checkpoint / resume of the learner: the flat parameters, both Adam moments and Adam's
step saved after two steps and loaded into a fresh learner continue training exactly as
the uninterrupted learner does (bit for bit: the step is deterministic), on the one-launch
small step (c0) and the multi-launch tensor-core step (c2); a learner with other networks
or hyperparameters refuses the checkpoint."""

import numpy as np
import pytest
import torch

from spo_mojo_b200.workloads import WORKLOADS, init_params, make_batch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def dev(batch):
    return {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in batch.items()}


def fresh(wl, rows, **kw):
    from spo_mojo_b200.learner import Learner
    L = Learner.for_workload(wl, max_rows=rows, **kw)
    p = init_params(wl, seed=0)
    L.load(actor=p.get("actor"), critic=p.get("critic"), log_alpha=wl.log_alpha)
    return L


@pytest.mark.parametrize("name,rows", [("c0", 256), ("c2", 4096)])
def test_resume_continues_exactly(tmp_path, name, rows):
    wl = WORKLOADS[name]
    batches = [dev(make_batch(wl, rows, seed=20 + i)) for i in range(4)]
    A = fresh(wl, rows)
    for b in batches[:2]:
        A.step(b)
    A.save_checkpoint(str(tmp_path))
    B = fresh(wl, rows)
    B.load_checkpoint(str(tmp_path))
    assert int(B.step_counter.item()) == 2
    for b in batches[2:]:
        A.step(b)
        B.step(b)
    torch.cuda.synchronize()
    assert torch.equal(A.params, B.params)
    assert torch.equal(A.adam_m, B.adam_m) and torch.equal(A.adam_v, B.adam_v)
    assert int(A.step_counter.item()) == int(B.step_counter.item()) == 4


def test_mismatched_learner_refuses_the_checkpoint(tmp_path):
    from spo_mojo_b200.learner import Learner
    wl = WORKLOADS["c0"]
    A = fresh(wl, 256)
    A.save_checkpoint(str(tmp_path))
    other = fresh(WORKLOADS["c1"], 256)
    with pytest.raises(ValueError, match="dims"):
        other.load_checkpoint(str(tmp_path))
    faster = Learner(actor_dims=wl.actor.dims, max_rows=256, lr_actor=10 * wl.lr, lr_critic=wl.lr)
    with pytest.raises(ValueError, match="lr_actor"):
        faster.load_checkpoint(str(tmp_path))
