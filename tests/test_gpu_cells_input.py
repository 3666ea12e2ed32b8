"""The learner fed board cells (the observation encoding fused into the first layer's load
stage, the legal mask derived from the empty cells) gives bit-identical gradients, losses
and parameters to the learner fed the encoded observations and mask."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("engine", ["tensor", "cuda"])
@pytest.mark.parametrize("wl_name,rows", [("c2", 4096), ("c0", 256), ("c3", 1000)])
def test_cells_batch_equals_obs_batch(engine, wl_name, rows):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from spo_mojo_b200.learner import Learner
    from spo_mojo_b200.workloads import WORKLOADS, cells_of, init_params, make_batch
    wl = WORKLOADS[wl_name]
    params = init_params(wl, seed=1)
    batch = make_batch(wl, rows, seed=9)
    dev = {k: torch.from_numpy(v).cuda() for k, v in batch.items()}
    cells = {k: v for k, v in dev.items() if k not in ("obs", "mask")}
    cells["cells"] = torch.from_numpy(cells_of(batch["obs"])).cuda()
    out = []
    for b in (dev, cells):
        L = Learner.for_workload(wl, max_rows=rows, engine=engine)
        L.load(actor=params.get("actor"), critic=params.get("critic"), log_alpha=wl.log_alpha)
        for _ in range(2):
            L.step(b)
        torch.cuda.synchronize()
        assert L.device_status() == 0
        out.append((L.grads.clone(), L.params.clone()))
    assert torch.equal(out[0][0], out[1][0])
    assert torch.equal(out[0][1], out[1][1])


def test_encode_round_trip_on_host():
    from spo_mojo_b200.workloads import WORKLOADS, cells_of, make_batch
    from oracle import data_oracle as D
    b = make_batch(WORKLOADS["c2"], 512, seed=2)
    obs, mask = D.encode_obs(cells_of(b["obs"]))
    assert np.array_equal(obs, b["obs"]) and np.array_equal(mask, b["mask"])
