"""The packed host-batch layout (no GPU): every field a 256-byte-aligned view of one
buffer, holding exactly the field's values."""

import numpy as np
import torch

from spo_mojo_b200 import learner as Lm


def test_packed_layout_views_alias_one_buffer():
    rng = np.random.default_rng(0)
    arrays = {"obs": rng.random((37, 27), dtype=np.float32), "mask": np.ones((37, 9), np.float32),
              "q": rng.random((37, 9), dtype=np.float32), "target": rng.random(37, dtype=np.float32)}
    like = {k: torch.as_tensor(v) for k, v in arrays.items()}
    offs, total = Lm._packed_layout(like)
    flat = torch.zeros(total, dtype=torch.uint8)
    views = Lm._packed_views(flat, like, offs)
    for k, v in like.items():
        views[k].copy_(v)
    end = 0
    for k, v in like.items():
        assert offs[k] % 256 == 0 and offs[k] >= end
        assert views[k].data_ptr() - flat.data_ptr() == offs[k]
        assert torch.equal(views[k], v)
        end = offs[k] + v.numel() * v.element_size()
    assert end <= total
