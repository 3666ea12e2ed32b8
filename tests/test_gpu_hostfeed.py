"""HostFeed: learner steps fed from pinned host batches through two device buffers (the
next batch's upload overlapping the current step) give exactly the parameters of the same
steps run on device-resident batches."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_overlapped_uploads_match_device_resident_steps():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from spo_mojo_b200.learner import HostFeed, Learner
    from spo_mojo_b200.workloads import WORKLOADS, init_params, make_batch
    wl = WORKLOADS["c2"]
    rows, steps = 4096, 4
    params = init_params(wl, seed=3)
    hosts = [{k: torch.from_numpy(v).pin_memory() for k, v in make_batch(wl, rows, seed=50 + i).items()}
             for i in range(steps)]

    ref = Learner.for_workload(wl, max_rows=rows)
    ref.load(actor=params["actor"], critic=params["critic"])
    for h in hosts:
        ref.step({k: v.cuda() for k, v in h.items()})
    torch.cuda.synchronize()

    L = Learner.for_workload(wl, max_rows=rows)
    L.load(actor=params["actor"], critic=params["critic"])
    stream = torch.cuda.Stream()
    feed = HostFeed(hosts[0], L.device, stream)
    with torch.cuda.stream(stream):
        j = feed.upload(hosts[0])
        for i in range(steps):
            b = feed.take(j)
            nxt = feed.upload(hosts[i + 1]) if i + 1 < steps else None
            L.step(b, stream=stream)
            feed.release(j)
            j = nxt
    torch.cuda.synchronize()
    assert torch.equal(L.params, ref.params)
    assert torch.equal(L.adam_v, ref.adam_v)
    assert L.device_status() == 0


def test_packed_host_batch_uploads_in_one_copy():
    """A PackedHostBatch (every field a view of one pinned buffer) is uploaded with one copy
    into the feed's packed device buffer; the fields arrive intact and the steps match the
    device-resident ones."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from spo_mojo_b200.learner import HostFeed, Learner, PackedHostBatch
    from spo_mojo_b200.workloads import WORKLOADS, init_params, make_batch
    wl = WORKLOADS["c0"]
    rows = wl.batch
    params = init_params(wl, seed=3)
    arrays = make_batch(wl, rows, seed=9)
    host = PackedHostBatch.of(arrays)
    ref = Learner.for_workload(wl, max_rows=rows)
    ref.load(actor=params["actor"])
    ref.step({k: torch.from_numpy(v).cuda() for k, v in arrays.items()})

    L = Learner.for_workload(wl, max_rows=rows)
    L.load(actor=params["actor"])
    stream = torch.cuda.Stream()
    feed = HostFeed(host, L.device, stream)
    with torch.cuda.stream(stream):
        n = feed.copy_into(0, host)
        L.step(feed.bufs[0], stream=stream)
    torch.cuda.synchronize()
    assert n == host.flat.numel()
    for k, v in arrays.items():
        assert torch.equal(feed.bufs[0][k].cpu(), torch.from_numpy(v))
    assert torch.equal(L.params, ref.params)
