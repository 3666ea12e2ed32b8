"""Data parallelism through libspo_cuda's NCCL communicator (GPU).

* A peer that never joins: spo_comm_init must give up after SPO_COMM_TIMEOUT_MS with
  SPO_ERR_TIMEOUT (the non-blocking init is aborted) instead of hanging. One GPU; no
  kernel runs.
* 2, 4 and 8 GPUs: each rank runs the learner backward on its 1/N of the batch with
  grad_scale = 1/B, one all-reduce of the flat gradient + statistics buffer, then apply;
  the result matches one GPU on the full batch. Each size is skipped when the box has
  fewer GPUs.
Child processes are spawned; NVLS is off (NCCL_NVLS_ENABLE=0) for these tests.
"""

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _join_alone(q):
    os.environ["SPO_COMM_TIMEOUT_MS"] = "3000"
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import time
    from spo_mojo_b200 import ffi
    from spo_mojo_b200.learner import Comm
    torch.cuda.set_device(0)
    uid = Comm.unique_id()
    t0 = time.time()
    try:
        Comm(uid, 2, 0)
        q.put(("joined", time.time() - t0))
    except ffi.SpoError as e:
        q.put((e.code, time.time() - t0))


def test_comm_init_gives_up_when_a_peer_never_joins():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_join_alone, args=(q,))
    p.start()
    code, elapsed = q.get(timeout=180)
    p.join(timeout=60)
    assert code in (-8, -6), code          # SPO_ERR_TIMEOUT (or NCCL's own error)
    assert elapsed < 60


def _rank(rank, world, q_uid, q_out, rows):
    try:
        _rank_body(rank, world, q_uid, q_out, rows)
    except Exception:                        # report instead of leaving the parent waiting
        import traceback
        q_out.put(("failed", rank, traceback.format_exc()))
        raise


def _rank_body(rank, world, q_uid, q_out, rows):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from spo_mojo_b200.learner import Comm, Learner
    from spo_mojo_b200.workloads import WORKLOADS, init_params, make_batch
    torch.cuda.set_device(rank)
    wl = WORKLOADS["c2"]
    params = init_params(wl, seed=0)
    batch = make_batch(wl, rows, seed=21)
    per = rows // world
    shard = {k: torch.from_numpy(v[rank * per:(rank + 1) * per]).cuda() for k, v in batch.items()}
    uid = Comm.unique_id() if rank == 0 else None
    if rank == 0:
        for _ in range(world - 1):
            q_uid.put(uid)
    else:
        uid = q_uid.get(timeout=120)
    comm = Comm(uid, world, rank)
    L = Learner.for_workload(wl, max_rows=per)
    L.load(actor=params["actor"], critic=params["critic"])
    L.backward(shard, grad_scale=1.0 / rows)
    comm.allreduce_(L.grads)
    L.apply()
    torch.cuda.synchronize()
    out = (L.grads.cpu().numpy(), L.params.cpu().numpy(), L.device_status())
    comm.close()
    if rank == 0:
        full = Learner.for_workload(wl, max_rows=rows)
        full.load(actor=params["actor"], critic=params["critic"])
        full.step({k: torch.from_numpy(v).cuda() for k, v in batch.items()})
        torch.cuda.synchronize()
        q_out.put(out + (full.grads.cpu().numpy(), full.params.cpu().numpy(), dict(
            a=(full.layout.actor_offset, full.layout.actor_size),
            c=(full.layout.critic_offset, full.layout.critic_size),
            s=full.layout.stats_offset)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_data_parallel_matches_one_gpu_on_the_full_batch(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q_uid, q_out = ctx.Queue(), ctx.Queue()
    rows = 8192
    procs = [ctx.Process(target=_rank, args=(r, world, q_uid, q_out, rows)) for r in range(world)]
    for p in procs:
        p.start()
    got = q_out.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
    assert not isinstance(got[0], str), f"rank {got[1]}:\n{got[2]}"
    g2, p2, status, g1, p1, lay = got
    assert all(p.exitcode == 0 for p in procs)
    assert status == 0
    for off, size in (lay["a"], lay["c"]):
        a, b = g2[off:off + size], g1[off:off + size]
        assert np.max(np.abs(a - b)) <= 1e-5 * np.max(np.abs(b))
        # Adam's first step is lr * g / (|g| + eps): compare every element whose update the
        # gradient determines (both zero, or clear of the summation-order difference d
        # between the two reductions by a factor 10 and large enough that the step's
        # sensitivity lr * eps * d / g^2 is below 5e-7); the others, within 2 lr
        d = float(np.max(np.abs(a - b)))
        clear = ((a == 0) & (b == 0)) | ((np.abs(b) >= 10 * d) & ((np.abs(b) - d) ** 2 * 5e-7 >= 3e-4 * 1e-8 * d))
        np.testing.assert_allclose(p2[off:off + size][clear], p1[off:off + size][clear],
                                   rtol=1e-4, atol=1e-6)
        assert np.all(np.abs(p2[off:off + size][~clear] - p1[off:off + size][~clear]) <= 2 * 3e-4 * 1.001 + 1e-6)
        assert (~clear).sum() <= 0.05 * size
    s = lay["s"]
    np.testing.assert_allclose(g2[s:s + 6], g1[s:s + 6], rtol=1e-5)
