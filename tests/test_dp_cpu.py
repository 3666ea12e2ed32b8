"""Data-parallel decomposition of the learner step on CPU ranks (gloo, world size 2).

Each rank takes its contiguous shard of the global batch, computes the gradient with
the loss scale 1/B_global (what spo_learner_backward does with grad_scale = 1/B), and
the ranks sum their flat gradient + statistics buffers with one all-reduce. The result
must equal the single-rank full-batch gradient, and the dual gradient computed after the
all-reduce from the summed KL statistic must equal the full-batch one. The arithmetic is
the oracle's (float64); the point is the sharding and scaling logic, not the kernels.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import spo_oracle as O
from spo_mojo_b200.workloads import Workload, NetSpec, make_batch, init_params

WL = Workload("dp", actor=NetSpec((27, 32, 32, 9)), critic=NetSpec((27, 32, 32, 1)), batch=64)


def _flat(batch, scale, params):
    x = batch["obs"]
    acts, z = O.mlp_forward(params["actor"], x)
    al = O.actor_loss(z, batch["mask"], batch["q"], batch["logits_old"], 0.0, 0.01, scale)
    ga = O.mlp_backward(params["actor"], x, acts, al["dz"])
    acts_c, v = O.mlp_forward(params["critic"], x)
    vl = O.value_loss(v, batch["target"], scale)
    gc = O.mlp_backward(params["critic"], x, acts_c, vl["dv"])
    parts = [t.ravel() for pair in ga + gc for t in pair]
    stats = np.array([al["loss"], al["kl_old_mean"], vl["loss"]])
    return np.concatenate(parts + [stats])


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        batch = make_batch(WL, WL.batch, seed=5)
        params = init_params(WL, seed=6)
        per = WL.batch // world
        shard = {k: v[rank * per:(rank + 1) * per] for k, v in batch.items()}
        local = torch.from_numpy(_flat(shard, 1.0 / WL.batch, params))
        dist.all_reduce(local)
        if rank == 0:
            out.put(local.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_gradients_sum_to_the_full_batch_gradient():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    batch = make_batch(WL, WL.batch, seed=5)
    want = _flat(batch, 1.0 / WL.batch, init_params(WL, seed=6))
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-14)
    # the dual gradient is formed after the reduction from the summed mean KL
    kl = got[-2]
    assert abs(O.sigmoid(0.0) * (0.01 - kl) - O.sigmoid(0.0) * (0.01 - want[-2])) < 1e-12


def _never_joining_peer(port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=0, world_size=2,
                                timeout=__import__("datetime").timedelta(seconds=3))
        out.put("joined")
    except Exception as e:  # the rendezvous gives up: the failure is reported, not hung
        out.put(type(e).__name__)


def test_missing_rank_fails_the_rendezvous_instead_of_hanging():
    """A rank that never joins: the host-side rendezvous (what bench.py and the DP
    learner build on) ends with an error within its timeout."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_never_joining_peer, args=(_free_port(), q))
    p.start()
    msg = q.get(timeout=120)
    p.join(timeout=30)
    assert msg != "joined"
