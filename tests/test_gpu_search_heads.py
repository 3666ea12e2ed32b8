"""The search models' network part on the GPU: TicTacToeActorHead / TicTacToeCriticHead
(the batched inference forward of envs/tictactoe_actor.mojo:108-191 and
envs/tictactoe_critic.mojo:145-192) after sync_from / sync_critic_from, at the search's
P = envs x particles = 4,096 boards (demos/train_spo.mojo:61,75) and at ragged counts,
against the oracle: the board encoding (oracle/data_oracle.py), the MLP forward and the
masking. Tolerances are the reference's actor and critic forward tests
(tests/test_actor.mojo:27: 2e-5 on logits; tests/test_critic_mlp.mojo:83-90: 3e-5 sqrt(H)
on V); masked logits must be exactly -FLT_MAX. Also the C++ mirror's golden program (the
reference's actor-backward goldens through include/spo_networks.hpp) on the GPU."""

import math
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

from oracle import data_oracle as D
from oracle import spo_oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
HIDDEN = 128
MAX_P = 4096


@pytest.fixture(scope="module")
def N():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from spo_mojo_b200 import networks
    return networks


@pytest.fixture(scope="module")
def ctx(N):
    return N.DeviceContext(0)


def _glorot(dims, rng):
    out = []
    for i in range(len(dims) - 1):
        lim = math.sqrt(6.0 / (dims[i] + dims[i + 1]))
        out.append((rng.uniform(-lim, lim, (dims[i], dims[i + 1])).astype(np.float32),
                    rng.uniform(-0.1, 0.1, dims[i + 1]).astype(np.float32)))
    return out


def _boards(rng, n):
    cells = rng.integers(-1, 2, (n, 9)).astype(np.float32)
    full = ~(cells == 0).any(axis=1)
    cells[full, rng.integers(0, 9, int(full.sum()))] = 0.0     # at least one legal move
    return cells


@pytest.fixture(scope="module")
def trained(N, ctx):
    """A 'trained' actor and critic (random weights and biases) the heads sync from."""
    rng = np.random.default_rng(42)
    a_dims = (27, HIDDEN, HIDDEN, 9)
    c_dims = (27, HIDDEN, HIDDEN, 1)
    pa, pc = _glorot(a_dims, rng), _glorot(c_dims, rng)
    src_a, src_c = N.MLPParams(ctx, a_dims), N.MLPParams(ctx, c_dims)
    src_a.load(pa)
    src_c.load(pc)
    return src_a, src_c, pa, pc


@pytest.mark.parametrize("p", [MAX_P, 1000, 1])
def test_actor_head_eval_root_matches_oracle(N, ctx, trained, p):
    src_a, src_c, pa, pc = trained
    head = N.TicTacToeActorHead(ctx, MAX_P, HIDDEN)
    head.sync_from(ctx, src_a)
    head.sync_critic_from(ctx, src_c)
    cells = _boards(np.random.default_rng(p), p)
    logits = torch.full((MAX_P * 9,), 7.0, device="cuda")
    value = torch.full((MAX_P,), 7.0, device="cuda")
    head.eval_root(ctx, torch.from_numpy(cells).cuda(), logits, value, p)
    ctx.synchronize()
    obs, mask = D.encode_obs(cells)
    _, z = O.mlp_forward(pa, obs)
    want = O.masked_logits(z, mask)
    got = logits[:p * 9].cpu().numpy().reshape(p, 9)
    legal = mask != 0
    assert np.max(np.abs(got[legal] - want[legal])) <= 2e-5
    assert np.all(got[~legal] == np.float32(O.NEG_INF))
    assert np.all(logits[p * 9:].cpu().numpy() == 7.0)        # nothing past the m boards
    _, v = O.mlp_forward(pc, obs)
    assert np.max(np.abs(value[:p].cpu().numpy() - v[:, 0])) <= 3e-5 * math.sqrt(HIDDEN)
    assert np.all(value[p:].cpu().numpy() == 7.0)


@pytest.mark.parametrize("p", [MAX_P, 777])
def test_critic_head_value_matches_oracle(N, ctx, trained, p):
    _, src_c, _, pc = trained
    head = N.TicTacToeCriticHead(ctx, MAX_P, HIDDEN)
    head.sync_from(ctx, src_c)
    cells = _boards(np.random.default_rng(100 + p), p)
    value = torch.empty(p, device="cuda")
    head.value(ctx, torch.from_numpy(cells).cuda(), value, p)
    ctx.synchronize()
    obs, _ = D.encode_obs(cells)
    _, v = O.mlp_forward(pc, obs)
    assert np.max(np.abs(value.cpu().numpy() - v[:, 0])) <= 3e-5 * math.sqrt(HIDDEN)


def test_heads_refuse_other_shapes_and_capacity(N, ctx, trained):
    src_a, src_c, _, _ = trained
    head = N.TicTacToeActorHead(ctx, 64, HIDDEN)
    with pytest.raises(ValueError, match="shape"):
        head.sync_from(ctx, src_c)                   # a critic is not an actor
    wide = N.MLPParams(ctx, (27, 2 * HIDDEN, 2 * HIDDEN, 9))
    with pytest.raises(ValueError, match="shape"):
        head.sync_from(ctx, wide)
    cells = torch.zeros(65 * 9, device="cuda")
    with pytest.raises(ValueError, match="reserved for 64"):
        head.eval_root(ctx, cells, torch.empty(65 * 9, device="cuda"), torch.empty(65, device="cuda"), 65)


def test_sync_then_retrain_does_not_alias(N, ctx, trained):
    """sync_from copies: changing the trained weights afterwards leaves the model's copy."""
    src_a, _, pa, _ = trained
    head = N.TicTacToeActorHead(ctx, 16, HIDDEN)
    head.sync_from(ctx, src_a)
    keep = head.params.flat.clone()
    src_a.flat.add_(1.0)
    ctx.synchronize()
    assert torch.equal(head.params.flat, keep)
    src_a.flat.sub_(1.0)
    ctx.synchronize()


@pytest.mark.parametrize("case,batch,hidden", [("bw_small", 5, 32), ("bw_big", 40, 64)])
def test_cpp_mirror_golden_program(tmp_path, case, batch, hidden):
    """tests/cpp/networks_golden.cpp: the reference's actor-backward goldens through the C++
    mirror (actor_probs, actor_log_probs, cross_entropy_rows, actor_backward) at the
    reference test's tolerances."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from spo_mojo_b200 import ffi
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    out = str(tmp_path / "networks_golden")
    libdir = os.path.dirname(ffi.LIB_PATH)
    cmd = [cxx, "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
           os.path.join(ROOT, "tests", "cpp", "networks_golden.cpp"), "-o", out,
           "-L", libdir, "-lspo_cuda", "-Wl,-rpath," + libdir,
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.join(CUDA, "lib64")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    gold = os.path.join(ROOT, "tests", "golden", "ref")
    r = subprocess.run([out, gold, case, str(batch), str(hidden)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
