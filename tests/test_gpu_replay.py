"""Device replay buffer and observation encoding (libspo_cuda spo_replay_sample,
spo_replay_gather, spo_encode_obs through spo_mojo_b200.replay) against the oracle:
bit-exact, as the work is integer indexing and copies."""

import numpy as np
import pytest
import torch

from oracle import data_oracle as D

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _buffer(capacity=5, t_len=4, obs_dim=27, num_actions=9, adds=7, seed=0):
    from spo_mojo_b200.replay import DeviceTrajectoryBuffer
    rng = np.random.default_rng(seed)
    buf = DeviceTrajectoryBuffer(capacity, t_len, obs_dim, num_actions)
    host = {k: np.zeros((capacity,) + s, np.float32) for k, s in
            (("obs", (t_len, obs_dim)), ("boot", (t_len, obs_dim)), ("reward", (t_len,)),
             ("done", (t_len,)), ("trunc", (t_len,)), ("q", (t_len, num_actions)))}
    ring = D.RingBuffer(capacity)
    for _ in range(adds):
        seq = {k: rng.standard_normal(v.shape[1:]).astype(np.float32) for k, v in host.items()}
        buf.add(seq["obs"], seq["reward"], seq["done"], seq["trunc"], seq["boot"], seq["q"])
        slot = ring.add()
        for k in host:
            host[k][slot] = seq[k]
    assert (buf.write, buf.count) == (ring.write, ring.count)
    return buf, host, ring


@pytest.mark.parametrize("n,count,seed,stream", [(1, 1, 0, 0), (20, 7, 123, 0), (4096, 1000, 999, 3),
                                                  (1 << 20, 65537, 2**31 + 5, 0xFFFFFFFF)])
def test_sample_indices_match_the_oracle(n, count, seed, stream):
    from spo_mojo_b200 import ffi
    idx = torch.empty(n, dtype=torch.int32, device="cuda")
    ffi.call("spo_replay_sample", None, idx.data_ptr(), n, count, seed, stream)
    torch.cuda.synchronize()
    assert np.array_equal(idx.cpu().numpy(), D.sample_indices(n, count, seed, stream))


def test_gathers_match_the_oracle_in_order_with_repeats():
    buf, host, ring = _buffer()
    idx = buf.sample_indices(64, 77, 1)
    want_idx = D.sample_indices(64, ring.count, 77, 1)
    assert np.array_equal(idx.cpu().numpy(), want_idx)
    fixed = [4, 0, 4, 2]
    for ids in (idx, fixed):
        ids_np = np.asarray(ids.cpu() if torch.is_tensor(ids) else ids)
        assert np.array_equal(buf.gather(ids).cpu().numpy(), D.gather(host["obs"], ids_np, ring.count))
        assert np.array_equal(buf.gather_bootstrap(ids).cpu().numpy(), D.gather(host["boot"], ids_np, ring.count))
        for which, k in enumerate(("reward", "done", "trunc")):
            assert np.array_equal(buf.gather_steps(ids, which).cpu().numpy(), D.gather(host[k], ids_np, ring.count))
        assert np.array_equal(buf.gather_q(ids).cpu().numpy(), D.gather(host["q"], ids_np, ring.count))


def test_out_of_range_and_empty_are_errors():
    from spo_mojo_b200 import ffi
    from spo_mojo_b200.replay import DeviceTrajectoryBuffer
    buf, host, ring = _buffer(capacity=5, adds=3)
    with pytest.raises(IndexError):
        buf.gather([0, 3])          # slot 3 was never written (count = 3)
    out = buf.gather([0, 3], check=False)
    assert torch.all(out[1] == 0) and torch.equal(out[0].cpu(), torch.from_numpy(host["obs"][0]))
    empty = DeviceTrajectoryBuffer(4, 2, 27)
    with pytest.raises(ffi.SpoError):
        empty.sample_indices(3, 1, 0)
    with pytest.raises(ValueError):
        buf.add(np.zeros(5), np.zeros(4), np.zeros(4), np.zeros(4), np.zeros(4 * 27), np.zeros(36))


def test_wraparound_overwrites_the_oldest():
    buf, host, ring = _buffer(capacity=3, adds=8)
    assert ring.count == 3
    got = buf.gather([0, 1, 2]).cpu().numpy()
    assert np.array_equal(got, host["obs"])


def test_encode_obs_matches_the_oracle():
    from spo_mojo_b200.replay import encode_obs
    rng = np.random.default_rng(4)
    cells = rng.integers(-1, 2, size=(10007, 9)).astype(np.float32)
    obs, mask = encode_obs(torch.from_numpy(cells).cuda())
    o, m = D.encode_obs(cells)
    assert np.array_equal(obs.cpu().numpy(), o) and np.array_equal(mask.cpu().numpy(), m)
