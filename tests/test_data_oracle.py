"""The data-format oracle (oracle/data_oracle.py) on CPU: the counter-based generator,
replay sampling/gather and the observation encoding, checked against the properties the
reference's own tests assert (tests/test_buffer.mojo, tests/test_rng.mojo) and against an
independent pure-Python restatement of the hash."""

import numpy as np
import pytest

from oracle import data_oracle as D


def _mix32_py(x):
    # ops/rng.mojo:43-52, one value at a time with Python integers
    x &= 0xFFFFFFFF
    x ^= x >> 16
    x = (x * 0x7FEB352D) & 0xFFFFFFFF
    x ^= x >> 15
    x = (x * 0x846CA68B) & 0xFFFFFFFF
    x ^= x >> 16
    return x


def test_mix32_matches_a_scalar_restatement():
    xs = [0, 1, 2, 3, 0x9E3779B9, 0xFFFFFFFF, 123456789] + list(range(1000, 1100))
    got = D.mix32(np.array(xs, dtype=np.uint64))
    assert [int(v) for v in got] == [_mix32_py(x) for x in xs]
    assert _mix32_py(0) == 0  # the finaliser maps 0 to 0


def test_rand_bits_cascade():
    for seed, stream, c in [(0, 0, 0), (123, 0, 5), (999, 7, 2**31 + 3)]:
        want = _mix32_py(seed ^ _mix32_py(stream ^ _mix32_py(c)))
        assert int(D.rand_bits(seed, stream, np.uint64(c))) == want


def test_sampling_is_deterministic_and_in_range():
    # tests/test_buffer.mojo:114-138: same seed -> same indices, another seed -> others
    a = D.sample_indices(20, 7, 123, 0)
    b = D.sample_indices(20, 7, 123, 0)
    c = D.sample_indices(20, 7, 999, 0)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert ((a >= 0) & (a < 7)).all()


def test_sampling_more_than_stored_covers_every_sequence():
    # tests/test_buffer.mojo:190-210: 32 draws from 3 sequences use all three
    idx = D.sample_indices(32, 3, 5, 0)
    assert set(idx.tolist()) == {0, 1, 2}


def test_empty_buffer_refuses_to_sample():
    with pytest.raises(ValueError):
        D.sample_indices(4, 0, 1, 0)


def test_ring_fifo_and_wraparound():
    # tests/test_buffer.mojo:46-79: slots 0, 1, 2 then back to 0; count saturates
    r = D.RingBuffer(3)
    assert [r.add() for _ in range(5)] == [0, 1, 2, 0, 1]
    assert r.count == 3 and r.write == 2


def test_gather_order_repeats_and_range():
    # tests/test_buffer.mojo:140-188
    field = np.arange(4 * 6, dtype=np.float32).reshape(4, 6)
    got = D.gather(field, [2, 0, 2, 3], count=4)
    assert np.array_equal(got, field[[2, 0, 2, 3]])
    with pytest.raises(IndexError):
        D.gather(field, [1, 4], count=4)


def test_encode_obs_planes_and_mask():
    cells = np.array([[1, -1, 0, 0, 1, 0, -1, 0, 0]], dtype=np.float32)
    obs, mask = D.encode_obs(cells)
    assert obs.shape == (1, 27)
    assert np.array_equal(obs[0, :9], [0, 0, 1, 1, 0, 1, 0, 1, 1])
    assert np.array_equal(obs[0, 9:18], [1, 0, 0, 0, 1, 0, 0, 0, 0])
    assert np.array_equal(obs[0, 18:], [0, 1, 0, 0, 0, 0, 1, 0, 0])
    assert np.array_equal(mask[0], obs[0, :9])
