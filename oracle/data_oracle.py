"""CPU oracle of the data formats either side of the learner step. TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may import this module; the library never calls it and has no CPU
fallback.

Restates, in numpy integer and float arithmetic:

* the project's counter-based generator ``rand_bits`` (ops/rng.mojo:43-58) and the replay
  buffer's ``sample_indices`` / ``gather*`` (rl_utils/buffer.mojo:138-211), including the
  ring-buffer write pointer of ``add`` (rl_utils/buffer.mojo:100-131);
* the observation encoding and legal mask (envs/tictactoe.mojo:449-480, 577-597), in the
  three-plane [empty | agent | rival] form the learner's 27-wide input uses.

Pinning. The reference ships no golden vectors for these (its tests,
tests/test_buffer.mojo and tests/test_rng.mojo, check properties: FIFO order and
wraparound, fields that do not cross, determinism under a seed, order and repeats of a
gather, sampling more than stored). ``tests/test_data_oracle.py`` restates those
properties against this oracle, and pins ``mix32`` against values worked by hand from its
definition; parity of the GPU kernels with this oracle is bit-exact (integer work).
"""

import numpy as np

M32 = 0xFFFFFFFF


def mix32(x):
    """ops/rng.mojo:43-52 (the "lowbias32" finaliser): xor-shift 16, multiply, xor-shift
    15, multiply, xor-shift 16, in uint32 arithmetic. Vectorised over numpy arrays."""
    x = np.asarray(x, dtype=np.uint64) & M32
    x ^= x >> np.uint64(16)
    x = (x * np.uint64(0x7FEB352D)) & M32
    x ^= x >> np.uint64(15)
    x = (x * np.uint64(0x846CA68B)) & M32
    x ^= x >> np.uint64(16)
    return x


def rand_bits(seed, stream, counter):
    """ops/rng.mojo:55-58: mix32(seed ^ mix32(stream ^ mix32(counter)))."""
    c = mix32(counter)
    return mix32(np.uint64(seed) ^ mix32(np.uint64(stream) ^ c))


def sample_indices(n, count, seed, stream):
    """rl_utils/buffer.mojo:138-152: n indices in [0, count), with replacement."""
    if count == 0:
        raise ValueError("the buffer is empty: there is nothing to sample")
    bits = rand_bits(seed, stream, np.arange(n, dtype=np.uint64))
    return (bits % np.uint64(count)).astype(np.int32)


def gather(field, idx, count):
    """rl_utils/buffer.mojo:154-211: field [capacity, span...] -> [len(idx), span...] in
    the order of idx; an index outside [0, count) raises, as the reference does."""
    idx = np.asarray(idx)
    if ((idx < 0) | (idx >= count)).any():
        raise IndexError("sequence index out of range")
    return np.asarray(field)[idx]


class RingBuffer:
    """The write pointer and count of TrajectoryBuffer.add (rl_utils/buffer.mojo:100-131):
    sequence i goes to slot `write`, which wraps at capacity; count saturates."""

    def __init__(self, capacity):
        self.capacity, self.write, self.count = capacity, 0, 0

    def add(self):
        slot = self.write
        self.write = (self.write + 1) % self.capacity
        self.count = min(self.count + 1, self.capacity)
        return slot


def encode_obs(cells):
    """envs/tictactoe.mojo:449-480 and 577-597: cells [n, 9] coded +1 agent, -1 rival,
    0 empty -> obs [n, 27] = plane-major [empty | agent | rival] 0/1 planes, and the
    legal mask [n, 9] = the empty plane."""
    cells = np.asarray(cells, dtype=np.float32)
    obs = np.concatenate([(cells == 0), (cells == 1), (cells == -1)], axis=1).astype(np.float32)
    return obs, obs[:, :9].copy()
