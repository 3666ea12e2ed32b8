"""The replay buffer of rl_utils/buffer.mojo (TrajectoryBuffer) held in HBM.

The reference keeps the buffer in host lists and uploads the gathered batch at every
update (rl_utils/buffer.mojo:1-13 calls moving it to the device "an improvement"). Here
the fields live in device memory; `add` copies one sequence into its ring slot, and
`sample_indices` / `gather*` run as libspo_cuda kernels (spo_replay_sample,
spo_replay_gather), so a learner batch is assembled without a host round trip.

Names, argument meaning and errors follow the reference class: capacity, t_len, obs_dim,
num_actions; add(obs, reward, done, truncated, bootstrap_obs, q) validates sizes and
overwrites the oldest sequence once full; sample_indices(n, seed, stream) draws with
replacement from the stored sequences with the project's counter-based generator and
raises on an empty buffer; gather / gather_steps / gather_bootstrap / gather_q return the
sequences in the order of the indices, repeats allowed, and raise on an index outside the
stored range.
"""

import ctypes

import torch

from . import ffi


def _stream(stream, device):
    return (stream or torch.cuda.current_stream(device)).cuda_stream


class DeviceTrajectoryBuffer:
    """Ring buffer of fixed-length sequences in device memory (float32 fields)."""

    def __init__(self, capacity, t_len, obs_dim, num_actions=0, device=None):
        if capacity < 1 or t_len < 1 or obs_dim < 1 or num_actions < 0:
            raise ValueError("capacity, t_len and obs_dim must be positive")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.capacity, self.t_len, self.obs_dim, self.num_actions = capacity, t_len, obs_dim, num_actions
        self.write = 0
        self.count = 0
        z = lambda *shape: torch.zeros(shape, dtype=torch.float32, device=self.device)  # noqa: E731
        self.obs = z(capacity, t_len, obs_dim)
        self.bootstrap_obs = z(capacity, t_len, obs_dim)
        self.reward = z(capacity, t_len)
        self.done = z(capacity, t_len)
        self.truncated = z(capacity, t_len)
        self.q = z(capacity, t_len, num_actions) if num_actions > 0 else None
        self._err = torch.zeros(1, dtype=torch.int32, device=self.device)

    def size(self):
        return self.count

    def is_full(self):
        return self.count >= self.capacity

    def add(self, obs, reward, done, truncated, bootstrap_obs, q=None):
        """Store ONE sequence of t_len steps (host or device arrays); once full, the oldest
        is overwritten."""
        T, D, A = self.t_len, self.obs_dim, self.num_actions
        f = lambda x: torch.as_tensor(x, dtype=torch.float32).reshape(-1)  # noqa: E731
        obs, bootstrap_obs = f(obs), f(bootstrap_obs)
        reward, done, truncated = f(reward), f(done), f(truncated)
        if reward.numel() != T or done.numel() != T or truncated.numel() != T:
            raise ValueError(f"the sequence should have {T} steps")
        if obs.numel() != T * D or bootstrap_obs.numel() != T * D:
            raise ValueError("the observations should be t_len * obs_dim")
        qn = 0 if q is None else f(q).numel()
        if qn != T * A:
            raise ValueError(f"q should have t_len * num_actions = {T * A} values, and has {qn}")
        slot = self.write
        self.obs[slot].copy_(obs.view(T, D), non_blocking=True)
        self.bootstrap_obs[slot].copy_(bootstrap_obs.view(T, D), non_blocking=True)
        self.reward[slot].copy_(reward, non_blocking=True)
        self.done[slot].copy_(done, non_blocking=True)
        self.truncated[slot].copy_(truncated, non_blocking=True)
        if A:
            self.q[slot].copy_(f(q).view(T, A), non_blocking=True)
        self.write = (self.write + 1) % self.capacity
        if self.count < self.capacity:
            self.count += 1

    def sample_indices(self, n, seed, stream_id, stream=None):
        """`n` indices of stored sequences, with replacement (int32 device tensor)."""
        if self.count == 0:
            raise ffi.SpoError(-1, "the buffer is empty: there is nothing to sample")
        idx = torch.empty(int(n), dtype=torch.int32, device=self.device)
        ffi.call("spo_replay_sample", _stream(stream, self.device), idx.data_ptr(), int(n), self.count,
                 ctypes.c_uint32(seed & 0xFFFFFFFF), ctypes.c_uint32(stream_id & 0xFFFFFFFF))
        return idx

    def _gather(self, field, idx, stream=None, check=True):
        idx = torch.as_tensor(idx, dtype=torch.int32, device=self.device).contiguous()
        n = idx.numel()
        span = field[0].numel()
        out = torch.empty((n,) + tuple(field.shape[1:]), dtype=torch.float32, device=self.device)
        self._err.zero_()
        ffi.call("spo_replay_gather", _stream(stream, self.device), out.data_ptr(), field.data_ptr(),
                 idx.data_ptr(), n, span, self.count, self._err.data_ptr())
        if check and int(self._err.item()) != 0:
            raise IndexError("sequence index out of range")
        return out

    def gather(self, indices, stream=None, check=True):
        """Those sequences' observations: [len(indices), t_len, obs_dim]."""
        return self._gather(self.obs, indices, stream, check)

    def gather_steps(self, indices, which, stream=None, check=True):
        """One per-step field: 0 = reward, 1 = done, 2 = truncated -> [len(indices), t_len]."""
        field = (self.reward, self.done, self.truncated)[which]
        return self._gather(field, indices, stream, check)

    def gather_bootstrap(self, indices, stream=None, check=True):
        return self._gather(self.bootstrap_obs, indices, stream, check)

    def gather_q(self, indices, stream=None, check=True):
        if self.num_actions == 0:
            raise ValueError("this buffer was created without q (num_actions = 0)")
        return self._gather(self.q, indices, stream, check)


def encode_obs(cells, stream=None, with_mask=True):
    """Board cells [n, 9] (+1 agent, -1 rival, 0 empty; float32 device tensor) -> obs
    [n, 27] plane-major [empty | agent | rival] and the legal mask [n, 9]
    (envs/tictactoe.mojo:449-480, 577-597)."""
    cells = cells.contiguous()
    n = cells.shape[0]
    obs = torch.empty(n, 27, dtype=torch.float32, device=cells.device)
    mask = torch.empty(n, 9, dtype=torch.float32, device=cells.device) if with_mask else None
    ffi.call("spo_encode_obs", _stream(stream, cells.device), obs.data_ptr(),
             mask.data_ptr() if mask is not None else None, cells.data_ptr(), n)
    return obs, mask
