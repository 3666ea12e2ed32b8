"""Learner-step workloads, the flat parameter layout, and seeded synthetic inputs.

Five workloads are defined (the learner-step configurations this library is
measured on):

  c0  actor 27-128-128-9, batch 256 (the reference's own scale)
  c1  critic 27-128-128-1, batch 4,096
  c2  actor + critic 27-256-256-256-{9,1}, batch 65,536, with the log_alpha dual
  c3  actor + critic 27-512-512-512-{9,1}, global batch 1,048,576 (data parallel)
  c4  actor 27-1024-1024-1024-1024-9, batch 262,144

Inputs are synthetic and seeded (numpy default_rng), with the shapes and value
distributions of the learner's real inputs:
  * tic-tac-toe boards, each of the 9 cells uniform over {empty, X, O}, encoded as
    three 0/1 planes [empty | X | O] (plane-major, as the reference's obs encoder
    envs/tictactoe.mojo:449-480 lays out its planes), rows with no empty cell
    resampled (tests/golden/gen/gen_actor.py:64-76 does the same);
  * legal mask = the empty plane;
  * q ~ Dirichlet(0.3) over the legal cells, 0 elsewhere;
  * pi_old logits ~ N(0, 1), masked with the most negative finite float32;
  * critic targets = sum_{k<5} 0.99^k r_k + 0.99^5 v_boot, r uniform on {-1, 0, 1},
    v_boot ~ U[-1, 1];
  * weights Glorot-uniform (limit sqrt(6 / (fan_in + fan_out))), biases zero.

Flat layout. Each network's tensors live in ONE flat float32 buffer in the
reference's order w1, b1, w2, b2, ... (W stored [in, out] row-major,
networks/linear.mojo:7-11), each tensor starting on a 64-float (256-byte) boundary
so that every weight tile can be read with 16-byte vector loads and TMA. The pad
floats are zero and stay zero under Adam (zero gradient, zero moments). The same
layout is computed by ``spo_mlp_param_layout`` in the C library.
"""

from dataclasses import dataclass, field

import numpy as np

ALIGN_FLOATS = 64
OBS_DIM = 27
NUM_ACTIONS = 9
NEG_INF = np.float32(np.finfo(np.float32).min)


def _align(n):
    return (n + ALIGN_FLOATS - 1) // ALIGN_FLOATS * ALIGN_FLOATS


@dataclass(frozen=True)
class NetSpec:
    """Dimensions d0 .. dL of an MLP with L Linear layers (ReLU between them)."""
    dims: tuple

    @property
    def num_layers(self):
        return len(self.dims) - 1

    def offsets(self):
        """[(w_offset, b_offset)] per layer, and the padded total, in floats."""
        off = 0
        out = []
        for i in range(self.num_layers):
            w = off
            off = _align(off + self.dims[i] * self.dims[i + 1])
            b = off
            off = _align(off + self.dims[i + 1])
            out.append((w, b))
        return out, off

    @property
    def padded_size(self):
        return self.offsets()[1]

    @property
    def param_count(self):
        return sum(self.dims[i] * self.dims[i + 1] + self.dims[i + 1]
                   for i in range(self.num_layers))

    def macs_per_sample(self):
        """Multiply-accumulates per sample: forward + dW + dX (no dX for layer 1)."""
        fwd = sum(self.dims[i] * self.dims[i + 1] for i in range(self.num_layers))
        dx = fwd - self.dims[0] * self.dims[1]
        return fwd + fwd + dx

    def pack(self, params):
        """List of (W, b) -> padded flat float32 array."""
        offs, total = self.offsets()
        flat = np.zeros(total, np.float32)
        for (wo, bo), (w, b), i in zip(offs, params, range(self.num_layers)):
            flat[wo:wo + w.size] = np.asarray(w, np.float32).reshape(-1)
            flat[bo:bo + b.size] = np.asarray(b, np.float32).reshape(-1)
        return flat

    def unpack(self, flat):
        """Padded flat array -> list of (W [d_i, d_i+1], b [d_i+1])."""
        offs, _ = self.offsets()
        flat = np.asarray(flat)
        out = []
        for i, (wo, bo) in enumerate(offs):
            k, n = self.dims[i], self.dims[i + 1]
            out.append((flat[wo:wo + k * n].reshape(k, n), flat[bo:bo + n].copy()))
        return out


@dataclass(frozen=True)
class Workload:
    name: str
    actor: NetSpec = None
    critic: NetSpec = None
    batch: int = 256                 # global batch (rows per step over all ranks)
    dual: bool = True                # alpha*KL(pi_old||pi) term and log_alpha dual
    lr: float = 3e-4
    beta1: float = 0.9
    beta2: float = 0.999
    adam_eps: float = 1e-8
    max_grad_norm: float = float("inf")   # no clip stated for these workloads
    kl_eps: float = 0.01
    log_alpha: float = 0.0
    extra: dict = field(default_factory=dict)

    def flops_per_sample(self):
        macs = 0
        for net in (self.actor, self.critic):
            if net is not None:
                macs += net.macs_per_sample()
        return 2 * macs

    def input_bytes_per_sample(self):
        b = OBS_DIM * 4
        if self.actor is not None:
            b += 3 * NUM_ACTIONS * 4          # mask, q, pi_old logits
        if self.critic is not None:
            b += 4                            # target
        return b

    def param_count(self):
        return sum(n.param_count for n in (self.actor, self.critic) if n is not None) + \
            (1 if (self.actor is not None and self.dual) else 0)

    def describe(self):
        parts = []
        if self.actor is not None:
            parts.append("actor " + "-".join(map(str, self.actor.dims)))
        if self.critic is not None:
            parts.append("critic " + "-".join(map(str, self.critic.dims)))
        return f"{self.name}: " + " + ".join(parts) + f", batch {self.batch}"


WORKLOADS = {
    "c0": Workload("c0", actor=NetSpec((27, 128, 128, 9)), batch=256),
    "c1": Workload("c1", critic=NetSpec((27, 128, 128, 1)), batch=4096, dual=False),
    "c2": Workload("c2", actor=NetSpec((27, 256, 256, 256, 9)),
                   critic=NetSpec((27, 256, 256, 256, 1)), batch=65536),
    "c3": Workload("c3", actor=NetSpec((27, 512, 512, 512, 9)),
                   critic=NetSpec((27, 512, 512, 512, 1)), batch=1048576),
    "c4": Workload("c4", actor=NetSpec((27, 1024, 1024, 1024, 1024, 9)), batch=262144),
}


# ---------------------------------------------------------------------------
# Synthetic inputs
# ---------------------------------------------------------------------------

def make_boards(rng, rows):
    """Boards as three 0/1 planes [empty | X | O] and the legal mask (empty plane)."""
    cells = rng.integers(0, 3, size=(rows, 9), dtype=np.int8)
    while True:
        full = ~(cells == 0).any(axis=1)
        n = int(full.sum())
        if n == 0:
            break
        cells[full] = rng.integers(0, 3, size=(n, 9), dtype=np.int8)
    obs = np.empty((rows, OBS_DIM), np.float32)
    obs[:, 0:9] = cells == 0
    obs[:, 9:18] = cells == 1
    obs[:, 18:27] = cells == 2
    mask = obs[:, 0:9].copy()
    return obs, mask


def cells_of(obs):
    """Board cells [rows, 9] coded +1 (X, the agent's plane) / -1 (O) / 0 (empty) from the
    three-plane observation; the inverse of the encoding the learner applies to cells."""
    obs = np.asarray(obs)
    return (obs[:, 9:18] - obs[:, 18:27]).astype(np.float32)


def make_q(rng, mask, concentration=0.3):
    """Dirichlet(concentration) over the legal cells (normalised gammas), 0 elsewhere."""
    g = rng.gamma(concentration, 1.0, size=mask.shape) * mask
    s = g.sum(axis=1, keepdims=True)
    empty = s[:, 0] <= 0
    if empty.any():                       # every gamma underflowed: uniform instead
        g[empty] = mask[empty]
        s[empty] = mask[empty].sum(axis=1, keepdims=True)
    return (g / s).astype(np.float32)


def make_old_logits(rng, mask):
    z = rng.standard_normal(mask.shape).astype(np.float32)
    return np.where(mask > 0, z, NEG_INF).astype(np.float32)


def make_targets(rng, rows, gamma=0.99, n=5):
    r = rng.integers(-1, 2, size=(rows, n)).astype(np.float64)
    boot = rng.uniform(-1.0, 1.0, size=rows)
    disc = gamma ** np.arange(n)
    return ((r * disc).sum(axis=1) + gamma ** n * boot).astype(np.float32).reshape(rows, 1)


def make_batch(workload, rows, seed=0):
    """One batch of seeded synthetic learner inputs (dict of float32 arrays)."""
    rng = np.random.default_rng(seed)
    obs, mask = make_boards(rng, rows)
    out = {"obs": obs, "mask": mask}
    if workload.actor is not None:
        out["q"] = make_q(rng, mask)
        out["logits_old"] = make_old_logits(rng, mask)
    if workload.critic is not None:
        out["target"] = make_targets(rng, rows)
    return out


def glorot_params(net, rng):
    out = []
    for i in range(net.num_layers):
        fi, fo = net.dims[i], net.dims[i + 1]
        lim = np.sqrt(6.0 / (fi + fo))
        out.append((rng.uniform(-lim, lim, size=(fi, fo)).astype(np.float32),
                    np.zeros(fo, np.float32)))
    return out


def init_params(workload, seed=0):
    """Glorot-uniform weights, zero biases; actor first, then critic, from one stream."""
    rng = np.random.default_rng(seed)
    out = {}
    if workload.actor is not None:
        out["actor"] = glorot_params(workload.actor, rng)
    if workload.critic is not None:
        out["critic"] = glorot_params(workload.critic, rng)
    return out
