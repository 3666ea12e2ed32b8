"""Host-side mirror of the reference's networks/ API over libspo_cuda.

Same names, argument order and meaning as the Mojo functions of
josedanielchg/spo-mojo networks/ (and the pieces of ops/ and rl_utils/ they use),
with torch CUDA float32 tensors standing in for DeviceBuffer[float32] and a
DeviceContext wrapping one CUDA stream. Every function enqueues libspo_cuda kernels
on ctx's stream through the C ABI; nothing here computes on the CPU.

Parameter containers keep the reference's field names (w1, b1, w2, ...) but are
views into ONE flat buffer (the layout of spo_mlp_param_layout), so that the
optimiser can run over all tensors in one launch. Shape and capacity errors raise
(the reference raises Error in the same places).
"""

import ctypes

import torch

from . import ffi
from .workloads import NetSpec

OBS_DIM = 27
NUM_ACTIONS = 9
ADAM_EPS = 1e-5        # networks/optim.mojo:43 (Stoix's value)
BETA1, BETA2 = 0.9, 0.999


class DeviceContext:
    """std.gpu.host.DeviceContext: one device, one in-order stream (networks/mlp.mojo:109-110)."""

    def __init__(self, device=0, stream=None):
        self.device = torch.device("cuda", device)
        self.stream = stream if stream is not None else torch.cuda.current_stream(self.device)
        self._ws = None

    @property
    def handle(self):
        return self.stream.cuda_stream

    def synchronize(self):
        self.stream.synchronize()

    def enqueue_create_buffer(self, n):
        with torch.cuda.stream(self.stream):
            return torch.zeros(int(n), dtype=torch.float32, device=self.device)

    def workspace(self, nbytes):
        """Scratch for the calls that need it (grown on demand, reused)."""
        nbytes = int(max(nbytes, 256))
        if self._ws is None or self._ws.numel() < nbytes:
            self.synchronize()
            self._ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        return self._ws


def zero_buffer(ctx, n):
    """ops/buffers.mojo:21-34."""
    return ctx.enqueue_create_buffer(n)


def _p(t):
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------- Linear (networks/linear.mojo)

def linear_forward(ctx, y, x, w, bias, m, k, n, relu=False):
    """y = x @ W + b (networks/linear.mojo:86-95); relu=True fuses networks/mlp.mojo:34-46."""
    ffi.call("spo_linear_fwd", ctx.handle, _p(y), _p(x), _p(w), _p(bias), m, k, n, 1 if relu else 0)


def linear_backward(ctx, dw, db, dx, x, w, dy, m, k, n, relu_src=None):
    """dW = x^T dy, db = sum dy, dx = dy W^T (networks/linear.mojo:170-193)."""
    nbytes = ffi.lib().spo_linear_bwd_workspace_size(m, k, n)
    ws = ctx.workspace(nbytes)
    ffi.call("spo_linear_bwd", ctx.handle, _p(dw), _p(db), _p(dx), _p(x), _p(w), _p(dy),
             _p(relu_src), m, k, n, ws.data_ptr(), ws.numel())


def relu(ctx, a, n):
    """In-place ReLU (networks/mlp.mojo:34-46)."""
    ffi.call("spo_relu", ctx.handle, _p(a), n)


def relu_backward(ctx, grad, activation, n):
    """grad *= (activation > 0) in place (networks/mlp.mojo:155-166)."""
    ffi.call("spo_relu_bwd", ctx.handle, _p(grad), _p(activation), n)


# ---------------------------------------------------------------- MLP (networks/mlp.mojo)

class MLPParams:
    """Weights of an MLP with dims d0..dL as views into one flat buffer.

    CriticParams (networks/mlp.mojo:50-68) generalised to L layers; w1, b1, ...
    remain available as attributes.
    """

    def __init__(self, ctx, dims, flat=None):
        self.dims = tuple(int(d) for d in dims)
        self.spec = NetSpec(self.dims)
        offs, total = self.spec.offsets()
        self.flat = flat if flat is not None else zero_buffer(ctx, total)
        self.w, self.b = [], []
        for i, (wo, bo) in enumerate(offs):
            k, n = self.dims[i], self.dims[i + 1]
            self.w.append(self.flat[wo:wo + k * n].view(k, n))
            self.b.append(self.flat[bo:bo + n])

    def __getattr__(self, name):
        if len(name) >= 2 and name[0] in "wb" and name[1:].isdigit():
            i = int(name[1:]) - 1
            return (self.w if name[0] == "w" else self.b)[i]
        raise AttributeError(name)

    @property
    def in_dim(self):
        return self.dims[0]

    @property
    def hidden(self):
        return self.dims[1]

    @property
    def out_dim(self):
        return self.dims[-1]

    @property
    def desc(self):
        return ffi.MlpDesc.of(self.dims)

    def load(self, params):
        """Copy a list of (W, b) host or device arrays into the flat buffer."""
        for i, (w, b) in enumerate(params):
            self.w[i].copy_(torch.as_tensor(w, dtype=torch.float32))
            self.b[i].copy_(torch.as_tensor(b, dtype=torch.float32))


CriticParams = MLPParams
ActorParams = MLPParams   # networks/actor.mojo:39-40


def zero_critic_params(ctx, in_dim, hidden, out_dim, depth=2):
    """networks/mlp.mojo:71-81 (depth = number of hidden layers)."""
    return MLPParams(ctx, (in_dim,) + (hidden,) * depth + (out_dim,))


def zero_actor_params(ctx, hidden, in_dim=OBS_DIM, depth=2):
    """networks/actor.mojo:45-47."""
    return MLPParams(ctx, (in_dim,) + (hidden,) * depth + (NUM_ACTIONS,))


class CriticCache:
    """One forward's post-ReLU activations and output (networks/mlp.mojo:84-102)."""

    def __init__(self, ctx, max_batch, dims):
        self.dims = tuple(dims)
        self.max_batch = int(max_batch)
        n_act = sum(self.max_batch * d for d in self.dims[1:-1])
        self.acts = zero_buffer(ctx, max(n_act, 1))
        self.value = zero_buffer(ctx, self.max_batch * self.dims[-1])

    def act(self, i, m):
        """a_{i+1} of the last forward with m rows, [m x d_{i+1}]."""
        off = sum(m * d for d in self.dims[1:1 + i])
        return self.acts[off:off + m * self.dims[i + 1]].view(m, self.dims[i + 1])

    def check(self, m):
        if m > self.max_batch:
            raise ValueError(f"the cache was reserved for {self.max_batch} rows and is being "
                             f"asked for {m}")


ActorCache = CriticCache


def critic_forward(ctx, params, cache, x, m):
    """V(s) for m inputs; activations stay in cache (networks/mlp.mojo:105-123)."""
    cache.check(m)
    d = params.desc
    ffi.call("spo_mlp_fwd", ctx.handle, ctypes.byref(d), _p(params.flat), _p(x), m,
             _p(cache.acts), _p(cache.value))


class CriticGrads:
    """Gradients with the layout of the parameters (networks/mlp.mojo:169-186)."""

    def __init__(self, ctx, dims):
        self.p = MLPParams(ctx, dims)
        self.flat = self.p.flat

    def __getattr__(self, name):
        if name.startswith("d") and len(name) >= 3:
            return getattr(self.p, name[1:])
        raise AttributeError(name)


class CriticScratch:
    """dvalue and the backward's working memory (networks/mlp.mojo:189-209)."""

    def __init__(self, ctx, max_batch, dims):
        self.dims = tuple(dims)
        self.dvalue = zero_buffer(ctx, max_batch * self.dims[-1])
        d = ffi.MlpDesc.of(self.dims)
        nbytes = ffi.lib().spo_mlp_bwd_workspace_size(ctypes.byref(d), max_batch)
        self.ws = torch.empty(int(nbytes), dtype=torch.uint8, device=ctx.device)


def backward_from_dvalue(ctx, params, cache, grads, scratch, x, m):
    """All gradients from scratch.dvalue (networks/mlp.mojo:236-275)."""
    cache.check(m)
    d = params.desc
    ffi.call("spo_mlp_bwd", ctx.handle, ctypes.byref(d), _p(params.flat), _p(x), _p(cache.acts),
             _p(scratch.dvalue), m, _p(grads.flat), scratch.ws.data_ptr(), scratch.ws.numel())


def critic_backward(ctx, params, cache, grads, scratch, x, target, m):
    """Gradients for L = mean 0.5 (V - target)^2 (networks/mlp.mojo:212-233)."""
    n_out = m * params.out_dim
    ffi.call("spo_value_loss_grad", ctx.handle, _p(scratch.dvalue), _p(cache.value), _p(target),
             n_out, 1.0 / n_out)
    backward_from_dvalue(ctx, params, cache, grads, scratch, x, m)


# ---------------------------------------------------------------- actor (networks/actor.mojo)

def actor_logits(ctx, params, cache, obs, mask, m):
    """Masked logits into cache.value (networks/actor.mojo:74-87)."""
    critic_forward(ctx, params, cache, obs, m)
    ffi.call("spo_mask_logits", ctx.handle, _p(cache.value), _p(mask), m * params.out_dim)


def actor_probs(ctx, params, cache, obs, mask, probs_out, m):
    """pi(a|s), masked (networks/actor.mojo:90-103)."""
    actor_logits(ctx, params, cache, obs, mask, m)
    ffi.call("spo_softmax_rows", ctx.handle, _p(probs_out), _p(cache.value), m, params.out_dim)


def actor_log_probs(ctx, params, cache, obs, mask, log_probs_out, m):
    """log pi(a|s) computed directly (networks/actor.mojo:106-122)."""
    actor_logits(ctx, params, cache, obs, mask, m)
    ffi.call("spo_log_softmax_rows", ctx.handle, _p(log_probs_out), _p(cache.value), m,
             params.out_dim)


class Actor:
    """The actor with its buffers for up to max_batch boards (networks/actor.mojo:125-194)."""

    def __init__(self, ctx, max_batch, hidden, in_dim=OBS_DIM, depth=2):
        self.params = zero_actor_params(ctx, hidden, in_dim, depth)
        self.cache = ActorCache(ctx, max_batch, self.params.dims)
        self.mask = zero_buffer(ctx, max_batch * NUM_ACTIONS)
        self.probs = zero_buffer(ctx, max_batch * NUM_ACTIONS)
        self.log_probs = zero_buffer(ctx, max_batch * NUM_ACTIONS)
        self.hidden = hidden
        self.max_batch = max_batch

    def _check(self, m):
        if m > self.max_batch:
            raise ValueError(f"the actor was reserved for {self.max_batch} boards and is being "
                             f"asked for {m}")

    def forward(self, ctx, obs, mask, m):
        self._check(m)
        actor_probs(ctx, self.params, self.cache, obs, mask, self.probs, m)

    def forward_log(self, ctx, obs, mask, m):
        self._check(m)
        actor_log_probs(ctx, self.params, self.cache, obs, mask, self.log_probs, m)


# ---------------------------------------------------------------- softmax (ops/softmax.mojo)

def softmax_rows(ctx, out, a, rows, row_size):
    ffi.call("spo_softmax_rows", ctx.handle, _p(out), _p(a), rows, row_size)


def log_softmax_rows(ctx, out, a, rows, row_size):
    ffi.call("spo_log_softmax_rows", ctx.handle, _p(out), _p(a), rows, row_size)


def logsumexp_rows(ctx, out, a, rows, row_size):
    ffi.call("spo_logsumexp_rows", ctx.handle, _p(out), _p(a), rows, row_size)


# ---------------------------------------------------------------- loss (networks/actor_loss.mojo)

def cross_entropy_rows(ctx, loss_out, q, log_pi, n_rows, num_actions):
    ffi.call("spo_cross_entropy_rows", ctx.handle, _p(loss_out), _p(q), _p(log_pi), n_rows, num_actions)


def entropy_rows(ctx, h_out, q, n_rows, num_actions):
    ffi.call("spo_entropy_rows", ctx.handle, _p(h_out), _p(q), n_rows, num_actions)


def kl_rows(ctx, kl_out, cross_entropy, entropy, n_rows):
    ffi.call("spo_kl_rows", ctx.handle, _p(kl_out), _p(cross_entropy), _p(entropy), n_rows)


def actor_backward(ctx, params, cache, grads, scratch, x, pi, q, mask, m):
    """Gradients of the eq-11 loss (networks/actor_loss.mojo:194-214)."""
    n_out = m * params.out_dim
    ffi.call("spo_logits_grad", ctx.handle, _p(scratch.dvalue), _p(pi), _p(q), _p(mask), n_out, 1.0 / m)
    backward_from_dvalue(ctx, params, cache, grads, scratch, x, m)


def actor_loss_fwd_bwd(ctx, dz, stats, logits, mask, q, m, num_actions=NUM_ACTIONS, logits_old=None,
                       log_alpha=None, eps_kl=0.01, scale=None, dlog_alpha=None):
    """The eq-11 loss on logits the caller computed, with the alpha*KL(pi_old || pi) term
    when logits_old is given: dz = dL/dz (the reference's logits_grad_kernel, scaled by
    1/m unless scale is given), the batch statistics into stats[0:5] (ffi.STAT) and the
    dual gradient into dlog_alpha[0] (optional). log_alpha: a one-element device tensor."""
    ws = ctx.workspace(ffi.lib().spo_loss_workspace_size())
    ffi.call("spo_actor_loss_fwd_bwd", ctx.handle, _p(logits), _p(mask), _p(q), _p(logits_old),
             _p(log_alpha), eps_kl, m, num_actions, (1.0 / m if m else 0.0) if scale is None else scale, _p(dz),
             _p(stats), _p(dlog_alpha), ws.data_ptr(), ws.numel())


def value_loss_fwd_bwd(ctx, dv, stats, value, target, n, scale=None):
    """0.5 * MSE on values the caller computed (networks/mlp.mojo:141-152): dv and
    stats[ffi.STAT['critic_loss']]."""
    ws = ctx.workspace(ffi.lib().spo_loss_workspace_size())
    ffi.call("spo_value_loss_fwd_bwd", ctx.handle, _p(value), _p(target), n,
             (1.0 / n if n else 0.0) if scale is None else scale, _p(dv), _p(stats), ws.data_ptr(), ws.numel())


# ---------------------------------------------------------------- optimiser (networks/optim.mojo)

class AdamState:
    """One tensor's (or one flat buffer's) two moments, starting at zero (:102-112)."""

    def __init__(self, ctx, size):
        self.m = zero_buffer(ctx, size)
        self.v = zero_buffer(ctx, size)
        self.size = size


def sum_squares(ctx, x, n):
    """Sum of squares, returned to the host like the reference (:115-130)."""
    out = zero_buffer(ctx, 1)
    ws = ctx.workspace(ffi.lib().spo_sum_squares_workspace_size())
    ffi.call("spo_sum_squares", ctx.handle, _p(x), n, _p(out), ws.data_ptr(), ws.numel())
    ctx.synchronize()
    return float(out.item())


def global_clip_scale(total_sq, max_norm):
    """:133-142."""
    return float(ffi.lib().spo_global_clip_scale(total_sq, max_norm))


def adam_step(ctx, param, grad, state, n, lr, grad_scale, step, eps=ADAM_EPS, b1=BETA1, b2=BETA2):
    """One Adam step over n elements (:172-187); step starts at 1."""
    ffi.call("spo_adam_flat", ctx.handle, _p(param), _p(grad), _p(state.m), _p(state.v), n, lr,
             b1, b2, eps, step, grad_scale)


def ema_update(ctx, target, online, n, tau):
    """target <- tau * online + (1 - tau) * target (:163-169)."""
    ffi.call("spo_ema", ctx.handle, _p(target), _p(online), n, tau)


def truncated_gae(ctx, adv, targets, reward, discount, v_tm1, v_t, truncation, batch, t_len, lambda_):
    """rl_utils/multistep.mojo:72-82."""
    ffi.call("spo_truncated_gae", ctx.handle, _p(adv), _p(targets), _p(reward), _p(discount),
             _p(v_tm1), _p(v_t), _p(truncation), batch, t_len, lambda_)


# ---------------------------------------------------------------- search heads (envs/)

def check_sync_shape(src_dims, want_dims, what):
    """The weight-sync shape test of the search models (envs/tictactoe_actor.mojo:108-140,
    envs/tictactoe_critic.mojo:145-155): a network is copied only into one of the same
    shape; here every width must match (the reference compares input, hidden and output)."""
    src_dims, want_dims = tuple(int(d) for d in src_dims), tuple(int(d) for d in want_dims)
    if src_dims != want_dims:
        raise ValueError(f"the {what} does not have the model's shape: " + "x".join(map(str, src_dims)))


class TicTacToeActorHead:
    """The network part of the search's actor model (envs/tictactoe_actor.mojo:64-191):
    frozen copies of the trained actor and critic, refreshed from the learner with
    sync_from / sync_critic_from, and their batched forward over m boards (m = envs x
    particles in the search). The environment's dynamics and the bootstrap around them
    are not part of this library."""

    def __init__(self, ctx, max_batch, hidden, depth=2):
        self.params = zero_actor_params(ctx, hidden, OBS_DIM, depth)
        self.cache = ActorCache(ctx, max_batch, self.params.dims)
        self.obs = zero_buffer(ctx, max_batch * OBS_DIM)
        self.mask = zero_buffer(ctx, max_batch * NUM_ACTIONS)
        self.critic = zero_critic_params(ctx, OBS_DIM, hidden, 1, depth)
        self.ccache = CriticCache(ctx, max_batch, self.critic.dims)
        self.hidden = hidden
        self.max_batch = max_batch

    def sync_from(self, ctx, src):
        """The trained actor's weights into the model's (:121-140)."""
        check_sync_shape(src.dims, self.params.dims, "actor being copied")
        with torch.cuda.stream(ctx.stream):
            self.params.flat.copy_(src.flat)

    def sync_critic_from(self, ctx, src):
        """The trained critic's weights into the model's (:108-119)."""
        check_sync_shape(src.dims, self.critic.dims, "critic")
        with torch.cuda.stream(ctx.stream):
            self.critic.flat.copy_(src.flat)

    def _check(self, m):
        if m > self.max_batch:
            raise ValueError(f"the model was reserved for {self.max_batch} boards and is being "
                             f"asked for {m}")

    def _prior(self, ctx, state, out_logits, m):
        """Masked logits over m boards into out_logits; mask and observation come from the
        boards (state [m x 9], +1 agent / -1 rival / 0 empty) (:148-171)."""
        self._check(m)
        ffi.call("spo_encode_obs", ctx.handle, _p(self.obs), _p(self.mask), _p(state), m)
        actor_logits(ctx, self.params, self.cache, self.obs, self.mask, m)
        with torch.cuda.stream(ctx.stream):
            out_logits.view(-1)[:m * NUM_ACTIONS].copy_(self.cache.value[:m * NUM_ACTIONS])

    def eval_root(self, ctx, state, logits_out, value_out, m):
        """The prior, then V from the critic on the observation _prior encoded (:173-191)."""
        self._prior(ctx, state, logits_out, m)
        critic_forward(ctx, self.critic, self.ccache, self.obs, m)
        with torch.cuda.stream(ctx.stream):
            value_out.view(-1)[:m].copy_(self.ccache.value[:m])


class TicTacToeCriticHead:
    """The network part of the search's critic model (envs/tictactoe_critic.mojo:98-192)."""

    def __init__(self, ctx, max_batch, hidden, depth=2):
        self.params = zero_critic_params(ctx, OBS_DIM, hidden, 1, depth)
        self.cache = CriticCache(ctx, max_batch, self.params.dims)
        self.obs = zero_buffer(ctx, max_batch * OBS_DIM)
        self.hidden = hidden
        self.max_batch = max_batch

    def sync_from(self, ctx, src):
        """:145-162"""
        check_sync_shape(src.dims, self.params.dims, "critic being copied")
        with torch.cuda.stream(ctx.stream):
            self.params.flat.copy_(src.flat)

    def value(self, ctx, state, value_out, m):
        """V over m boards (the network half of eval_root, :170-192)."""
        if m > self.max_batch:
            raise ValueError(f"the model was reserved for {self.max_batch} boards and is being "
                             f"asked for {m}")
        ffi.call("spo_encode_obs", ctx.handle, _p(self.obs), None, _p(state), m)
        critic_forward(ctx, self.params, self.cache, self.obs, m)
        with torch.cuda.stream(ctx.stream):
            value_out.view(-1)[:m].copy_(self.cache.value[:m])
