"""The fused learner step: one M-step update of the actor and/or critic.

Wraps spo_learner_* of libspo_cuda (the composition of demos/train_spo.mojo:417-554
update(): critic block and actor block, each with its own global-norm clip and Adam,
plus the log_alpha dual). All state lives in flat device buffers with one layout
[actor | critic | log_alpha | statistics]; the caller owns them through this object.

Data parallel: every rank runs ``backward`` on its shard with grad_scale =
1 / global_batch, then the flat gradient buffer (gradients + loss statistics) is
summed across ranks with ONE all-reduce, then every rank runs the same ``apply``.
"""

import ctypes
import math

import torch

from . import ffi
from .workloads import NetSpec


class _DeviceArray:
    """__cuda_array_interface__ wrapper of n float32 values of library-owned device memory."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 2, "strides": None}


def _device_view(ptr, n, device):
    """A float32 tensor aliasing n floats of device memory owned by the library."""
    return torch.as_tensor(_DeviceArray(ptr, n), device=device)


class Learner:
    def __init__(self, actor_dims=None, critic_dims=None, max_rows=1, lr_actor=3e-4,
                 lr_critic=3e-4, beta1=0.9, beta2=0.999, adam_eps=1e-8,
                 max_grad_norm=math.inf, kl_eps=0.01, use_kl=True, dual=True, device=None,
                 engine="tensor"):
        if device is None:                   # the caller's current device (one per rank)
            device = torch.cuda.current_device()
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        d = ffi.LearnerDesc()
        d.actor = ffi.MlpDesc.of(actor_dims)
        d.critic = ffi.MlpDesc.of(critic_dims)
        d.max_rows = int(max_rows)
        d.lr_actor, d.lr_critic = lr_actor, lr_critic
        d.beta1, d.beta2, d.adam_eps = beta1, beta2, adam_eps
        d.max_grad_norm = max_grad_norm
        d.kl_eps = kl_eps
        d.use_kl = 1 if (use_kl and actor_dims is not None) else 0
        d.dual = 1 if (dual and d.use_kl) else 0
        if engine not in ("tensor", "cuda"):
            raise ValueError("engine must be 'tensor' (tcgen05 3xTF32 where shapes allow) or 'cuda'")
        d.engine = 0 if engine == "tensor" else 1
        self.desc = d
        self.actor_dims = tuple(actor_dims) if actor_dims is not None else None
        self.critic_dims = tuple(critic_dims) if critic_dims is not None else None
        self.layout = ffi.LearnerLayout()
        ffi.call("spo_learner_layout_of", ctypes.byref(d), ctypes.byref(self.layout))
        nbytes = ffi.lib().spo_learner_workspace_size(ctypes.byref(d))
        if nbytes == 0:
            raise ffi.SpoError(-1, ffi.last_error())
        total = self.layout.total
        dev = self.device
        self.workspace = torch.empty(int(nbytes), dtype=torch.uint8, device=dev)
        self.params = torch.zeros(total, dtype=torch.float32, device=dev)
        self.grads = torch.zeros(total, dtype=torch.float32, device=dev)
        self.adam_m = torch.zeros(total, dtype=torch.float32, device=dev)
        self.adam_v = torch.zeros(total, dtype=torch.float32, device=dev)
        self.step_counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.report = torch.zeros(ffi.REPORT_SIZE, dtype=torch.float32, device=dev)
        handle = ctypes.c_void_p()
        torch.cuda.synchronize(dev)
        ffi.call("spo_learner_create", ctypes.byref(d), self.workspace.data_ptr(),
                 self.workspace.numel(), ctypes.byref(handle))
        self._h = handle
        self._state = ffi.TrainState(self.params.data_ptr(), self.grads.data_ptr(),
                                     self.adam_m.data_ptr(), self.adam_v.data_ptr(),
                                     self.step_counter.data_ptr(), self.report.data_ptr())

    def close(self):
        if getattr(self, "_h", None):
            ffi.lib().spo_learner_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------ buffers
    def net_slice(self, which, buf=None):
        buf = self.params if buf is None else buf
        lay = self.layout
        if which == "actor":
            return buf[lay.actor_offset:lay.actor_offset + lay.actor_size]
        return buf[lay.critic_offset:lay.critic_offset + lay.critic_size]

    def tensors(self, which, buf=None):
        """[(W, b)] views of one network in a flat buffer (params by default)."""
        dims = self.actor_dims if which == "actor" else self.critic_dims
        spec = NetSpec(dims)
        flat = self.net_slice(which, buf)
        offs, _ = spec.offsets()
        out = []
        for i, (wo, bo) in enumerate(offs):
            k, n = dims[i], dims[i + 1]
            out.append((flat[wo:wo + k * n].view(k, n), flat[bo:bo + n]))
        return out

    def load(self, actor=None, critic=None, log_alpha=0.0):
        """Set parameters from lists of (W, b) arrays; reset Adam state and step."""
        self.params.zero_()
        for which, params in (("actor", actor), ("critic", critic)):
            if params is None:
                continue
            for (w, b), (tw, tb) in zip(params, self.tensors(which)):
                tw.copy_(torch.as_tensor(w, dtype=torch.float32))
                tb.copy_(torch.as_tensor(b, dtype=torch.float32))
        self.params[self.layout.alpha_index] = float(log_alpha)
        self.adam_m.zero_()
        self.adam_v.zero_()
        self.step_counter.zero_()

    # ------------------------------------------------------------ checkpoint
    CHECKPOINT_FILES = ("params.bin", "adam_m.bin", "adam_v.bin")

    def _checkpoint_meta(self):
        d = self.desc
        return {"format": "spo-learner-checkpoint/1", "actor_dims": self.actor_dims,
                "critic_dims": self.critic_dims, "total": int(self.layout.total),
                "lr_actor": d.lr_actor, "lr_critic": d.lr_critic, "beta1": d.beta1, "beta2": d.beta2,
                "adam_eps": d.adam_eps, "max_grad_norm": d.max_grad_norm, "kl_eps": d.kl_eps,
                "use_kl": int(d.use_kl), "dual": int(d.dual)}

    def save_checkpoint(self, path):
        """Write the learner's state into directory `path`: the flat parameter buffer and
        both Adam moments as raw little-endian float32 (`params.bin`, `adam_m.bin`,
        `adam_v.bin`; the layout of spo_learner_layout_of, the raw-f32 convention of the
        reference's golden tensors, tests/golden_io.mojo) and `checkpoint.json` (the
        networks, hyperparameters and Adam's step). Waits for the learner's device."""
        import json
        import os
        os.makedirs(path, exist_ok=True)
        torch.cuda.synchronize(self.device)
        for name, buf in zip(self.CHECKPOINT_FILES, (self.params, self.adam_m, self.adam_v)):
            buf.detach().cpu().numpy().astype("<f4").tofile(os.path.join(path, name))
        meta = self._checkpoint_meta()
        meta["step"] = int(self.step_counter.item())
        with open(os.path.join(path, "checkpoint.json"), "w") as f:
            json.dump(meta, f, indent=1)

    def load_checkpoint(self, path):
        """Restore a state written by save_checkpoint into this learner, which must have the
        same networks and hyperparameters (ValueError otherwise); the next step continues
        Adam where the saved one stopped."""
        import json
        import os
        import numpy as np
        with open(os.path.join(path, "checkpoint.json")) as f:
            meta = json.load(f)
        mine = self._checkpoint_meta()
        for k, v in mine.items():
            saved = meta.get(k)
            if isinstance(v, tuple):
                saved = tuple(saved) if saved is not None else None
            same = saved == v if not isinstance(v, float) else (
                saved is not None and (saved == v or math.isclose(saved, v, rel_tol=1e-6)))
            if not same:
                raise ValueError(f"checkpoint {path}: {k} is {saved!r}, this learner has {v!r}")
        total = int(self.layout.total)
        for name, buf in zip(self.CHECKPOINT_FILES, (self.params, self.adam_m, self.adam_v)):
            raw = np.fromfile(os.path.join(path, name), dtype="<f4")
            if raw.size != total:
                raise ValueError(f"checkpoint {path}: {name} holds {raw.size} floats, expected {total}")
            buf.copy_(torch.from_numpy(raw))
        self.step_counter.fill_(int(meta["step"]))
        torch.cuda.synchronize(self.device)

    @property
    def log_alpha(self):
        return self.params[self.layout.alpha_index]

    def stats_tensor(self):
        off = self.layout.stats_offset
        return self.grads[off:off + ffi.NUM_STATS]

    def stats(self):
        s = self.stats_tensor().tolist()
        return {k: s[v] for k, v in ffi.STAT.items()}

    def activations(self, which, rows):
        """Post-ReLU activations of the last forward, one [rows x d] tensor per hidden
        layer (a copy; hi + lo with the tensor-core engine)."""
        dims = self.actor_dims if which == "actor" else self.critic_dims
        out = []
        for layer in range(len(dims) - 2):
            hi, lo = ctypes.c_void_p(), ctypes.c_void_p()
            ffi.call("spo_learner_cache", self._h, 0 if which == "actor" else 1, layer,
                     ctypes.byref(hi), ctypes.byref(lo))
            n = rows * dims[layer + 1]
            t = _device_view(hi.value, n, self.device).clone()
            if lo.value:
                t += _device_view(lo.value, n, self.device)
            out.append(t.view(rows, dims[layer + 1]))
        return out

    def set_small_rows(self, max_rows):
        """Batches of at most max_rows rows run as one cooperative launch (0: never)."""
        ffi.call("spo_learner_set_small_rows", self._h, int(max_rows))

    def device_status(self):
        """0 when every bounded wait of the tensor-core kernels completed (synchronises)."""
        v = ctypes.c_int32()
        ffi.call("spo_learner_status", self._h, ctypes.byref(v))
        return v.value

    def report_dict(self):
        r = self.report.tolist()
        return {k: r[v] for k, v in ffi.REPORT.items()}

    # ------------------------------------------------------------ the step
    def _batch(self, batch, rows=None):
        """Batch dict -> spo_batch. Inputs: "obs" [rows x d0], or "cells" [rows x 9] board
        cells (+1 agent / -1 rival / 0 empty) encoded on the fly (then "mask" may be left
        out: the legal mask is the empty cells); "mask", "q", "logits_old" (actor),
        "target" (critic)."""
        g = batch.get
        first = g("obs") if g("obs") is not None else g("cells")
        rows = int(first.shape[0]) if rows is None else int(rows)
        ptr = lambda k: g(k).data_ptr() if g(k) is not None else None  # noqa: E731
        return ffi.Batch(ptr("obs"), ptr("mask"), ptr("q"), ptr("logits_old"), ptr("target"), rows,
                         ptr("cells"))

    def backward(self, batch, grad_scale=None, stream=None):
        b = self._batch(batch)
        scale = (1.0 / b.rows if b.rows else 0.0) if grad_scale is None else grad_scale
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        ffi.call("spo_learner_backward", self._h, s, ctypes.byref(b), scale, ctypes.byref(self._state))

    def apply(self, stream=None):
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        ffi.call("spo_learner_apply", self._h, s, ctypes.byref(self._state))

    def step(self, batch, stream=None):
        b = self._batch(batch)
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        ffi.call("spo_learner_step", self._h, s, ctypes.byref(b), ctypes.byref(self._state))

    def capture_step(self, batch, warmup=1):
        """Record one learner step on `batch` (fixed device tensors) as a CUDA graph; each
        `graph.replay()` then runs the whole step (every kernel, the device-side Adam step
        counter included) with one launch. Refill the batch tensors in place between
        replays. The step's kernels neither allocate nor synchronise, so the graph holds
        only libspo_cuda launches."""
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):  # first launches set kernel attributes outside the capture
                self.step(batch, stream=side)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.step(batch)
        return graph

    def forward(self, which, obs, mask=None, stream=None):
        """Inference forward of one network: (logits or V, pi or None)."""
        dims = self.actor_dims if which == "actor" else self.critic_dims
        rows = obs.shape[0]
        out = torch.empty(rows, dims[-1], dtype=torch.float32, device=self.device)
        pi = torch.empty_like(out) if which == "actor" else None
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        ffi.call("spo_learner_forward", self._h, s, 0 if which == "actor" else 1,
                 self.params.data_ptr(), obs.data_ptr(),
                 mask.data_ptr() if mask is not None else None, rows, out.data_ptr(),
                 pi.data_ptr() if pi is not None else None)
        return out, pi

    @classmethod
    def for_workload(cls, wl, max_rows=None, device=None, **kw):
        return cls(actor_dims=wl.actor.dims if wl.actor else None,
                   critic_dims=wl.critic.dims if wl.critic else None,
                   max_rows=max_rows or wl.batch, lr_actor=wl.lr, lr_critic=wl.lr,
                   beta1=wl.beta1, beta2=wl.beta2, adam_eps=wl.adam_eps,
                   max_grad_norm=wl.max_grad_norm, kl_eps=wl.kl_eps, use_kl=wl.dual,
                   dual=wl.dual, device=device, **kw)


def _packed_layout(like):
    """Byte offsets of the fields of a batch packed into one buffer (each field on a
    256-byte boundary) and the total size."""
    offs, off = {}, 0
    for k, v in like.items():
        offs[k] = off
        off += (v.numel() * v.element_size() + 255) // 256 * 256
    return offs, max(off, 256)


def _packed_views(flat, like, offs):
    return {k: flat[offs[k]:offs[k] + v.numel() * v.element_size()].view(v.dtype).view(v.shape)
            for k, v in like.items()}


class PackedHostBatch(dict):
    """A host batch whose fields are views of ONE pinned buffer (`flat`), so that its
    upload is one host-to-device copy instead of one per field. Fill it like a dict of
    tensors (`batch[k].copy_(...)`); `HostFeed.upload` recognises it."""

    def __init__(self, like):
        offs, total = _packed_layout(like)
        self.flat = torch.empty(total, dtype=torch.uint8).pin_memory()
        super().__init__(_packed_views(self.flat, like, offs))
        self.offsets = offs

    @classmethod
    def of(cls, arrays):
        """A packed pinned copy of a dict of numpy arrays or tensors."""
        like = {k: torch.as_tensor(v) for k, v in arrays.items()}
        b = cls(like)
        for k, v in like.items():
            b[k].copy_(v)
        return b


class HostFeed:
    """Feeds host (pinned) batches to the learner through two device buffers: the upload of
    the next step's inputs runs on a copy stream while the current step's kernels run on
    the compute stream (events order each buffer's upload before its step, and the step
    before the buffer's next upload). A `PackedHostBatch` with the same fields is uploaded
    with one copy (the device buffers share its packed layout).

        feed = HostFeed(host_batch, device, stream)
        j = feed.upload(host_batch)              # inputs of step 0
        for i in range(steps):
            b = feed.take(j)                     # the compute stream waits for the upload
            if i + 1 < steps:
                nxt = feed.upload(next_host_batch)
            learner.step(b, stream=stream)
            feed.release(j)                      # the buffer may be refilled after the step
            j = nxt
    """

    def __init__(self, like, device, compute_stream):
        self.device = torch.device(device) if not isinstance(device, torch.device) else device
        self.compute = compute_stream
        self.copy = torch.cuda.Stream(self.device)
        self._offs, total = _packed_layout(like)
        self.flats = [torch.empty(total, dtype=torch.uint8, device=self.device) for _ in range(2)]
        self.bufs = [_packed_views(f, like, self._offs) for f in self.flats]
        self.ready = [torch.cuda.Event() for _ in range(2)]
        self.free = [torch.cuda.Event() for _ in range(2)]
        self._next = 0

    def copy_into(self, j, host_batch):
        """Enqueue the upload of host_batch into buffer j on the current stream; returns
        the bytes copied."""
        if isinstance(host_batch, PackedHostBatch) and host_batch.offsets == self._offs \
                and host_batch.flat.numel() == self.flats[j].numel():
            self.flats[j].copy_(host_batch.flat, non_blocking=True)
            return host_batch.flat.numel()
        n = 0
        for k, v in host_batch.items():
            self.bufs[j][k].copy_(v, non_blocking=True)
            n += v.numel() * v.element_size()
        return n

    def upload(self, host_batch):
        j = self._next
        self._next ^= 1
        self.copy.wait_event(self.free[j])  # a never-recorded event does not block
        with torch.cuda.stream(self.copy):
            self.copy_into(j, host_batch)
        self.ready[j].record(self.copy)
        return j

    def take(self, j):
        self.compute.wait_event(self.ready[j])
        return self.bufs[j]

    def release(self, j):
        self.free[j].record(self.compute)


class Comm:
    """NCCL communicator of libspo_cuda (one per rank); ids shared by the caller."""

    def __init__(self, unique_id, nranks, rank):
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(unique_id), ffi.COMM_ID_BYTES)
        ffi.call("spo_comm_init", ctypes.byref(h), buf, nranks, rank)
        self._h = h

    @staticmethod
    def unique_id():
        buf = ctypes.create_string_buffer(ffi.COMM_ID_BYTES)
        ffi.call("spo_comm_get_unique_id", buf)
        return bytes(buf.raw)

    def allreduce_(self, tensor, stream=None):
        s = (stream or torch.cuda.current_stream(tensor.device)).cuda_stream
        ffi.call("spo_allreduce_sum", self._h, s, tensor.data_ptr(), tensor.numel())

    def close(self):
        if getattr(self, "_h", None):
            ffi.lib().spo_comm_destroy(self._h)
            self._h = None
