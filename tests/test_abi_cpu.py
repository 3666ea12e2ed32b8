"""The C ABI without a GPU: the library loads, exports exactly what include/spo_cuda.h
declares, and its pure host functions (layouts, sizes, clip scale, argument checks)
behave. No compute call is made."""

import ctypes
import math
import subprocess

import pytest

from spo_mojo_b200 import ffi
from spo_mojo_b200.workloads import WORKLOADS, NetSpec


def test_library_loads_and_exports_every_declared_symbol():
    L = ffi.lib()
    declared = ffi.header_symbols()
    assert len(declared) >= 40
    for name in declared:
        assert hasattr(L, name), name
    assert set(declared) == set(ffi.SIGNATURES), "ctypes table must match the header"
    out = subprocess.run(["nm", "-D", "--defined-only", ffi.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == set(declared), exported ^ set(declared)
    assert L.spo_abi_version() == 3


@pytest.mark.parametrize("dims", [(27, 128, 128, 9), (27, 512, 512, 512, 1), (18, 5, 3), (4, 5, 5, 1)])
def test_param_layout_matches_python(dims):
    d = ffi.MlpDesc.of(dims)
    L = len(dims) - 1
    w = (ctypes.c_int64 * L)()
    b = (ctypes.c_int64 * L)()
    tot = ctypes.c_int64()
    ffi.call("spo_mlp_param_layout", ctypes.byref(d), w, b, ctypes.byref(tot))
    offs, total = NetSpec(dims).offsets()
    assert [(w[i], b[i]) for i in range(L)] == offs
    assert tot.value == total
    for i in range(L):
        assert w[i] % 64 == 0 and b[i] % 64 == 0


def test_learner_layout_and_workspace():
    wl = WORKLOADS["c3"]
    desc = ffi.LearnerDesc()
    desc.actor = ffi.MlpDesc.of(wl.actor.dims)
    desc.critic = ffi.MlpDesc.of(wl.critic.dims)
    desc.max_rows = wl.batch
    desc.lr_actor = desc.lr_critic = 3e-4
    desc.beta1, desc.beta2, desc.adam_eps = 0.9, 0.999, 1e-8
    desc.max_grad_norm = math.inf
    desc.kl_eps = 0.01
    desc.use_kl = desc.dual = 1
    lay = ffi.LearnerLayout()
    ffi.call("spo_learner_layout_of", ctypes.byref(desc), ctypes.byref(lay))
    assert lay.actor_offset == 0 and lay.actor_size == wl.actor.padded_size
    assert lay.critic_offset == wl.actor.padded_size and lay.critic_size == wl.critic.padded_size
    assert lay.alpha_index == lay.critic_offset + lay.critic_size
    assert lay.stats_offset == lay.alpha_index + 64 and lay.total == lay.stats_offset + 64
    ws = ffi.lib().spo_learner_workspace_size(ctypes.byref(desc))
    # activations of both nets dominate: 2 nets x 1M rows x 1536 floats
    assert ws > 2 * wl.batch * 1536 * 4


def test_argument_errors_are_reported_not_launched():
    desc = ffi.LearnerDesc()
    desc.actor = ffi.MlpDesc.of((27, 128, 10))  # actor output must be 9
    desc.max_rows = 16
    lay = ffi.LearnerLayout()
    with pytest.raises(ffi.SpoError) as e:
        ffi.call("spo_learner_layout_of", ctypes.byref(desc), ctypes.byref(lay))
    assert e.value.code == -7 and "output width" in str(e.value)
    desc.actor = ffi.MlpDesc.of((27, 128, 9))
    desc.max_rows = 0
    with pytest.raises(ffi.SpoError) as e:
        ffi.call("spo_learner_layout_of", ctypes.byref(desc), ctypes.byref(lay))
    assert e.value.code == -2
    with pytest.raises(ffi.SpoError):
        ffi.call("spo_linear_fwd", None, None, None, None, None, 4, 4, 4, 0)   # null pointers
    with pytest.raises(ffi.SpoError):
        ffi.call("spo_adam_flat", None, 1, 1, 1, 1, 4, 1e-3, 0.9, 0.999, 1e-8, 0, 1.0)  # step 0


def test_global_clip_scale_known_answers():
    # networks/optim.mojo:133-142 and tests/test_optim.mojo:131-158: (3, 4, 12) -> 13
    f = ffi.lib().spo_global_clip_scale
    assert abs(f(169.0, 6.5) - 0.5) < 1e-7
    assert f(169.0, 13.0) == 1.0
    assert f(169.0, math.inf) == 1.0
    assert f(169.0, 0.0) == 1.0


def test_workspace_queries_are_monotone():
    L = ffi.lib()
    a = L.spo_linear_bwd_workspace_size(1024, 512, 512)
    b = L.spo_linear_bwd_workspace_size(4096, 512, 512)
    assert 0 < a <= b
    d = ffi.MlpDesc.of((27, 256, 256, 9))
    assert 0 < L.spo_mlp_bwd_workspace_size(ctypes.byref(d), 100) <= L.spo_mlp_bwd_workspace_size(ctypes.byref(d), 1000)
    assert L.spo_head_workspace_size(10, 128, 9) > 0
