"""spo_linear_bwd_noalloc: the Linear backward for callers that cannot allocate device
memory (for instance inside a framework that has reserved nearly all of the GPU's memory
for its own pool). It must give the same dW, db and dx as spo_linear_bwd, which takes a
caller-allocated workspace, on consecutive calls (its static scratch keeps the previous
call's contents), and refuse shapes beyond its static scratch.

This file is collected last so that a run stopping at the first failure has already run
every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# the tolerance of the linear backward tests (tests/test_linear_backward.mojo:287-292
# of the reference: 1e-5 * sqrt(M) absolute for dW and db, 1e-5 * sqrt(N) for dx),
# applied here between the two entry points
def _tol(rows):
    return 1e-5 * np.sqrt(rows)


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _ffi():
    from spo_mojo_b200 import ffi
    return ffi


def _run(entry, x, w, dy, relu_src, m, k, n, with_dx=True):
    f = _ffi()
    dw = torch.full((k, n), float("nan"), device="cuda")
    db = torch.full((n,), float("nan"), device="cuda")
    dx = torch.full((m, k), float("nan"), device="cuda")
    args = [None, dw.data_ptr(), db.data_ptr(), dx.data_ptr() if with_dx else None, x.data_ptr(),
            w.data_ptr(), dy.data_ptr(), None if relu_src is None else relu_src.data_ptr(), m, k, n]
    if entry == "spo_linear_bwd":
        nbytes = f.lib().spo_linear_bwd_workspace_size(m, k, n)
        ws = torch.empty(int(nbytes), dtype=torch.uint8, device="cuda")
        f.call(entry, *args, ws.data_ptr(), ws.numel())
    else:
        f.call(entry, *args)
    torch.cuda.synchronize()
    return dw, db, dx


@pytest.mark.parametrize("m,k,n,with_dx", [(4096, 512, 512, True), (777, 128, 256, True),
                                           (65536, 27, 512, True), (0, 128, 256, True),
                                           (3000, 64, 128, False)])
def test_noalloc_matches_workspace_entry_on_consecutive_calls(m, k, n, with_dx):
    g = torch.Generator(device="cuda").manual_seed(m + k + n)
    for call in range(2):
        x = torch.randn(m, k, device="cuda", generator=g).relu_()
        w = torch.randn(k, n, device="cuda", generator=g) / k ** 0.5
        dy = torch.randn(m, n, device="cuda", generator=g) * 1e-2
        relu_src = x if with_dx else None   # without dx: neither dx nor its ReLU mask
        want = _run("spo_linear_bwd", x, w, dy, relu_src, m, k, n, with_dx)
        got = _run("spo_linear_bwd_noalloc", x, w, dy, relu_src, m, k, n, with_dx)
        outs = zip(("dW", "db", "dx"), got, want, (_tol(m), _tol(m), _tol(n)))
        for name, a, b, tol in list(outs)[:3 if with_dx else 2]:
            if a.numel() == 0:     # dx of zero rows
                continue
            assert torch.isfinite(a).all(), f"call {call}: {name} not fully written"
            assert float((a - b).abs().max()) <= tol, f"call {call}: {name}"
        if m == 0:  # no rows: the gradients of the weights are zero
            assert float(got[0].abs().max()) == 0.0 and float(got[1].abs().max()) == 0.0


@pytest.mark.parametrize("k,n", [(2048, 2048),          # k*n alone is 4,194,304 floats > 2,097,152
                                 (2**40, 2**30),        # k*n wraps int64: refused, not wrapped
                                 (2**40, 64),           # k alone too large
                                 (1, 8192)])            # 256*n alone fills the scratch
def test_noalloc_refuses_shapes_beyond_its_scratch(k, n):
    f = _ffi()
    with pytest.raises(f.SpoError) as e:
        f.call("spo_linear_bwd_noalloc", None, 1, 1, None, 1, 1, 1, None, 16, k, n)
    assert e.value.code == -4 and "static scratch" in str(e.value)


@pytest.mark.parametrize("case,m,k,n", [(0, 3, 4, 8), (1, 20, 18, 64), (2, 64, 64, 64), (3, 1, 1, 1)])
def test_noalloc_matches_the_reference_goldens(case, m, k, n):
    # the reference's linear backward goldens (tests/test_linear_backward.mojo:287-292),
    # at that test's tolerance, on two calls in a row through the shared static scratch
    from golden_io import read_f32
    x, w, dy = (torch.from_numpy(np.ascontiguousarray(read_f32(f"linbwd{case}_{s}"), dtype=np.float32))
                .cuda() for s in ("x", "w", "dy"))
    for call in range(2):
        dw, db, dx = _run("spo_linear_bwd_noalloc", x, w, dy, None, m, k, n)
        for name, got, tol in (("dw", dw, _tol(m)), ("db", db, _tol(m)), ("dx", dx, _tol(n))):
            want = read_f32(f"linbwd{case}_{name}").reshape(-1)
            err = float(np.max(np.abs(got.cpu().numpy().reshape(-1) - want)))
            assert err <= tol, f"call {call}: {name} off by {err}"
