"""The tcgen05 3xTF32 GEMM (spo_tc_gemm) against float64 products, for each fused
epilogue the learner uses. The bar is fp32-level accuracy: max |error| <= 1e-5 of
max |reference| (plain TF32 would sit near 1e-3)."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def ffi():
    from spo_mojo_b200 import ffi as f
    return f


def split(x):
    f = ffi()
    hi, lo = torch.empty_like(x), torch.empty_like(x)
    f.call("spo_split_tf32", None, hi.data_ptr(), lo.data_ptr(), x.data_ptr(), x.numel(), 0)
    return hi, lo


def run(desc):
    f = ffi()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    desc.err = err.data_ptr()
    grid, splits = ctypes.c_int32(), ctypes.c_int32()
    f.call("spo_tc_gemm_shape", ctypes.byref(desc), ctypes.byref(grid), ctypes.byref(splits))
    f.call("spo_tc_gemm", None, ctypes.byref(desc))
    torch.cuda.synchronize()
    assert int(err.item()) == 0, "a bounded wait in the kernel gave up"
    return grid.value, splits.value


def rel_err(got, want):
    want = np.asarray(want, np.float64)
    return float(np.max(np.abs(np.asarray(got, np.float64) - want)) / max(np.max(np.abs(want)), 1e-30))


def test_split_halves_are_tf32_and_close():
    x = torch.randn(4099, device="cuda") * 10
    hi, lo = split(x)
    assert torch.all((hi.view(torch.int32) & 0x1FFF) == 0)
    assert torch.all((lo.view(torch.int32) & 0x1FFF) == 0)
    err = ((hi.double() + lo.double()) - x.double()).abs()
    assert torch.all(err <= x.double().abs() * 2.0 ** -22)


@pytest.mark.parametrize("keep_positive", [0, 1])
def test_split_keeps_nan_and_infinities(keep_positive):
    """NaN (CUDA's canonical 0x7fffffff, its negation, a quiet and a payload-only NaN) stays
    NaN in hi, infinities stay infinite, the largest finite floats round to infinity as
    cvt.rna does, and tiny positive subnormals keep their value in hi for ReLU outputs."""
    f = ffi()
    pats = [0x7FFFFFFF, 0xFFFFFFFF, 0x7FC00000, 0x7F800001, 0x7FFFF000, 0xFFFFF000,
            0x7F800000, 0xFF800000, 0x7F7FFFFF, 0x00000001, 0x00000FFF, 0x3F800000]
    x = torch.tensor(np.array(pats, dtype=np.uint32).view(np.int32), device="cuda").view(torch.float32)
    hi, lo = torch.empty_like(x), torch.empty_like(x)
    f.call("spo_split_tf32", None, hi.data_ptr(), lo.data_ptr(), x.data_ptr(), x.numel(), keep_positive)
    torch.cuda.synchronize()
    h = hi.cpu().numpy()
    assert np.all(np.isnan(h[:6]))
    assert h[6] == np.inf and h[7] == -np.inf and h[8] == np.inf
    if keep_positive:
        assert h[9] > 0 and h[10] > 0 and lo.cpu().numpy()[9] == 0
    assert h[11] == 1.0 and lo.cpu().numpy()[11] == 0


@pytest.mark.parametrize("M,K,N", [(128, 128, 128), (1000, 256, 256), (4096, 512, 512), (300, 1024, 1024),
                                   (4099, 32, 512), (1000, 32, 1024), (77, 32, 256)])
def test_forward_bias_relu(M, K, N):
    f = ffi()
    g = torch.Generator(device="cuda").manual_seed(M + K + N)
    x = torch.randn(M, K, device="cuda", generator=g).relu_()
    w = torch.randn(K, N, device="cuda", generator=g) / K ** 0.5
    b = torch.randn(N, device="cuda", generator=g) * 0.1
    xh, xl = split(x)
    wth, wtl = split(w.t().contiguous())
    yh, yl = torch.empty(M, N, device="cuda"), torch.empty(M, N, device="cuda")
    d = f.TcGemmDesc(kind=f.TC_FWD, a_hi=xh.data_ptr(), a_lo=xl.data_ptr(), b_hi=wth.data_ptr(),
                     b_lo=wtl.data_ptr(), m=M, n=N, k=K, bias=b.data_ptr(), c_hi=yh.data_ptr(),
                     c_lo=yl.data_ptr())
    run(d)
    want = np.maximum(x.double().cpu().numpy() @ w.double().cpu().numpy() + b.double().cpu().numpy(), 0)
    got = (yh.double() + yl.double()).cpu().numpy()
    assert rel_err(got, want) <= 1e-5
    assert np.array_equal(yh.cpu().numpy() > 0, got > 0)   # hi carries the ReLU mask


@pytest.mark.parametrize("M,Kout,Nin", [(1000, 512, 512), (256, 128, 128), (2048, 1024, 512)])
@pytest.mark.parametrize("kind", ["dx", "dx_f32"])
def test_dx_mask_colsum(M, Kout, Nin, kind):
    """dZ_prev = (dY W^T) * [act > 0] with W [Nin x Kout]; column sums = bias grad."""
    f = ffi()
    g = torch.Generator(device="cuda").manual_seed(M + Kout + Nin)
    dy = torch.randn(M, Kout, device="cuda", generator=g) * 1e-3
    w = torch.randn(Nin, Kout, device="cuda", generator=g) / Kout ** 0.5
    act = torch.randn(M, Nin, device="cuda", generator=g).relu_()
    ah, _ = split(act)
    dyh, dyl = split(dy)
    wh, wl = split(w)
    out_h = torch.empty(M, Nin, device="cuda")
    out_l = torch.empty(M, Nin, device="cuda")
    desc = f.TcGemmDesc(kind=f.TC_DX if kind == "dx" else f.TC_DX_F32, a_hi=dyh.data_ptr(),
                        a_lo=dyl.data_ptr(), b_hi=wh.data_ptr(), b_lo=wl.data_ptr(), m=M, n=Nin,
                        k=Kout, mask=ah.data_ptr(), c_hi=out_h.data_ptr(),
                        c_lo=out_l.data_ptr() if kind == "dx" else None)
    grid = ctypes.c_int32()
    f.call("spo_tc_gemm_shape", ctypes.byref(desc), ctypes.byref(grid), None)
    cs = torch.full((grid.value, Nin), float("nan"), device="cuda")
    desc.colsum = cs.data_ptr()
    run(desc)
    want = (dy.double() @ w.double().t()).cpu().numpy() * (act.cpu().numpy() > 0)
    got = (out_h.double() + (out_l.double() if kind == "dx" else 0)).cpu().numpy()
    assert rel_err(got, want) <= 1e-5
    assert np.all(got[act.cpu().numpy() <= 0] == 0)
    assert rel_err(cs.double().sum(0).cpu().numpy(), want.sum(0)) <= 1e-5


def pack_mask(m):
    """[M x N] bool -> [M x N/32] uint32, bit j of word w = column 32 w + j."""
    return np.packbits(np.asarray(m, bool), axis=1, bitorder="little").view(np.uint32)


@pytest.mark.parametrize("M,K,N", [(1000, 256, 256), (4096, 512, 512), (300, 1024, 1024), (4099, 32, 512),
                                   (1000, 32, 1024)])
def test_forward_writes_packed_relu_mask(M, K, N):
    f = ffi()
    g = torch.Generator(device="cuda").manual_seed(7 * M + K)
    x = torch.randn(M, K, device="cuda", generator=g).relu_()
    w = torch.randn(K, N, device="cuda", generator=g) / K ** 0.5
    b = torch.randn(N, device="cuda", generator=g) * 0.1
    xh, xl = split(x)
    wth, wtl = split(w.t().contiguous())
    yh, yl = torch.empty(M, N, device="cuda"), torch.empty(M, N, device="cuda")
    bits = torch.full((M + 1, N // 32), -1, dtype=torch.int32, device="cuda")  # + a guard row
    d = f.TcGemmDesc(kind=f.TC_FWD, a_hi=xh.data_ptr(), a_lo=xl.data_ptr(), b_hi=wth.data_ptr(),
                     b_lo=wtl.data_ptr(), m=M, n=N, k=K, bias=b.data_ptr(), c_hi=yh.data_ptr(),
                     c_lo=yl.data_ptr(), c_bits=bits.data_ptr())
    run(d)
    got = bits.cpu().numpy().view(np.uint32)
    assert np.array_equal(got[:M], pack_mask(yh.cpu().numpy() > 0))
    assert np.all(got[M] == 0xFFFFFFFF)


@pytest.mark.parametrize("M,Kout,Nin", [(1000, 512, 512), (2048, 1024, 512), (129, 128, 256)])
@pytest.mark.parametrize("kind", ["dx", "dx_f32"])
def test_dx_packed_mask_equals_float_mask(M, Kout, Nin, kind):
    """The dX epilogue reading the packed mask gives bit-identical outputs and column sums."""
    f = ffi()
    g = torch.Generator(device="cuda").manual_seed(M + 3 * Kout + Nin)
    dy = torch.randn(M, Kout, device="cuda", generator=g) * 1e-3
    w = torch.randn(Nin, Kout, device="cuda", generator=g) / Kout ** 0.5
    act = torch.randn(M, Nin, device="cuda", generator=g).relu_()
    ah, _ = split(act)
    bits = torch.from_numpy(pack_mask(ah.cpu().numpy() > 0).view(np.int32)).cuda()
    dyh, dyl = split(dy)
    wh, wl = split(w)
    outs = []
    for use_bits in (False, True):
        out_h = torch.full((M, Nin), float("nan"), device="cuda")
        out_l = torch.full((M, Nin), float("nan"), device="cuda")
        desc = f.TcGemmDesc(kind=f.TC_DX if kind == "dx" else f.TC_DX_F32, a_hi=dyh.data_ptr(),
                            a_lo=dyl.data_ptr(), b_hi=wh.data_ptr(), b_lo=wl.data_ptr(), m=M, n=Nin,
                            k=Kout, mask=None if use_bits else ah.data_ptr(),
                            mask_bits=bits.data_ptr() if use_bits else None, c_hi=out_h.data_ptr(),
                            c_lo=out_l.data_ptr() if kind == "dx" else None)
        grid = ctypes.c_int32()
        f.call("spo_tc_gemm_shape", ctypes.byref(desc), ctypes.byref(grid), None)
        cs = torch.full((grid.value, Nin), float("nan"), device="cuda")
        desc.colsum = cs.data_ptr()
        run(desc)
        outs.append((out_h.cpu(), out_l.cpu() if kind == "dx" else None, cs.cpu()))
    (h0, l0, c0), (h1, l1, c1) = outs
    assert torch.equal(h0, h1) and torch.equal(c0, c1)
    if kind == "dx":
        assert torch.equal(l0, l1)


@pytest.mark.parametrize("rows,Kin,N,chunk", [(4096, 512, 512, 1024), (1000, 128, 128, 256),
                                               (65536, 256, 256, 4096), (777, 1024, 1024, 224)])
def test_dw_split_partials(rows, Kin, N, chunk):
    """dW = act^T dZ from row-major act [rows x Kin] and dZ [rows x N] (both MN-major
    operands), rows split in chunks, one partial per chunk."""
    f = ffi()
    g = torch.Generator(device="cuda").manual_seed(rows + Kin)
    act = torch.randn(rows, Kin, device="cuda", generator=g).relu_()
    dz = torch.randn(rows, N, device="cuda", generator=g) * 1e-4
    ah, al = split(act)
    zh, zl = split(dz)
    splits = -(-rows // chunk)
    part = torch.full((splits, Kin, N), float("nan"), device="cuda")
    d = f.TcGemmDesc(kind=f.TC_DW, a_hi=ah.data_ptr(), a_lo=al.data_ptr(), b_hi=zh.data_ptr(),
                     b_lo=zl.data_ptr(), m=Kin, n=N, k=rows, k_chunk=chunk, c_part=part.data_ptr())
    grid, sp = run(d)
    assert sp == splits
    want = act.double().t().cpu().numpy() @ dz.double().cpu().numpy()
    got = part.double().sum(0).cpu().numpy()
    assert rel_err(got, want) <= 1e-5


@pytest.mark.parametrize("M,K,N", [(1000, 256, 256), (4096, 512, 512), (300, 1024, 1024), (777, 32, 128)])
def test_forward_plain_fp32_operand_equals_presplit(M, K, N):
    """A given as plain fp32 (a_lo NULL: split in shared memory by the kernel) and the
    output written as plain fp32 with its packed ReLU mask: bit-identical to the same
    product from A split beforehand by spo_split_tf32, and within 1e-5 of float64."""
    f = ffi()
    g = torch.Generator(device="cuda").manual_seed(11 * M + K)
    x = torch.randn(M, K, device="cuda", generator=g)
    if K > 32:
        x = x.relu_()
    w = torch.randn(K, N, device="cuda", generator=g) / K ** 0.5
    b = torch.randn(N, device="cuda", generator=g) * 0.1
    xh, xl = split(x)
    wth, wtl = split(w.t().contiguous())
    outs = []
    for raw in (True, False):
        y = torch.full((M, N), float("nan"), device="cuda")
        bits = torch.full((M + 1, N // 32), -1, dtype=torch.int32, device="cuda")  # + a guard row
        d = f.TcGemmDesc(kind=f.TC_FWD, a_hi=(x if raw else xh).data_ptr(), a_lo=None if raw else xl.data_ptr(),
                         b_hi=wth.data_ptr(), b_lo=wtl.data_ptr(), m=M, n=N, k=K, bias=b.data_ptr(),
                         c_hi=y.data_ptr(), c_bits=bits.data_ptr())
        run(d)
        outs.append((y.cpu(), bits.cpu().numpy().view(np.uint32)))
    (y1, b1), (y0, b0) = outs
    assert torch.equal(y1, y0) and np.array_equal(b1, b0)
    want = np.maximum(x.double().cpu().numpy() @ w.double().cpu().numpy() + b.double().cpu().numpy(), 0)
    assert rel_err(y1.numpy(), want) <= 1e-5
    assert np.array_equal(b1[:M], pack_mask(y1.numpy() > 0)) and np.all(b1[M] == 0xFFFFFFFF)


@pytest.mark.parametrize("M,Kout,Nin", [(1000, 512, 512), (2048, 1024, 512), (129, 128, 256)])
def test_dx_plain_fp32_operand_equals_presplit(M, Kout, Nin):
    f = ffi()
    g = torch.Generator(device="cuda").manual_seed(M + 5 * Kout + Nin)
    dy = torch.randn(M, Kout, device="cuda", generator=g) * 1e-3
    w = torch.randn(Nin, Kout, device="cuda", generator=g) / Kout ** 0.5
    act = torch.randn(M, Nin, device="cuda", generator=g).relu_()
    bits = torch.from_numpy(pack_mask(act.cpu().numpy() > 0).view(np.int32)).cuda()
    dyh, dyl = split(dy)
    wh, wl = split(w)
    outs = []
    for raw in (True, False):
        out = torch.full((M, Nin), float("nan"), device="cuda")
        desc = f.TcGemmDesc(kind=f.TC_DX_F32, a_hi=(dy if raw else dyh).data_ptr(),
                            a_lo=None if raw else dyl.data_ptr(), b_hi=wh.data_ptr(), b_lo=wl.data_ptr(),
                            m=M, n=Nin, k=Kout, mask_bits=bits.data_ptr(), c_hi=out.data_ptr())
        grid = ctypes.c_int32()
        f.call("spo_tc_gemm_shape", ctypes.byref(desc), ctypes.byref(grid), None)
        cs = torch.full((grid.value, Nin), float("nan"), device="cuda")
        desc.colsum = cs.data_ptr()
        run(desc)
        outs.append((out.cpu(), cs.cpu()))
    (o1, c1), (o0, c0) = outs
    assert torch.equal(o1, o0) and torch.equal(c1, c0)
    want = (dy.double() @ w.double().t()).cpu().numpy() * (act.cpu().numpy() > 0)
    assert rel_err(o1.numpy(), want) <= 1e-5


@pytest.mark.parametrize("rows,Kin,N,chunk", [(4096, 512, 512, 1024), (1000, 128, 128, 256),
                                               (65536, 256, 256, 4096), (777, 1024, 1024, 224)])
def test_dw_plain_fp32_operands_equal_presplit(rows, Kin, N, chunk):
    f = ffi()
    g = torch.Generator(device="cuda").manual_seed(3 * rows + Kin)
    act = torch.randn(rows, Kin, device="cuda", generator=g).relu_()
    dz = torch.randn(rows, N, device="cuda", generator=g) * 1e-4
    ah, al = split(act)
    zh, zl = split(dz)
    splits = -(-rows // chunk)
    parts = []
    for raw in (True, False):
        part = torch.full((splits, Kin, N), float("nan"), device="cuda")
        d = f.TcGemmDesc(kind=f.TC_DW, a_hi=(act if raw else ah).data_ptr(), a_lo=None if raw else al.data_ptr(),
                         b_hi=(dz if raw else zh).data_ptr(), b_lo=None if raw else zl.data_ptr(),
                         m=Kin, n=N, k=rows, k_chunk=chunk, c_part=part.data_ptr())
        run(d)
        parts.append(part.cpu())
    assert torch.equal(parts[0], parts[1])
    want = act.double().t().cpu().numpy() @ dz.double().cpu().numpy()
    assert rel_err(parts[0].double().sum(0).numpy(), want) <= 1e-5


def test_unsupported_shapes_are_rejected():
    f = ffi()
    d = f.TcGemmDesc(kind=f.TC_FWD, m=128, n=96, k=128)  # n not a multiple of 128
    with pytest.raises(f.SpoError) as e:
        f.call("spo_tc_gemm_shape", ctypes.byref(d), None, None)
    assert e.value.code == -7


def test_bounded_wait_runs_out_and_the_device_recovers():
    """The failure path of the kernel's bounded waits, without a fault: the operands of each
    CTA's first k-block are never loaded and every wait is limited to 2 ms
    (spo_tc_gemm_withheld). The MMA issuer's wait runs out; the kernel must drain, free its
    tensor memory, report a nonzero code in its error word and return; then a normal launch
    on the same device must be exact again."""
    import time
    f = ffi()
    M, K, N = 512, 64, 128
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(M, K, device="cuda", generator=g).relu_()
    w = torch.randn(K, N, device="cuda", generator=g) / K ** 0.5
    b = torch.zeros(N, device="cuda")
    xh, xl = split(x)
    wth, wtl = split(w.t().contiguous())
    yh, yl = torch.empty(M, N, device="cuda"), torch.empty(M, N, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    d = f.TcGemmDesc(kind=f.TC_FWD, a_hi=xh.data_ptr(), a_lo=xl.data_ptr(), b_hi=wth.data_ptr(),
                     b_lo=wtl.data_ptr(), m=M, n=N, k=K, bias=b.data_ptr(), c_hi=yh.data_ptr(),
                     c_lo=yl.data_ptr(), err=err.data_ptr())
    torch.cuda.synchronize()
    t0 = time.time()
    f.call("spo_tc_gemm_withheld", None, ctypes.byref(d), 2000)
    torch.cuda.synchronize()
    assert time.time() - t0 < 10.0
    code = int(err.item())
    assert code in (1, 2, 3, 4, 5), code  # a wait gave up (which role first is a race)
    with pytest.raises(f.SpoError, match="needs desc->err"):
        f.call("spo_tc_gemm_withheld", None, ctypes.byref(f.TcGemmDesc(
            kind=f.TC_FWD, a_hi=xh.data_ptr(), a_lo=xl.data_ptr(), b_hi=wth.data_ptr(), b_lo=wtl.data_ptr(),
            m=M, n=N, k=K, bias=b.data_ptr(), c_hi=yh.data_ptr(), c_lo=yl.data_ptr())), 2000)
    d.err = None
    run(d)                                 # the same launch without the withheld stage
    want = np.maximum(x.double().cpu().numpy() @ w.double().cpu().numpy(), 0)
    assert rel_err((yh.double() + yl.double()).cpu().numpy(), want) <= 1e-5
