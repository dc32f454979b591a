"""The remaining elementwise folds on a B200 against the oracle, bit for
bit: remf, the rounding divisions, the high product half and carry of the
*_extended ops, negf, flush_denormals, extsi / extui / trunci and select.
They are the same kernels and host paths as the configs' folds; random bit
patterns include NaN payloads, subnormals, infinities and integer edge
values."""
import numpy as np
import pytest

from test_gpu_parity import FLOATS, INTS, SIZES, SZ, rbits, same

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", FLOATS)
def test_remf_vs_oracle(dt, dcf, oracle):
    for n in SIZES:
        a, b = rbits(dt, n, 101 + n), rbits(dt, n, 202 + n)
        same(dcf.binary("remf", dt, a, b), oracle.binary("remf", dt, a, b), n)
    a, b = rbits(dt, 4097, 5), rbits(dt, 1, 6)
    same(dcf.binary("remf", dt, a, b, rhs_splat=True), oracle.binary("remf", dt, a, b, rhs_splat=True), 4097)


@pytest.mark.parametrize("dt", INTS)
@pytest.mark.parametrize("op", ["ceildivui", "ceildivsi", "floordivsi", "mulsi_hi", "mului_hi", "addui_carry"])
def test_more_int_binary_vs_oracle(op, dt, dcf, oracle):
    for n in SIZES:
        a, b = rbits(dt, n, 7 + n), rbits(dt, n, 8 + n)
        same(dcf.binary(op, dt, a, b), oracle.binary(op, dt, a, b), n)
        if "div" in op:
            # without zero divisors (and, for i1, without the refusing
            # minimum) so that values are compared, not only refusals
            b = np.where(b == 0, b.dtype.type(1), b)
            if dt == "i1":
                a = np.zeros_like(a)
            same(dcf.binary(op, dt, a, b), oracle.binary(op, dt, a, b), n)
    a, b = rbits(dt, 4097, 9), rbits(dt, 1, 10)
    same(dcf.binary(op, dt, a, b, rhs_splat=True), oracle.binary(op, dt, a, b, rhs_splat=True), 4097)


@pytest.mark.parametrize("dt", FLOATS)
@pytest.mark.parametrize("op", ["negf", "flush_denormals"])
def test_sign_ops_vs_oracle(op, dt, dcf, oracle):
    for n in SIZES:
        a = rbits(dt, n, 31 + n, "raw")
        same(dcf.convert(op, dt, dt, a), oracle.convert(op, dt, dt, a), n)


@pytest.mark.parametrize("src", INTS)
@pytest.mark.parametrize("dst", INTS)
def test_int_width_casts_vs_oracle(src, dst, dcf, oracle):
    ops = []
    if SZ[dst] > SZ[src] or (src == "i1" and dst != "i1"):
        ops = ["extsi", "extui"]
    elif SZ[dst] < SZ[src] or (dst == "i1" and src != "i1"):
        ops = ["trunci"]
    else:
        ops = ["trunci"]   # same width: index_cast between i64 and index
    for op in ops:
        for n in SIZES:
            a = rbits(src, n, 51 + n)
            same(dcf.convert(op, src, dst, a), oracle.convert(op, src, dst, a), n)


@pytest.mark.parametrize("es", [1, 2, 4, 8])
def test_select_vs_oracle(es, dcf, oracle):
    dt = {1: "i8", 2: "f16", 4: "f32", 8: "i64"}[es]
    for n in SIZES + [1 << 20]:
        c = rbits("i1", n, 61 + n)
        t, f = rbits(dt, n, 62 + n), rbits(dt, n, 63 + n)
        same(dcf.select(c, t, f), oracle.select(c, t, f), n)
    n = 4099
    c, t, f = rbits("i1", n, 1), rbits(dt, n, 2), rbits(dt, 1, 3)
    for cs, ts, fs in [(True, False, False), (False, True, False), (False, False, True), (True, True, True)]:
        cc, tt, ff = (c[:1] if cs else c), (t[:1] if ts else t), (f if fs else rbits(dt, n, 4))
        same(dcf.select(cc, tt, ff, n=n, cond_splat=cs, t_splat=ts, f_splat=fs),
             oracle.select(cc, tt, ff, n=n, cond_splat=cs, t_splat=ts, f_splat=fs), n)


def test_new_ops_through_the_device_api(dcf, oracle):
    import torch
    dev = torch.device("cuda:0")
    n = 1 << 20
    a, b = rbits("i32", n, 71), rbits("i32", n, 72)
    b = np.where(b == 0, np.uint32(3), b)
    ta, tb = (torch.from_numpy(x.view(np.int32)).to(dev) for x in (a, b))
    out = torch.empty_like(ta)
    st = torch.empty(16, dtype=torch.uint8, device=dev)
    for op in ("floordivsi", "ceildivsi", "mulsi_hi"):
        dcf.status_reset(st)
        dcf.binary_async(op, "i32", ta, tb, out, st)
        r = dcf.status_read(st)
        want = oracle.binary(op, "i32", a, b)
        assert r.folded == want.folded
        if want.folded:
            assert np.array_equal(out.cpu().numpy().view(np.uint32), want.out)
    c = torch.from_numpy(rbits("i1", n, 73)).to(dev)
    dcf.status_reset(st)
    dcf.select_async(c, ta, tb, out, st)
    assert dcf.status_read(st).folded
    want = oracle.select(c.cpu().numpy(), a, b)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.out)
