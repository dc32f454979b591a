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


def test_hex_decode_many(dcf, oracle):
    # Many literals in one launch, aligned and unaligned, against the
    # oracle's decoder; a bad digit in any piece is reported.
    import ctypes
    import torch
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(3)
    sizes = [0, 1, 7, 8, 9, 100, 4096, 65537, 1 << 20]
    raws = [rng.integers(0, 256, n, dtype=np.uint8) for n in sizes]
    texts = [oracle.hex_encode(r.tobytes()) for r in raws]
    offs, total = [], 0
    for i, t in enumerate(texts):
        total += (i % 3)                     # some pieces start unaligned
        offs.append(total)
        total += len(t) + 16
    blob = np.zeros(total, dtype=np.uint8)
    for o, t in zip(offs, texts):
        blob[o:o + len(t)] = np.frombuffer(t, dtype=np.uint8)
    dtext = torch.from_numpy(blob).to(dev)
    outs = [torch.zeros(max(1, len(r)), dtype=torch.uint8, device=dev) for r in raws]

    class Piece(ctypes.Structure):
        _fields_ = [("in_", ctypes.c_void_p), ("out", ctypes.c_void_p), ("nchars", ctypes.c_uint64)]
    arr = (Piece * len(raws))()
    for i, (o, t) in enumerate(zip(offs, texts)):
        arr[i].in_, arr[i].out, arr[i].nchars = dtext.data_ptr() + o, outs[i].data_ptr(), len(t)
    dpieces = torch.from_numpy(np.frombuffer(bytes(arr), dtype=np.uint8).copy()).to(dev)
    st = torch.empty(16, dtype=torch.uint8, device=dev)
    dcf.status_reset(st)
    assert dcf.lib().dcf_hex_decode_many_async(dpieces.data_ptr(), len(raws), max(len(t) for t in texts),
                                               st.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    assert dcf.status_read(st).folded
    for r, o in zip(raws, outs):
        assert np.array_equal(o.cpu().numpy()[:len(r)], r)
    blob2 = blob.copy()
    blob2[offs[5] + 17] = ord("g")
    dtext.copy_(torch.from_numpy(blob2))
    dcf.status_reset(st)
    assert dcf.lib().dcf_hex_decode_many_async(dpieces.data_ptr(), len(raws), max(len(t) for t in texts),
                                               st.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    assert not dcf.status_read(st).folded


@pytest.mark.parametrize("shape", [(8, 8), (64, 64), (72, 136), (136, 72), (1024, 8), (8, 1024), (2048, 4096),
                                   (4104, 520)])
def test_bulk_tensor_transpose(shape, dcf):
    # 2-byte transposes whose extents are multiples of 8 run as the TMA
    # pipeline (partial 64 x 64 edge tiles included); bit-exact against numpy.
    import torch
    rng = np.random.default_rng(shape[0] * 7 + shape[1])
    w = rng.integers(0, 1 << 16, shape, dtype=np.uint16)
    f = dcf.transpose(w, shape, (1, 0))
    assert np.array_equal(f.out, w.T)
    dev = torch.device("cuda:0")
    tin = torch.from_numpy(w.view(np.int16)).to(dev)
    tout = torch.empty(shape[1], shape[0], dtype=torch.int16, device=dev)
    st = torch.empty(16, dtype=torch.uint8, device=dev)
    dcf.status_reset(st)
    import ctypes
    sh = (ctypes.c_int64 * 2)(*shape)
    pm = (ctypes.c_int64 * 2)(1, 0)
    assert dcf.lib().dcf_permute_status_async(2, 2, sh, pm, tin.data_ptr(), tout.data_ptr(), st.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert dcf.status_read(st).folded
    assert np.array_equal(tout.cpu().numpy().view(np.uint16), w.T)


def test_permute_groups_take_the_transpose(dcf, oracle):
    # A rank-3 permutation that swaps two groups of dims is a 2-D transpose.
    x = np.arange(16 * 24 * 8, dtype=np.uint16).reshape(16, 24, 8)
    for perms in [(1, 2, 0), (2, 0, 1), (0, 2, 1)]:
        f = dcf.transpose(x, x.shape, perms)
        assert np.array_equal(f.out, oracle.transpose(x, x.shape, perms)), perms


def test_hash_many(dcf, oracle):
    import ctypes
    import torch
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(8)
    sizes = [0, 1, 7, 8, 9, 100, 4096, 65537, 1 << 20]
    blob = rng.integers(0, 256, sum(sizes) + 64 * len(sizes), dtype=np.uint8)
    d = torch.from_numpy(blob).to(dev)

    class Piece(ctypes.Structure):
        _fields_ = [("data", ctypes.c_void_p), ("nbytes", ctypes.c_uint64)]
    arr = (Piece * len(sizes))()
    offs, o = [], 0
    for i, n in enumerate(sizes):
        o += i % 5                  # unaligned starts too
        offs.append(o)
        arr[i].data, arr[i].nbytes = d.data_ptr() + o, n
        o += n + 8
    dp = torch.from_numpy(np.frombuffer(bytes(arr), dtype=np.uint8).copy()).to(dev)
    out = torch.empty(len(sizes), dtype=torch.int64, device=dev)
    assert dcf.lib().dcf_hash_many_async(dp.data_ptr(), len(sizes), max(sizes), out.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream) == 0
    got = out.cpu().numpy().view(np.uint64)
    for i, (o, n) in enumerate(zip(offs, sizes)):
        assert int(got[i]) == oracle.hash_bytes(blob[o:o + n].tobytes()), (i, n)


MATH_F = ["absf", "ceil", "floor", "roundeven", "round", "trunc", "sqrt", "rsqrt"]


@pytest.mark.parametrize("dt", FLOATS)
@pytest.mark.parametrize("op", MATH_F)
def test_math_float_unary_vs_oracle(op, dt, dcf, oracle):
    # Random bits refuse sqrt / rsqrt at the first negative element; the
    # same values with the sign cleared fold, so both outcomes are compared.
    sign = {1: 0x80, 2: 0x8000, 4: 0x80000000, 8: 0x8000000000000000}[SZ[dt]]
    for n in SIZES:
        for mode in ("mixed", "raw"):
            a = rbits(dt, n, 71 + n, mode)
            same(dcf.convert(op, dt, dt, a), oracle.convert(op, dt, dt, a), n)
            pos = a & a.dtype.type(~sign & ((1 << 8 * SZ[dt]) - 1))
            same(dcf.convert(op, dt, dt, pos), oracle.convert(op, dt, dt, pos), n)
    a = rbits(dt, 1, 9)
    same(dcf.convert(op, dt, dt, a, n=4097, splat=True), oracle.convert(op, dt, dt, a, n=4097, splat=True), 4097)


@pytest.mark.parametrize("dt", INTS)
@pytest.mark.parametrize("op", ["absi", "ctlz", "cttz", "ctpop"])
def test_math_int_unary_vs_oracle(op, dt, dcf, oracle):
    for n in SIZES:
        a = rbits(dt, n, 81 + n)
        same(dcf.convert(op, dt, dt, a), oracle.convert(op, dt, dt, a), n)


@pytest.mark.parametrize("dt", FLOATS)
def test_copysign_vs_oracle(dt, dcf, oracle):
    for n in SIZES:
        a, b = rbits(dt, n, 91 + n, "raw"), rbits(dt, n, 92 + n, "raw")
        same(dcf.binary("copysign", dt, a, b), oracle.binary("copysign", dt, a, b), n)


@pytest.mark.parametrize("dt", INTS)
def test_ipowi_vs_oracle(dt, dcf, oracle):
    for n in SIZES:
        a, b = rbits(dt, n, 93 + n), rbits(dt, n, 94 + n)
        # small exponents and bases too, where the powers do not wrap to 0
        small = (np.arange(n) % 7).astype(a.dtype)
        for x, y in [(a, b), (small, b), (a, small), (np.where(a == 0, a.dtype.type(3), a), b)]:
            same(dcf.binary("ipowi", dt, x, y), oracle.binary("ipowi", dt, x, y), n)


def _refusal_positions(n, te):
    return [0, 1, te - 1, te, 7 * te + 3, n // 3, n // 2 + 1, (n // te - 1) * te, (n // te) * te - 1,
            (n // te) * te, n - 1]


@pytest.mark.parametrize("dt", ["i32", "i8", "i64"])
def test_refusals_at_tile_boundaries_report_the_lowest_index(dt, dcf, oracle):
    # The bulk-copy kernel reduces each warp's lowest refusing index and
    # takes the minimum over all CTAs; the index it reports must be the
    # lowest wherever the refusals are.  One zero divisor at each position
    # (the first tile, tile boundaries, the middle, the last whole tile, the
    # ragged tail), then zero divisors everywhere from a point on, then 1%
    # random zeros.
    te = 16384 // SZ[dt]
    n = te * 1500 + 777
    a = rbits(dt, n, 301)
    b = rbits(dt, n, 302)
    b = np.where(b == 0, b.dtype.type(1), b)
    a = np.where(a == a.dtype.type(1 << (8 * SZ[dt] - 1)), a.dtype.type(5), a)   # no INT_MIN / -1
    for pos in _refusal_positions(n, te):
        b2 = b.copy()
        b2[pos] = 0
        g, c = dcf.binary("divsi", dt, a, b2), oracle.binary("divsi", dt, a, b2)
        assert not c.folded and c.first_fail_index == pos
        same(g, c, n)
    for start in (0, te * 700 + 5, n - 3):
        b2 = b.copy()
        b2[start:] = 0
        same(dcf.binary("remsi", dt, a, b2), oracle.binary("remsi", dt, a, b2), n)
    b2 = b.copy()
    b2[np.random.default_rng(5).integers(0, n, n // 100)] = 0
    same(dcf.binary("divui", dt, a, b2), oracle.binary("divui", dt, a, b2), n)
    # and a fold that folds, after the refusals, on the same buffers
    same(dcf.binary("divui", dt, a, b), oracle.binary("divui", dt, a, b), n)


def test_refused_conversion_reports_the_lowest_index_device_entry(dcf, oracle):
    # truncf refuses at its first inexact element; through the device entry
    # point, twice on the same status-reset buffers, and with the refusal
    # only in the last tile.
    import torch
    n = 4096 * 3000 + 11
    x = oracle.convert("extf", "f16", "f32", rbits("f16", n, 311, "nonan")).out
    for pos in (0, n // 2, (n // 4096 - 1) * 4096 + 1, n - 1):
        x2 = x.copy()
        x2[pos] = np.uint32(0x3F800001)       # 1 + 2^-23: not exact in f16
        c = oracle.convert("truncf", "f32", "f16", x2)
        assert not c.folded and c.first_fail_index == pos
        xt = torch.from_numpy(x2.view(np.int32)).cuda()
        out = torch.empty(n, dtype=torch.int16, device="cuda")
        st = torch.empty(2, dtype=torch.int64, device="cuda")
        for _ in range(2):
            dcf.status_reset(st)
            dcf.convert_async("truncf", "f32", "f16", xt, out, st)
            r = dcf.status_read(st)
            assert (r.folded, r.first_fail_index) == (False, pos)
