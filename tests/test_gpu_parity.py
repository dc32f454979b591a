"""Parity of libdcfold.so (through its C ABI) with the oracle and with the
reference's golden vectors, on a B200.

Integer, byte and index results are compared bit for bit; float results are
compared bit for bit too (the fold must print the same literal), including
NaN payloads.  Every case also compares the all-or-nothing outcome: folded
or not, and the lowest refusing element.
"""
import numpy as np
import pytest

from golden_cases import case_id, check_case, element_cases

pytestmark = pytest.mark.gpu

CASES = element_cases()
SIZES = [1, 31, 32, 33, 127, 4097, 100003]
FLOATS = ["f16", "bf16", "f32", "f64", "f8E5M2", "f8E4M3", "f8E3M4"]
INTS = ["i1", "i8", "i16", "i32", "i64"]
ST = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}
SZ = {"i1": 1, "i8": 1, "i16": 2, "i32": 4, "i64": 8, "f16": 2, "bf16": 2, "f32": 4, "f64": 8,
      "f8E5M2": 1, "f8E4M3": 1, "f8E3M4": 1}
LAYOUT = {"f16": (5, 10), "bf16": (8, 7), "f32": (8, 23), "f64": (11, 52), "f8E5M2": (5, 2), "f8E4M3": (4, 3),
          "f8E3M4": (3, 4)}


def rbits(dt, n, seed, mode="mixed"):
    """Element storage with edge values: random bit patterns (NaN payloads,
    subnormals, infinities) mixed with ordinary values."""
    rng = np.random.default_rng(seed)
    st = ST[SZ[dt]]
    w = 8 * SZ[dt]
    if dt == "i1":
        return rng.integers(0, 2, n, dtype=np.uint8)
    raw = rng.integers(0, 1 << 63, n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, n, dtype=np.uint64)
    x = (raw & np.uint64((1 << w) - 1) if w < 64 else raw).astype(st)
    if dt in LAYOUT:
        e, m = LAYOUT[dt]
        bias = (1 << (e - 1)) - 1
        if mode != "raw":
            # ordinary values: exponent near the bias, so arithmetic is exercised
            k = n * 3 // 4
            ex = rng.integers(max(1, bias - 3), min((1 << e) - 1, bias + 4), k).astype(np.uint64)
            mant = rng.integers(0, 1 << m, k, dtype=np.uint64)
            sign = rng.integers(0, 2, k, dtype=np.uint64)
            x[:k] = ((sign << np.uint64(e + m)) | (ex << np.uint64(m)) | mant).astype(st)
            rng.shuffle(x)
        specials = [0, 1 << (e + m), ((1 << e) - 1) << m, (((1 << e) - 1) << m) | (1 << (e + m)),
                    (((1 << e) - 1) << m) | (1 << (m - 1)), 1, (1 << m) - 1]
        if mode == "nonan":
            expm = ((1 << e) - 1) << m
            bad = ((x.astype(np.uint64) & np.uint64(expm)) == np.uint64(expm))
            x[bad] = st(1 << m)
            specials = [s for s in specials if (s & (((1 << e) - 1) << m)) != (((1 << e) - 1) << m)]
    else:
        specials = [0, 1, (1 << w) - 1, 1 << (w - 1), (1 << (w - 1)) - 1]
    idx = rng.choice(n, size=min(n, max(1, n // 10)), replace=False)
    x[idx] = np.array(specials, dtype=np.uint64)[np.arange(len(idx)) % len(specials)].astype(st)
    return x


def same(f_gpu, f_cpu, n):
    assert f_gpu.folded == f_cpu.folded, (f_gpu.folded, f_cpu.folded, f_gpu.first_fail_index, f_cpu.first_fail_index)
    assert f_gpu.first_fail_index == f_cpu.first_fail_index
    if f_cpu.folded:
        a, b = f_gpu.out[:n], f_cpu.out[:n]
        if not np.array_equal(a, b):
            bad = np.nonzero(a != b)[0]
            i = int(bad[0])
            raise AssertionError(f"{len(bad)} mismatches; first at {i}: gpu {a[i]:#x} cpu {b[i]:#x}")
        assert f_gpu.is_splat == f_cpu.is_splat


@pytest.mark.parametrize("case", CASES, ids=[case_id(c) for c in CASES])
def test_golden_vectors(case, dcf):
    check_case(case, dcf)


FLOAT_BIN = ["addf", "subf", "mulf", "divf", "maximumf", "minimumf", "maxnumf", "minnumf"]


@pytest.mark.parametrize("dt", FLOATS)
@pytest.mark.parametrize("op", FLOAT_BIN)
def test_float_binary_vs_oracle(op, dt, dcf, oracle):
    for n in SIZES:
        a, b = rbits(dt, n, 1 + n), rbits(dt, n, 2 + n)
        same(dcf.binary(op, dt, a, b), oracle.binary(op, dt, a, b), n)
    n = 4097
    a, b = rbits(dt, n, 7), rbits(dt, 1, 8)
    same(dcf.binary(op, dt, a, b, rhs_splat=True), oracle.binary(op, dt, a, b, rhs_splat=True), n)
    same(dcf.binary(op, dt, b, a, lhs_splat=True), oracle.binary(op, dt, b, a, lhs_splat=True), n)
    same(dcf.binary(op, dt, b, b, lhs_splat=True, rhs_splat=True),
         oracle.binary(op, dt, b, b, lhs_splat=True, rhs_splat=True), 1)


@pytest.mark.parametrize("dt", ["f32", "f64", "f16", "bf16"])
@pytest.mark.parametrize("op", ["addf", "subf", "mulf", "divf"])
@pytest.mark.parametrize("mode", [1, 2, 3, 4])
def test_rounding_modes_vs_oracle(op, dt, mode, dcf, oracle):
    a, b = rbits(dt, 50000, 11 * mode), rbits(dt, 50000, 13 * mode)
    same(dcf.binary(op, dt, a, b, flags=mode), oracle.binary(op, dt, a, b, flags=mode), 50000)
    a, b = rbits(dt, 50000, 17 * mode, "nonan"), rbits(dt, 50000, 19 * mode, "nonan")
    same(dcf.binary(op, dt, a, b, flags=mode), oracle.binary(op, dt, a, b, flags=mode), 50000)


@pytest.mark.parametrize("dt", ["f32", "bf16", "f64"])
def test_negative_default_nan_flag(dt, dcf, oracle):
    inf = {"f32": 0x7F800000, "bf16": 0x7F80, "f64": 0x7FF0000000000000}[dt]
    a = np.array([inf, 0, inf], dtype=ST[SZ[dt]])
    b = np.array([inf, 0, 1], dtype=ST[SZ[dt]])
    for fl in (0, 1 << 16):
        for op in ("subf", "divf", "mulf"):
            same(dcf.binary(op, dt, a, b, flags=fl), oracle.binary(op, dt, a, b, flags=fl), 3)


INT_BIN = ["addi", "subi", "muli", "andi", "ori", "xori", "shli", "shrui", "shrsi", "divsi", "divui", "remsi",
           "remui", "maxsi", "maxui", "minsi", "minui"]


@pytest.mark.parametrize("dt", INTS)
@pytest.mark.parametrize("op", INT_BIN)
def test_int_binary_vs_oracle(op, dt, dcf, oracle):
    w = 1 if dt == "i1" else 8 * SZ[dt]
    for n in SIZES:
        a, b = rbits(dt, n, 3 + n), rbits(dt, n, 4 + n)
        same(dcf.binary(op, dt, a, b), oracle.binary(op, dt, a, b), n)
        # refusal-free operands so the values themselves are compared
        if op.startswith("sh"):
            b = (b.astype(np.uint64) % np.uint64(w)).astype(b.dtype)
        if op in ("divsi", "divui", "remsi", "remui"):
            b = np.where(b == 0, b.dtype.type(1), b)
            if op == "divsi":
                imin = b.dtype.type(1 << (w - 1)) if w > 1 else b.dtype.type(1)
                neg1 = b.dtype.type((1 << w) - 1) if w < 64 else b.dtype.type(0xFFFFFFFFFFFFFFFF)
                b = np.where((a == imin) & (b == neg1), b.dtype.type(1), b)
        same(dcf.binary(op, dt, a, b), oracle.binary(op, dt, a, b), n)
    a, b = rbits(dt, 4097, 9), rbits(dt, 1, 10)
    same(dcf.binary(op, dt, a, b, rhs_splat=True), oracle.binary(op, dt, a, b, rhs_splat=True), 4097)


@pytest.mark.parametrize("dt", INTS)
@pytest.mark.parametrize("pred", range(10))
def test_cmpi_vs_oracle(pred, dt, dcf, oracle):
    a, b = rbits(dt, 4097, 20 + pred), rbits(dt, 4097, 40 + pred)
    b[::3] = a[::3]
    fl = pred << 8
    same(dcf.binary("cmpi", dt, a, b, flags=fl), oracle.binary("cmpi", dt, a, b, flags=fl), 4097)


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32", "f64"])
@pytest.mark.parametrize("pred", range(16))
def test_cmpf_vs_oracle(pred, dt, dcf, oracle):
    a, b = rbits(dt, 4097, 60 + pred), rbits(dt, 4097, 80 + pred)
    b[::3] = a[::3]
    fl = pred << 8
    same(dcf.binary("cmpf", dt, a, b, flags=fl), oracle.binary("cmpf", dt, a, b, flags=fl), 4097)


@pytest.mark.parametrize("src", FLOATS)
@pytest.mark.parametrize("dst", FLOATS)
def test_float_convert_vs_oracle(src, dst, dcf, oracle):
    if src == dst:
        pytest.skip("same type")
    op = "extf" if SZ[dst] >= SZ[src] else "truncf"
    for seed, mode in ((1, "mixed"), (2, "raw"), (3, "nonan")):
        x = rbits(src, 20011, seed, mode)
        same(dcf.convert(op, src, dst, x), oracle.convert(op, src, dst, x), len(x))
    # mostly-representable input so the fold succeeds and values are compared
    y = oracle.convert("extf" if op == "truncf" else "truncf", dst, src, rbits(dst, 20011, 4, "nonan"))
    if y.folded:
        same(dcf.convert(op, src, dst, y.out), oracle.convert(op, src, dst, y.out), 20011)
    # every element exactly representable
    ok_vals = []
    for v in rbits(src, 3000, 5, "raw"):
        ok, _ = oracle.float_convert_bits(src, dst, int(v))
        if ok:
            ok_vals.append(int(v))
    if ok_vals:
        z = np.array(ok_vals, dtype=ST[SZ[src]])
        fg, fc = dcf.convert(op, src, dst, z), oracle.convert(op, src, dst, z)
        assert fc.folded
        same(fg, fc, len(z))


@pytest.mark.parametrize("idt", INTS)
@pytest.mark.parametrize("fdt", FLOATS)
def test_int_float_casts_vs_oracle(idt, fdt, dcf, oracle):
    x = rbits(idt, 20011, 31)
    for op in ("sitofp", "uitofp"):
        same(dcf.convert(op, idt, fdt, x), oracle.convert(op, idt, fdt, x), len(x))
    for seed, mode in ((32, "mixed"), (33, "nonan")):
        y = rbits(fdt, 20011, seed, mode)
        for op in ("fptosi", "fptoui"):
            same(dcf.convert(op, fdt, idt, y), oracle.convert(op, fdt, idt, y), len(y))
    # in-range values: the fold succeeds
    w = 1 if idt == "i1" else 8 * SZ[idt]
    vals = oracle.convert("sitofp", idt, fdt, rbits(idt, 20011, 34)).out
    fs = oracle.convert("fptosi", fdt, idt, vals)
    if fs.folded:
        same(dcf.convert("fptosi", fdt, idt, vals), fs, len(vals))
    del w


@pytest.mark.parametrize("dt", FLOATS)
def test_reciprocal_vs_oracle(dt, dcf, oracle):
    for n in SIZES:
        x = rbits(dt, n, 50 + n)
        same(dcf.reciprocal(dt, x), oracle.reciprocal(dt, x), n)
    x = rbits(dt, 1, 99)
    same(dcf.reciprocal(dt, x, n=1, splat=True), oracle.reciprocal(dt, x, n=1, splat=True), 1)


@pytest.mark.parametrize("n", [0, 1, 7, 8, 9, 4096, 100003])
def test_hex_codec(n, dcf, oracle):
    rng = np.random.default_rng(n)
    data = bytes(rng.integers(0, 256, n, dtype=np.uint8))
    enc = dcf.hex_encode(data)
    assert enc == oracle.hex_encode(data)
    assert dcf.hex_decode(enc) == data
    assert dcf.hex_decode(enc.lower()) == data


def test_hex_decode_rejects_bad_digit(dcf):
    with pytest.raises(dcf.DcfError) as e:
        dcf.hex_decode(b"00FFG1")
    assert e.value.code == -7
    with pytest.raises(dcf.DcfError):
        dcf.hex_decode(b"ABC")


@pytest.mark.parametrize("es", [1, 2, 4, 8])
def test_splat_check(es, dcf):
    x = np.full(10007, 5, dtype=ST[es])
    assert dcf.splat_check(x)
    x[9000] = 6
    assert not dcf.splat_check(x)


@pytest.mark.parametrize("shape", [(64, 64), (128, 192), (1, 1), (33, 65), (1000, 3), (3, 1000), (257, 129)])
@pytest.mark.parametrize("es", [1, 2, 4, 8])
def test_transpose2d(shape, es, dcf, oracle):
    rng = np.random.default_rng(es)
    x = rng.integers(0, 255, size=shape[0] * shape[1] * es, dtype=np.uint8).view(ST[es]).reshape(shape)
    f = dcf.transpose(x, shape, (1, 0))
    assert f.folded
    assert np.array_equal(f.out, oracle.transpose(x, shape, (1, 0)))
    assert np.array_equal(f.out, x.T)


@pytest.mark.parametrize("perms", [(0, 2, 1), (2, 1, 0), (1, 0, 2), (2, 0, 1), (1, 2, 0), (0, 1, 2)])
def test_transpose_nd(perms, dcf, oracle):
    rng = np.random.default_rng(3)
    shape = (6, 35, 17)
    x = rng.integers(0, 1 << 16, size=shape, dtype=np.uint16)
    f = dcf.transpose(x, shape, perms)
    assert np.array_equal(f.out, np.transpose(x, perms))
    assert np.array_equal(f.out, oracle.transpose(x, shape, perms))


def test_batch_vs_oracle(dcf, oracle):
    jobs = []
    for i in range(37):
        n = 1000 + 97 * i
        jobs.append({"op": "addf", "dtype": "f32", "lhs": rbits("f32", n, i), "rhs": rbits("f32", n, 100 + i)})
        jobs.append({"op": "divsi", "dtype": "i32", "lhs": rbits("i32", n, i), "rhs": rbits("i32", n, 200 + i)})
        jobs.append({"op": "reciprocal", "dtype": "bf16", "lhs": rbits("bf16", n, 300 + i)})
        jobs.append({"op": "truncf", "dtype": "f32", "out_dtype": "bf16", "lhs": rbits("f32", n, 400 + i) & np.uint32(0xFFFF0000)})
    res = dcf.batch(jobs)
    for j, r in zip(jobs, res):
        if j["op"] == "reciprocal":
            want = oracle.reciprocal(j["dtype"], j["lhs"])
        elif j["op"] == "truncf":
            want = oracle.convert("truncf", "f32", "bf16", j["lhs"])
        else:
            want = oracle.binary(j["op"], j["dtype"], j["lhs"], j["rhs"])
        same(r, want, len(j["lhs"]))


def test_host_pinned_and_pageable_agree(dcf, oracle):
    import torch
    n = 9_000_001
    a = torch.empty(n, dtype=torch.float32).pin_memory()
    b = torch.empty(n, dtype=torch.float32).pin_memory()
    o = torch.empty(n, dtype=torch.float32).pin_memory()
    a.numpy()[:] = np.random.default_rng(1).standard_normal(n).astype(np.float32)
    b.numpy()[:] = np.random.default_rng(2).standard_normal(n).astype(np.float32)
    f1 = dcf.binary("mulf", "f32", a.numpy(), b.numpy(), out=o.numpy().view(np.uint32))
    f2 = dcf.binary("mulf", "f32", a.numpy().copy(), b.numpy().copy())
    f3 = oracle.binary("mulf", "f32", a.numpy(), b.numpy())
    same(f1, f3, n)
    same(f2, f3, n)


TMA_CASES = [("binary", "addf", "f32", None), ("binary", "maximumf", "f32", None), ("binary", "mulf", "f64", None),
             ("binary", "divsi", "i32", None), ("binary", "addi", "i8", None), ("binary", "cmpf", "f32", 4 << 8),
             ("binary", "minnumf", "bf16", None), ("convert", "extf", "bf16", "f32"), ("convert", "sitofp", "i8", "f64"),
             ("convert", "truncf", "f32", "f16"), ("convert", "fptosi", "f64", "i16")]


@pytest.mark.parametrize("kind,op,dt,extra", TMA_CASES, ids=[f"{c[1]}-{c[2]}" for c in TMA_CASES])
def test_bulk_copy_path_vs_oracle(kind, op, dt, extra, dcf, oracle):
    """Large enough for the cp.async.bulk pipeline (>= 2 tiles of 16 KB per
    SM), with a ragged tail that is not a whole tile or vector."""
    n = (16384 // SZ[dt]) * 300 + 12345
    if kind == "binary":
        fl = extra or 0
        a, b = rbits(dt, n, 71, "nonan"), rbits(dt, n, 72, "nonan")
        if op == "divsi":   # nonzero divisors and no INT_MIN / -1 pair
            b = np.where((b == 0) | (b == b.dtype.type(0xFFFFFFFF)), b.dtype.type(3), b)
        same(dcf.binary(op, dt, a, b, flags=fl), oracle.binary(op, dt, a, b, flags=fl), n)
        s = rbits(dt, 1, 73, "nonan")
        if op == "divsi":
            s[:] = 7
        same(dcf.binary(op, dt, a, s, rhs_splat=True, flags=fl), oracle.binary(op, dt, a, s, rhs_splat=True, flags=fl), n)
        same(dcf.binary(op, dt, s, b, lhs_splat=True, n=n, flags=fl),
             oracle.binary(op, dt, s, b, lhs_splat=True, n=n, flags=fl), n)
        if op == "divsi":   # a refusal deep inside the tiled range, another in the tail
            b2 = b.copy()
            mid = n // 2 + 1
            b2[n - 5] = 0
            b2[mid] = 0
            g, c = dcf.binary(op, dt, a, b2), oracle.binary(op, dt, a, b2)
            assert not c.folded and c.first_fail_index == mid
            same(g, c, n)
    else:
        x = rbits(dt, n, 74, "nonan")
        if op == "truncf":
            x = oracle.convert("extf", "f16", "f32", rbits("f16", n, 75, "nonan")).out
        if op == "fptosi":
            x = oracle.convert("sitofp", "i16", "f64", rbits("i16", n, 76)).out
        same(dcf.convert(op, dt, extra, x), oracle.convert(op, dt, extra, x), n)


@pytest.mark.parametrize("op", ["muli", "shli", "shrui", "shrsi", "divsi", "divui", "remsi", "remui"])
def test_i8_lanes_exhaustive_and_i16_edges(op, dcf, oracle):
    # Every i8 pair (the lane-wise word path packs four per word and divides
    # through f32), then i16 pairs around the largest dividends and the
    # smallest divisors, where an inexact quotient would first show.
    x, y = np.meshgrid(np.arange(256, dtype=np.uint8), np.arange(256, dtype=np.uint8))
    a, b = x.ravel().copy(), y.ravel().copy()
    if op.startswith("sh"):
        b %= np.uint8(8)
    if op in ("divsi", "divui", "remsi", "remui"):
        b = np.where(b == 0, np.uint8(1), b)
        if op == "divsi":
            b = np.where((a == 0x80) & (b == 0xFF), np.uint8(1), b)
    same(dcf.binary(op, "i8", a, b), oracle.binary(op, "i8", a, b), a.size)
    # and with the refusals left in: the lowest refusing element
    a2, b2 = x.ravel().copy(), y.ravel().copy()
    same(dcf.binary(op, "i8", a2, b2), oracle.binary(op, "i8", a2, b2), a2.size)
    big = np.concatenate([np.arange(65536 - 512, 65536), np.arange(0, 512), np.arange(32768 - 256, 32768 + 256)])
    small = np.concatenate([np.arange(1, 300), np.arange(65536 - 300, 65536)])
    xa, yb = np.meshgrid(big.astype(np.uint16), small.astype(np.uint16))
    a, b = xa.ravel().copy(), yb.ravel().copy()
    if op.startswith("sh"):
        b %= np.uint16(16)
    if op == "divsi":
        b = np.where((a == 0x8000) & (b == 0xFFFF), np.uint16(1), b)
    same(dcf.binary(op, "i16", a, b), oracle.binary(op, "i16", a, b), a.size)


def i16_division_boundaries():
    """Every i16 divisor with the dividends next to its multiples (n d - 1,
    n d, n d + 1), where a quotient taken from a reciprocal is first wrong,
    as unsigned lanes and as signed lanes of all four sign combinations."""
    xs, ys = [], []
    for d in range(1, 65536):
        m = np.arange(0, 65536 // d + 2, dtype=np.int64) * d
        m = np.concatenate([m - 1, m, m + 1, [0, 1, 32767, 32768, 65535]])
        m = m[(m >= 0) & (m < 65536)]
        xs.append(m)
        ys.append(np.full(m.size, d))
    for d in range(1, 32769):
        m = np.arange(0, 32768 // d + 2, dtype=np.int64) * d
        m = np.concatenate([m - 1, m, m + 1])
        m = m[(m >= 0) & (m <= 32768)]
        for sd in (1, -1) if d < 32768 else (-1,):
            for sx in (1, -1):
                v = sx * m
                v = v[(v >= -32768) & (v <= 32767)]
                xs.append(v & 0xFFFF)
                ys.append(np.full(v.size, (sd * d) & 0xFFFF))
    return np.concatenate(xs).astype(np.uint16), np.concatenate(ys).astype(np.uint16)


@pytest.mark.parametrize("op", ["divsi", "divui", "remsi", "remui"])
def test_i16_lane_division_boundaries(op, dcf, oracle):
    a, b = i16_division_boundaries()
    if op == "divsi":
        b = np.where((a == 0x8000) & (b == 0xFFFF), np.uint16(1), b)
    for shift in (0, 1):  # every pair in both lanes of its word
        a2, b2 = np.roll(a, shift).copy(), np.roll(b, shift).copy()
        same(dcf.binary(op, "i16", a2, b2), oracle.binary(op, "i16", a2, b2), a2.size)
