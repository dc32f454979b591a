"""The oracle against independent arithmetic (CPU): numpy's IEEE-754 float
ops and casts, Python integers, exact rationals for the directed rounding
modes, binascii for the hex codec, numpy for permutations.

These pin the parts of the restatement that the reference's golden vectors
do not reach (large arrays, subnormals, every integer width, bf16).
"""
import binascii
from fractions import Fraction

import numpy as np
import pytest

from mlirpass_b200.workloads import splitmix64

rng = np.random.default_rng(1234)


def rand_f32(n, special=True):
    x = rng.standard_normal(n).astype(np.float32) * np.float32(100.0)
    b = x.view(np.uint32).copy()
    if special:
        k = n // 16
        idx = rng.choice(n, size=6 * k, replace=False)
        b[idx[:k]] = 0x7F800000                    # +inf
        b[idx[k:2 * k]] = 0xFF800000               # -inf
        b[idx[2 * k:3 * k]] = rng.integers(1, 1 << 23, size=k, dtype=np.uint32)  # denormals
        b[idx[3 * k:4 * k]] = 0                    # +0
        b[idx[4 * k:5 * k]] = 0x80000000           # -0
        b[idx[5 * k:6 * k]] = 0x7F7FFFFF           # max
    return b.view(np.float32)


def qnan_mask(bits, e, m):
    expm = ((1 << e) - 1) << m
    return ((bits & expm) == expm) & ((bits & ((1 << m) - 1)) != 0)


@pytest.mark.parametrize("op", ["addf", "subf", "mulf", "divf"])
def test_f32_arith_matches_numpy(op, oracle):
    a, b = rand_f32(20000), rand_f32(20000)
    with np.errstate(all="ignore"):
        ref = {"addf": a + b, "subf": a - b, "mulf": a * b, "divf": a / b}[op]
    f = oracle.binary(op, "f32", a, b)
    assert f.folded
    got = f.out.view(np.uint32)
    refb = ref.view(np.uint32)
    nan = np.isnan(ref)
    assert np.array_equal(got[~nan], refb[~nan])
    # invalid operations give the positive default quiet NaN
    assert np.all(got[nan] == 0x7FC00000)
    f2 = oracle.binary(op, "f32", a, b, flags=1 << 16)
    assert np.all(f2.out.view(np.uint32)[nan] == 0xFFC00000)


@pytest.mark.parametrize("op", ["addf", "subf", "mulf", "divf"])
def test_f64_and_f16_arith_match_numpy(op, oracle):
    with np.errstate(all="ignore"):
        a = rng.standard_normal(5000) * 1e3
        b = rng.standard_normal(5000) * 1e-3
        b[::50] = 0.0
        ref = {"addf": a + b, "subf": a - b, "mulf": a * b, "divf": a / b}[op]
        f = oracle.binary(op, "f64", a, b)
        assert np.array_equal(f.out.view(np.uint64), ref.view(np.uint64))
        h1 = (rng.standard_normal(5000) * 30).astype(np.float16)
        h2 = (rng.standard_normal(5000) * 30).astype(np.float16)
        h2[::40] = np.float16(0)
        hr = {"addf": h1 + h2, "subf": h1 - h2, "mulf": h1 * h2, "divf": h1 / h2}[op]
        fh = oracle.binary(op, "f16", h1, h2)
        hb = hr.view(np.uint16)
        nan = np.isnan(hr)
        assert np.array_equal(fh.out[~nan], hb[~nan])


def bf16_round(x32):
    u = x32.view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


@pytest.mark.parametrize("op", ["addf", "mulf", "divf"])
def test_bf16_arith_is_correctly_rounded(op, oracle):
    a = bf16_round((rng.standard_normal(5000) * 10).astype(np.float32))
    b = bf16_round((rng.standard_normal(5000) * 10).astype(np.float32))
    af = (a.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    bf = (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    with np.errstate(all="ignore"):
        exact = {"addf": af + bf, "mulf": af * bf, "divf": af / bf}[op]  # f64: exact or 53-bit
    # round f64 -> f32 -> bf16 is safe here (no ties created at f32 for these magnitudes is not
    # guaranteed), so round directly from the double with integer arithmetic.
    want = []
    for v in exact:
        want.append(int(oracle.lib().dco_round_from_double(17, float(v))))
    f = oracle.binary(op, "bf16", a, b)
    assert [int(x) for x in f.out] == want


def directed(q: Fraction, mode: str):
    """Exact directed rounding of a rational to f32 (normal range only)."""
    x = float(q)
    f = np.float32(x)
    fq = Fraction(float(f))
    if fq == q:
        return f
    up = np.nextafter(f, np.float32(np.inf)) if fq < q else f
    dn = f if fq < q else np.nextafter(f, np.float32(-np.inf))
    if mode == "down":
        return dn
    if mode == "up":
        return up
    return dn if q > 0 else up   # toward zero


@pytest.mark.parametrize("op", ["addf", "subf", "mulf", "divf"])
@pytest.mark.parametrize("mode,code", [("down", 1), ("up", 2), ("zero", 3)])
def test_f32_directed_rounding(op, mode, code, oracle):
    a = (rng.standard_normal(400) * 10).astype(np.float32)
    b = (rng.standard_normal(400) * 10).astype(np.float32)
    f = oracle.binary(op, "f32", a, b, flags=code)
    assert f.folded
    for x, y, got in zip(a, b, f.out.view(np.float32)):
        qa, qb = Fraction(float(x)), Fraction(float(y))
        q = {"addf": qa + qb, "subf": qa - qb, "mulf": qa * qb, "divf": qa / qb}[op]
        assert got == directed(q, mode), (op, mode, x, y)


def test_nearest_away_refuses_inexact_only(oracle):
    a = np.array([1.0, 1.0], np.float32)
    b = np.array([2.0, 3.0], np.float32)
    f = oracle.binary("addf", "f32", a, b, flags=4)
    assert f.folded                        # both sums exact
    a2 = np.array([1.0, 1.0000001], np.float32)
    f2 = oracle.binary("mulf", "f32", a2, np.array([3.0, 3.0], np.float32), flags=4)
    assert not f2.folded and f2.first_fail_index == 1


def test_minmax_rules(oracle):
    qnan, snan = 0x7FC00001, 0x7F800001
    a = np.array([0x80000000, 0, qnan, 0x3F800000, snan, 0x3F800000], np.uint32)
    b = np.array([0, 0x80000000, 0x3F800000, qnan, 0x3F800000, snan], np.uint32)
    mx = oracle.binary("maximumf", "f32", a, b).out
    mn = oracle.binary("minimumf", "f32", a, b).out
    mxn = oracle.binary("maxnumf", "f32", a, b).out
    assert list(mx) == [0, 0, qnan, qnan, snan | 0x400000, snan | 0x400000]
    assert list(mn) == [0x80000000, 0x80000000, qnan, qnan, snan | 0x400000, snan | 0x400000]
    # *numf: a quiet NaN loses to the number, a signalling one wins quieted
    assert list(mxn) == [0, 0, 0x3F800000, 0x3F800000, snan | 0x400000, snan | 0x400000]


WIDTHS = {"i8": (np.int8, 8), "i16": (np.int16, 16), "i32": (np.int32, 32), "i64": (np.int64, 64)}
STORAGE_OF = {"i1": np.uint8, "i8": np.uint8, "i16": np.uint16, "i32": np.uint32, "i64": np.uint64,
              "f16": np.uint16, "bf16": np.uint16, "f32": np.uint32, "f64": np.uint64}


def ints(dt, n, seed):
    t, w = WIDTHS[dt]
    r = splitmix64(seed, n)
    v = (r & np.uint64((1 << w) - 1)).astype(np.dtype(t).str.replace("i", "u")).view(t)
    edge = np.array([np.iinfo(t).min, np.iinfo(t).max, -1, 0, 1], dtype=t)
    v[::7] = edge[(np.arange(len(v[::7])) % 5)]
    return v


def py_int_op(op, a, b, w):
    m = (1 << w) - 1
    ua, ub = a & m, b & m
    sa = ua - (1 << w) if ua >> (w - 1) else ua
    sb = ub - (1 << w) if ub >> (w - 1) else ub
    if op == "addi": return (ua + ub) & m
    if op == "subi": return (ua - ub) & m
    if op == "muli": return (ua * ub) & m
    if op == "andi": return ua & ub
    if op == "ori": return ua | ub
    if op == "xori": return ua ^ ub
    if op in ("shli", "shrui", "shrsi"):
        if ub >= w: return None
        if op == "shli": return (ua << ub) & m
        if op == "shrui": return ua >> ub
        return (sa >> ub) & m
    if op == "divsi":
        if ub == 0 or (sa == -(1 << (w - 1)) and sb == -1): return None
        q = abs(sa) // abs(sb)
        return (q if (sa < 0) == (sb < 0) else -q) & m
    if op == "divui":
        return None if ub == 0 else ua // ub
    if op == "remsi":
        if ub == 0: return None
        r = abs(sa) % abs(sb)
        return (r if sa >= 0 else -r) & m
    if op == "remui":
        return None if ub == 0 else ua % ub
    if op == "maxsi": return ua if sa > sb else ub
    if op == "minsi": return ua if sa < sb else ub
    if op == "maxui": return max(ua, ub)
    if op == "minui": return min(ua, ub)
    raise ValueError(op)


@pytest.mark.parametrize("dt", ["i8", "i16", "i32", "i64"])
@pytest.mark.parametrize("op", ["addi", "subi", "muli", "andi", "ori", "xori", "shli", "shrui", "shrsi",
                                "divsi", "divui", "remsi", "remui", "maxsi", "minsi", "maxui", "minui"])
def test_int_ops_match_python(op, dt, oracle):
    t, w = WIDTHS[dt]
    a, b = ints(dt, 700, 11), ints(dt, 700, 12)
    if op.startswith("sh"):
        b = (np.abs(b.astype(np.int64)) % w).astype(t)
    if op in ("divsi", "divui", "remsi", "remui"):
        b = np.where(b == 0, t(3), b).astype(t)
        if op == "divsi":
            b = np.where((a == np.iinfo(t).min) & (b == -1), t(2), b).astype(t)
    ua = [int(x) & ((1 << w) - 1) for x in a]
    ub = [int(x) & ((1 << w) - 1) for x in b]
    want = [py_int_op(op, x, y, w) for x, y in zip(ua, ub)]
    assert all(v is not None for v in want)
    f = oracle.binary(op, dt, a, b)
    assert f.folded
    assert [int(x) for x in f.out] == want


@pytest.mark.parametrize("dt", ["i8", "i32", "i64"])
def test_int_refusals(dt, oracle):
    t, w = WIDTHS[dt]
    a = np.array([5, np.iinfo(t).min, 7, 9], t)
    b = np.array([1, -1, 2, 0], t)
    f = oracle.binary("divsi", dt, a, b)
    assert not f.folded and f.first_fail_index == 1       # INT_MIN / -1
    f = oracle.binary("remsi", dt, a, b)
    assert not f.folded and f.first_fail_index == 3       # only the zero divisor refuses
    f = oracle.binary("remsi", dt, a[:3], b[:3])
    assert f.folded and int(f.out[1]) == 0                # INT_MIN % -1 folds to 0
    s = np.array([0, w - 1, w, 1], t)
    f = oracle.binary("shli", dt, a, s)
    assert not f.folded and f.first_fail_index == 2


def test_conversions_match_numpy(oracle):
    x = rand_f32(30000)
    xb = x.view(np.uint32)
    nan = np.isnan(x)
    h = x.astype(np.float16)
    exact16 = (h.astype(np.float32).view(np.uint32) == xb) & ~nan
    for i in np.nonzero(exact16)[0][:3000]:
        ok, r = oracle.float_convert_bits("f32", "f16", int(xb[i]))
        assert ok and r == int(h.view(np.uint16)[i])
    for i in np.nonzero(~exact16 & ~nan)[0][:3000]:
        ok, _ = oracle.float_convert_bits("f32", "f16", int(xb[i]))
        assert not ok
    # bf16: representable iff the low 16 bits are zero
    for b in [0x3F800000, 0x3F800001, 0x00010000, 0x00008000, 0x7F800000, 0x7FC00000, 0x7FA00000, 0x7FC00001]:
        ok, r = oracle.float_convert_bits("f32", "bf16", b)
        if b in (0x7FA00000,):
            assert not ok                       # signalling NaN refuses
        elif b & 0xFFFF:
            assert not ok
        else:
            assert ok and r == b >> 16
    # extf is always exact for non-NaN values
    hv = np.arange(0, 65536, 7, dtype=np.uint16)
    f = oracle.convert("extf", "f16", "f32", hv)
    hf = hv.view(np.float16)
    isn = np.isnan(hf)
    quiet = (hv & 0x200) != 0
    if np.all(~isn | quiet):
        assert f.folded
    ok_idx = ~isn
    # refusals stop the fold at a signalling NaN; compare on a NaN-free slice
    hv2 = hv[~isn]
    f2 = oracle.convert("extf", "f16", "f32", hv2)
    assert f2.folded
    assert np.array_equal(f2.out.view(np.float32), hv2.view(np.float16).astype(np.float32))
    del ok_idx


def test_int_float_casts_match_numpy(oracle):
    i32 = ints("i32", 20000, 5)
    f = oracle.convert("sitofp", "i32", "f32", i32)
    assert np.array_equal(f.out.view(np.float32), i32.astype(np.float32))
    i64 = ints("i64", 20000, 6)
    f = oracle.convert("sitofp", "i64", "f32", i64)
    assert np.array_equal(f.out.view(np.float32), i64.astype(np.float32))
    f = oracle.convert("sitofp", "i64", "f64", i64)
    assert np.array_equal(f.out.view(np.float64), i64.astype(np.float64))
    # non-f32 kinds round through f64 first (Rust `as f64`, then from_f64)
    f = oracle.convert("sitofp", "i64", "f16", i64)
    assert np.array_equal(f.out.view(np.float16), i64.astype(np.float64).astype(np.float16))
    u = ints("i32", 20000, 7).view(np.uint32)
    f = oracle.convert("uitofp", "i32", "f32", u)
    assert np.array_equal(f.out.view(np.float32), u.astype(np.float32))
    x = (rng.standard_normal(20000) * 1e6).astype(np.float32)
    f = oracle.convert("fptosi", "f32", "i32", x)
    assert f.folded
    assert np.array_equal(f.out.view(np.int32), np.trunc(x).astype(np.int32))
    bad = np.array([1.0, 2.5e9, 3.0], np.float32)
    f = oracle.convert("fptosi", "f32", "i32", bad)
    assert not f.folded and f.first_fail_index == 1
    f = oracle.convert("fptoui", "f32", "i32", np.array([0.0, -0.5, -1.0], np.float32))
    assert not f.folded and f.first_fail_index == 2      # -0.5 truncates to -0, allowed
    f = oracle.convert("fptosi", "f32", "i8", np.array([127.9, -128.9, 128.0], np.float32))
    assert not f.folded and f.first_fail_index == 2


def test_reciprocal_and_splat(oracle):
    x = rand_f32(5000, special=False)
    f = oracle.reciprocal("f32", x)
    with np.errstate(all="ignore"):
        assert np.array_equal(f.out.view(np.float32), np.float32(1.0) / x)
    assert oracle.splat_check(np.full(100, 7, np.uint32))
    assert not oracle.splat_check(np.arange(100, dtype=np.uint32))
    f = oracle.binary("addf", "f32", np.full(64, 1.0, np.float32), np.full(64, 2.0, np.float32))
    assert f.folded and f.is_splat


def test_hex_and_transpose(oracle):
    data = bytes(rng.integers(0, 256, 4099, dtype=np.uint8))
    enc = oracle.hex_encode(data)
    assert enc == binascii.hexlify(data).upper()
    assert oracle.hex_decode(enc) == data
    assert oracle.hex_decode(enc.lower()) == data
    x = rng.integers(0, 1 << 16, size=(3, 5, 7), dtype=np.uint16)
    for perms in [(1, 0, 2), (2, 1, 0), (0, 2, 1), (2, 0, 1)]:
        assert np.array_equal(oracle.transpose(x, x.shape, perms), np.transpose(x, perms))


def _sx(v, w):
    return v - (1 << w) if v >> (w - 1) else v


def _py_more(op, a, b, w):
    """Python-integer statement of the rounding divisions, the high product
    half and the addui carry (exact arithmetic, then the range check)."""
    m = (1 << w) - 1
    sa, sb = _sx(a, w), _sx(b, w)
    lo, hi = -(1 << (w - 1)), (1 << (w - 1)) - 1
    if op == "ceildivui":
        return None if b == 0 else -(-a // b) & m
    if op in ("ceildivsi", "floordivsi"):
        if b == 0:
            return None
        q = -((-sa) // sb) if op == "ceildivsi" else sa // sb
        if op == "ceildivsi" and sa != 0 and (sa == lo or sb == lo):
            return None                      # an overflowing step of :557-595
        if not lo <= q <= hi:
            return None
        return q & m
    if op == "mulsi_hi":
        return ((sa * sb) >> w) & m
    if op == "mului_hi":
        return ((a * b) >> w) & m
    if op == "addui_carry":
        return int(((a + b) & m) < a)
    raise ValueError(op)


@pytest.mark.parametrize("dt", ["i1", "i8", "i16", "i32", "i64"])
@pytest.mark.parametrize("op", ["ceildivui", "ceildivsi", "floordivsi", "mulsi_hi", "mului_hi", "addui_carry"])
def test_more_int_ops_match_python(op, dt, oracle):
    w = {"i1": 1, "i8": 8, "i16": 16, "i32": 32, "i64": 64}[dt]
    m = (1 << w) - 1
    rng = np.random.default_rng(5)
    vals = [0, 1, m, m - 1, 1 << (w - 1), (1 << (w - 1)) - 1] if w > 1 else [0, 1]
    pairs = [(x, y) for x in vals for y in vals]
    pairs += [(int(x) & m, int(y) & m) for x, y in rng.integers(0, 2**63, (400, 2), dtype=np.uint64)]
    st = STORAGE_OF[dt]
    for x, y in pairs:
        want = _py_more(op, x, y, w)
        f = oracle.binary(op, dt, np.array([x], st), np.array([y], st))
        if want is None:
            assert not f.folded, (op, dt, x, y)
        else:
            assert f.folded and int(f.out[0]) == want, (op, dt, x, y, int(f.out[0]), want)


def test_ext_trunc_negf_flush(oracle):
    x = np.array([0, 1, 0x7F, 0x80, 0xFF], np.uint8)
    assert list(oracle.convert("extsi", "i8", "i32", x).out) == [0, 1, 0x7F, 0xFFFFFF80, 0xFFFFFFFF]
    assert list(oracle.convert("extui", "i8", "i32", x).out) == [0, 1, 0x7F, 0x80, 0xFF]
    assert list(oracle.convert("extsi", "i1", "i8", np.array([0, 1], np.uint8)).out) == [0, 0xFF]
    y = np.array([0x12345678, 0xFFFFFF80], np.uint32)
    assert list(oracle.convert("trunci", "i32", "i8", y).out) == [0x78, 0x80]
    f = np.array([0x3F800000, 0x80000000, 0x7FC00001, 0x00000001, 0x807FFFFF, 0x00800000], np.uint32)
    assert list(oracle.convert("negf", "f32", "f32", f).out) == [0xBF800000, 0, 0xFFC00001, 0x80000001, 0x007FFFFF,
                                                                 0x80800000]
    assert list(oracle.convert("flush_denormals", "f32", "f32", f).out) == [0x3F800000, 0x80000000, 0x7FC00001, 0,
                                                                            0x80000000, 0x00800000]


@pytest.mark.parametrize("dt", ["f32", "f64", "f16", "bf16"])
def test_remf_matches_fmod(dt, oracle):
    import math
    rng = np.random.default_rng(9)
    if dt in ("f32", "f64"):
        npt = {"f32": np.float32, "f64": np.float64}[dt]
        a = (rng.standard_normal(3000) * 1e3).astype(npt)
        b = (rng.standard_normal(3000) * 10).astype(npt)
        f = oracle.binary("remf", dt, a.view(STORAGE_OF[dt]), b.view(STORAGE_OF[dt]))
        want = np.array([math.fmod(float(x), float(y)) for x, y in zip(a, b)], npt)
        assert f.folded and np.array_equal(f.out, want.view(STORAGE_OF[dt]))
    else:
        a = rng.integers(0, 0x7C00, 3000, dtype=np.uint16)
        b = rng.integers(0x0400, 0x7C00, 3000, dtype=np.uint16)
        f = oracle.binary("remf", dt, a, b)
        if dt == "f16":
            want = [math.fmod(float(x), float(y)) for x, y in zip(a.view(np.float16), b.view(np.float16))]
            assert np.array_equal(f.out, np.array(want, np.float16).view(np.uint16))
        else:
            wa = (a.astype(np.uint32) << 16).view(np.float32)
            wb = (b.astype(np.uint32) << 16).view(np.float32)
            want = np.array([math.fmod(float(x), float(y)) for x, y in zip(wa, wb)], np.float32)
            assert not np.any(want.view(np.uint32) & 0xFFFF)   # exact in bf16
            assert np.array_equal(f.out, (want.view(np.uint32) >> 16).astype(np.uint16))
    # invalid and special operands
    one, zero, inf = 0x3F800000, 0, 0x7F800000
    got = oracle.binary("remf", "f32", np.array([inf, one, one, 0x7FC00005], np.uint32),
                        np.array([one, zero, inf, one], np.uint32)).out
    assert list(got) == [0x7FC00000, 0x7FC00000, one, 0x7FC00005]


def test_select(oracle):
    c = np.array([1, 0, 1, 0, 2], np.uint8)
    t = np.arange(5, dtype=np.uint32)
    e = np.arange(10, 15, dtype=np.uint32)
    assert list(oracle.select(c, t, e).out) == [0, 11, 2, 13, 4]
    f = oracle.select(np.array([0], np.uint8), t, np.array([7], np.uint32), n=5, cond_splat=True, f_splat=True)
    assert list(f.out) == [7] * 5 and f.is_splat


def test_byte_hash_formula(oracle):
    # The documented dedup hash, restated in Python.
    M = (1 << 64) - 1

    def mix(z):
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)

    def py_hash(b):
        h = 0
        for i in range(0, (len(b) + 7) // 8):
            w = int.from_bytes(b[8 * i:8 * i + 8], "little")
            h = (h + mix(w ^ ((i * 0x9E3779B97F4A7C15) & M))) & M
        return (h + mix(len(b))) & M

    rng = np.random.default_rng(4)
    for n in (0, 1, 7, 8, 9, 64, 1000, 4097):
        b = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert oracle.hash_bytes(b) == py_hash(b), n


@pytest.mark.parametrize("dt,np_t,ut", [("f32", np.float32, np.uint32), ("f64", np.float64, np.uint64)])
def test_math_float_ops_match_numpy(dt, np_t, ut, oracle):
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(4000) * 10.0 ** rng.integers(-3, 8, 4000),
                        np.array([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 0.0, -0.0, np.inf, -np.inf, 4.0, 1e-300])
                        ]).astype(np_t)
    bits = x.view(ut)
    def fold(op, v):
        f = oracle.convert(op, dt, dt, v.view(ut))
        assert f.folded, op
        return f.out.view(np_t)
    with np.errstate(all="ignore"):
        for op, ref in [("absf", np.abs), ("ceil", np.ceil), ("floor", np.floor), ("roundeven", np.rint),
                        ("trunc", np.trunc)]:
            assert np.array_equal(fold(op, x).view(ut), ref(x).view(ut)), op
        # round: half away from zero
        r = np.where(x >= 0, np.floor(x + np_t(0.5)), -np.floor(-x + np_t(0.5)))
        exact = np.abs(x) < 2.0 ** (23 if dt == "f32" else 52)
        assert np.array_equal(fold("round", x)[exact], r[exact])
        assert np.array_equal(fold("round", x)[~exact].view(ut), x[~exact].view(ut))
        pos = np.abs(x)
        pos = pos[pos.view(ut) != 0]     # +0 folds; -0 refuses (sign bit set)
        assert np.array_equal(fold("sqrt", pos).view(ut), np.sqrt(pos).view(ut))
        assert np.array_equal(fold("rsqrt", pos).view(ut), (np_t(1) / np.sqrt(pos)).view(ut))
    # refusals: a set sign bit (-0 and -NaN too) for sqrt / rsqrt
    for op in ("sqrt", "rsqrt"):
        for v in (-0.0, -1.0, -np.nan):
            f = oracle.convert(op, dt, dt, np.array([4.0, v], dtype=np_t).view(ut))
            assert not f.folded and f.first_fail_index == 1
    # NaN comes back quieted
    snan = np.array([0x7F800001 if dt == "f32" else 0x7FF0000000000001], dtype=ut)
    for op in ("ceil", "floor", "roundeven", "round", "trunc", "sqrt", "rsqrt"):
        q = oracle.convert(op, dt, dt, snan).out
        assert int(q[0]) == int(snan[0]) | (1 << (22 if dt == "f32" else 51)), op
    # round / trunc / sqrt / rsqrt exist for f32 and f64 only
    for op in ("round", "trunc", "sqrt", "rsqrt"):
        assert not oracle.convert(op, "f16", "f16", np.array([0x3C00], np.uint16)).folded


def test_math_integral_ops_on_narrow_floats(oracle):
    # f16: every bit pattern against numpy's float16 rounding of the double
    a = np.arange(1 << 16, dtype=np.uint16)
    x = a.view(np.float16)
    ok = ~np.isnan(x)
    for op, ref in [("ceil", np.ceil), ("floor", np.floor), ("roundeven", np.rint)]:
        got = oracle.convert(op, "f16", "f16", a).out
        with np.errstate(invalid="ignore"):
            want = ref(x.astype(np.float64)).astype(np.float16).view(np.uint16)
        assert np.array_equal(got[ok], want[ok]), op
        assert np.array_equal(got[~ok], a[~ok] | np.uint16(0x200)), op


@pytest.mark.parametrize("w", [1, 8, 16, 32, 64])
def test_math_int_ops_match_python(w, oracle):
    dt = {1: "i1", 8: "i8", 16: "i16", 32: "i32", 64: "i64"}[w]
    st = {1: np.uint8, 8: np.uint8, 16: np.uint16, 32: np.uint32, 64: np.uint64}[w]
    rng = np.random.default_rng(w)
    m = (1 << w) - 1
    vals = [0, 1, m, m >> 1, (m >> 1) + 1] + [int(v) & m for v in rng.integers(0, 1 << 62, 200)]
    a = np.array(vals, dtype=st)
    def sx(v):
        return v - (1 << w) if v >> (w - 1) else v
    want = {
        "absi": [abs(sx(v)) & m for v in vals],
        "ctlz": [w - v.bit_length() for v in vals],
        "cttz": [w if v == 0 else (v & -v).bit_length() - 1 for v in vals],
        "ctpop": [bin(v).count("1") for v in vals],
    }
    for op, exp in want.items():
        assert [int(x) for x in oracle.convert(op, dt, dt, a).out] == exp, op
    b = np.array([int(v) % 9 for v in vals], dtype=st) if w > 1 else a
    f = oracle.binary("ipowi", dt, a, b)
    if w == 1:
        assert not f.folded
        return
    assert [int(x) for x in f.out] == [pow(x, int(y), 1 << w) for x, y in zip(vals, b)]
    # negative exponents: 1 for base 1, +-1 for base -1 by parity, else 0; base 0 refuses
    neg = np.array([m, m - 1], dtype=st)
    assert [int(x) for x in oracle.binary("ipowi", dt, np.array([1, m], st), neg).out] == [1, 1]
    assert [int(x) for x in oracle.binary("ipowi", dt, np.array([m, 5], st), neg).out] == [m, 0]
    assert not oracle.binary("ipowi", dt, np.array([0], st), np.array([m], st)).folded


def test_copysign_matches_numpy(oracle):
    rng = np.random.default_rng(5)
    a = rng.integers(0, 1 << 32, 1000, dtype=np.uint64).astype(np.uint32)
    b = rng.integers(0, 1 << 32, 1000, dtype=np.uint64).astype(np.uint32)
    got = oracle.binary("copysign", "f32", a, b).out
    assert np.array_equal(got, (a & np.uint32(0x7FFFFFFF)) | (b & np.uint32(0x80000000)))
