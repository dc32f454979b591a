"""A bit-level model, on the CPU, of the float-domain lane division of
8- and 16-bit words (`div_lanes` and `lane_recip` in
mlirpass_b200/csrc/dcf_ew_int.cu), checked against integer division.

The kernel's arithmetic is restated step by step with numpy: byte
permutations, the magic-number unpacking, the reciprocal seed and its
refinement steps (each fma rounded once to f32), the floor taken by an fma
rounded toward zero onto the 2^23 grid, the sign rules and the packing.
The reciprocal's accuracy is checked over every divisor below 2^16 (the
bound the floor argument needs), and the whole division over every 8-bit
pair in every lane position and over 16-bit pairs next to the multiples of
their divisors.  The GPU tests check the kernel itself against the oracle.
"""
import numpy as np
import pytest

M = np.float32(8388608.0)  # 2^23


def flt(u):
    return np.asarray(u, dtype=np.uint32).view(np.float32)


def bits(f):
    return np.asarray(f, dtype=np.float32).view(np.uint32)


def fma_rn(a, b, c):
    # Exact in f64 for the operands that occur here (products of at most
    # 24 + 17 significant bits near the addend's scale), then one rounding.
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def fma_rz_magic(a, b):
    # fma(a, b, 2^23) rounded toward zero, for 0 <= a b < 2^23: the integer
    # part of 2^23 + a b (every value stays far from an integer, so the
    # f64 sum's rounding cannot cross one).
    return np.floor(a.astype(np.float64) * b.astype(np.float64) + 8388608.0).astype(np.float32)


def byte_perm(x, y, s):
    out = np.zeros_like(x)
    for n in range(4):
        idx = (s >> (4 * n)) & 7
        src = x if idx < 4 else y
        out |= ((src >> np.uint32(8 * (idx & 3))) & np.uint32(0xFF)) << np.uint32(8 * n)
    return out


def lane_recip(W, signed, d):
    one = np.ones_like(d)
    r = flt((np.int64(0x7EF311C3) - bits(d).astype(np.int64)).astype(np.uint32))
    e = fma_rn(-d, r, one)
    if signed:
        r = fma_rn(r, e, r)
        if W == 16:
            r = fma_rn(r, fma_rn(-d, r, one), r)
    else:
        r = fma_rn(r, fma_rn(e, e, e), r)
        if W == 16:
            r = fma_rn(r, fma_rn(-d, r, one), r)
    return r


def div_lanes(op, W, a, b):
    signed, rem = op in ("divsi", "remsi"), op in ("remsi", "remui")
    bias = (0x80808080 if W == 8 else 0x80008000) if signed else 0
    doff = np.float32(8388608.0 + (1 << (W - 1))) if signed else M
    xoff = doff if signed else np.float32(8388608.0 - 0.5)
    wrap = np.float32(8388608.0 + (1 << W)) if signed else np.float32(8388608.0 - 0.5)
    a, b = a ^ np.uint32(bias), b ^ np.uint32(bias)
    f = []
    for k in range(32 // W):
        sel = (0x7440 | k) if W == 8 else (0x7400 | ((2 * k + 1) << 4) | (2 * k))
        x = flt(byte_perm(a, np.uint32(0x4B000000), sel)) - xoff
        d = flt(byte_perm(b, np.uint32(0x4B000000), sel)) - doff
        ad = np.abs(d) if signed else d
        xh = (np.abs(x) + np.float32(0.5)).astype(np.float32) if signed else x
        qm = fma_rz_magic(xh, lane_recip(W, signed, ad))
        if op == "divui":
            v = qm
        elif op == "remui":
            v = (fma_rn(-(qm - M).astype(np.float32), ad, xh) + wrap).astype(np.float32)
        else:
            q = (qm - M).astype(np.float32)
            v = fma_rn(-q, ad, np.abs(x)) if rem else q
            v = (np.copysign(v, x if rem else (x * d).astype(np.float32)) + wrap).astype(np.float32)
        f.append(bits(v))
    if W == 8:
        return byte_perm(byte_perm(f[0], f[1], 0x0040), byte_perm(f[2], f[3], 0x0040), 0x5410)
    return byte_perm(f[0], f[1], 0x5410)


def expected(op, W, x, y):
    m = (1 << W) - 1
    if op in ("divui", "remui"):
        return (x // y if op == "divui" else x % y) & m
    sx = np.where(x >= 1 << (W - 1), x - (1 << W), x)
    sy = np.where(y >= 1 << (W - 1), y - (1 << W), y)
    q = np.abs(sx) // np.abs(sy) * np.sign(sx) * np.sign(sy)
    return (q if op == "divsi" else sx - q * sy) & m


def check(op, W, xs, ys):
    n = 32 // W
    L = len(xs) // n * n
    X = xs[:L].reshape(-1, n).astype(np.uint32)
    Y = ys[:L].reshape(-1, n).astype(np.uint32)
    a = np.zeros(len(X), np.uint32)
    b = np.zeros(len(X), np.uint32)
    for k in range(n):
        a |= X[:, k] << np.uint32(W * k)
        b |= Y[:, k] << np.uint32(W * k)
    got = div_lanes(op, W, a, b)
    for k in range(n):
        g = ((got >> np.uint32(W * k)) & np.uint32((1 << W) - 1)).astype(np.int64)
        w = expected(op, W, X[:, k].astype(np.int64), Y[:, k].astype(np.int64))
        keep = np.ones(len(g), bool)
        if op == "divsi":  # the signed minimum / -1 refuses; its lane value is unused
            keep = ~((X[:, k] == 1 << (W - 1)) & (Y[:, k] == (1 << W) - 1))
        bad = np.nonzero((g != w) & keep)[0]
        assert bad.size == 0, (op, W, k, int(X[bad[0], k]), int(Y[bad[0], k]), int(g[bad[0]]), int(w[bad[0]]))


@pytest.mark.parametrize("W,signed", [(8, True), (8, False), (16, True), (16, False)])
def test_reciprocal_accuracy_covers_the_floor(W, signed):
    # (|x| + 1/2) |e| < 1/2 for the largest magnitude of the width is what
    # makes floor((|x| + 1/2) r) exact; checked over every divisor (the
    # tightest width, 8-bit signed with one Newton step, reaches 0.33).
    top = (1 << (W - 1)) if signed else (1 << W) - 1
    d = np.arange(1, top + 1, dtype=np.float32)
    e = np.abs(1.0 - d.astype(np.float64) * lane_recip(W, signed, d).astype(np.float64)).max()
    assert (top + 0.5) * e < 0.4, (W, signed, e)


def test_seed_error_over_integer_divisors():
    d = np.arange(1, 65536, dtype=np.float32)
    r0 = flt((np.int64(0x7EF311C3) - bits(d).astype(np.int64)).astype(np.uint32))
    assert np.abs(1.0 - d.astype(np.float64) * r0).max() < 0.0506


@pytest.mark.parametrize("op", ["divsi", "divui", "remsi", "remui"])
def test_every_8bit_pair_in_every_lane(op):
    x, y = np.meshgrid(np.arange(256), np.arange(1, 256))
    x, y = x.ravel(), y.ravel()
    for rot in range(4):
        check(op, 8, np.roll(x, rot), np.roll(y, rot))


@pytest.mark.parametrize("op", ["divsi", "divui", "remsi", "remui"])
def test_16bit_pairs_next_to_multiples(op):
    rng = np.random.default_rng(5)
    xs, ys = [], []
    for d in np.concatenate([np.arange(1, 600), rng.integers(600, 65536, 1500), [32767, 32768, 65535]]):
        d = int(d)
        m = np.arange(0, 65536 // d + 2, dtype=np.int64) * d
        m = np.concatenate([m - 1, m, [0, 32767, 32768, 65535]])
        m = m[(m >= 0) & (m < 65536)]
        xs.append(m)
        ys.append(np.full(m.size, d))
        if d <= 32768:  # the same magnitudes with every sign combination
            for sx in (1, -1):
                for sd in (1, -1):
                    v = sx * m[m <= 32768]
                    v = v[(v >= -32768) & (v <= 32767)]
                    if -32768 <= sd * d <= 32767:
                        xs.append(v & 0xFFFF)
                        ys.append(np.full(v.size, (sd * d) & 0xFFFF))
    xs, ys = np.concatenate(xs), np.concatenate(ys)
    for rot in range(2):
        check(op, 16, np.roll(xs, rot), np.roll(ys, rot))
