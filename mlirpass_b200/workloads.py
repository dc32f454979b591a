"""Synthetic dense-constant workloads (the five fold configurations).

No public dataset is involved: every tensor is generated from SplitMix64
(the generator of mlirpass's fuzzer, fuzz/src/rng.rs:1-38, restated here)
with the seed `config * 1000 + tensor index`.  The *_np functions are the
numpy definitions; libdcfgen.so (gen/dcf_gen.c) computes the same values
fast enough for the full-size configurations.  All arrays are raw element
storage (uint bit patterns or float32 views) as the fold library takes them.

  config 1  two 1024x1024 f32 uniform[-1,1), one addf
  config 2  four 4096x4096 f32 uniform[-4,4); the divisor has 0.5% exact
            zeros with a nonzero numerator; chain addf, mulf, subf, divf,
            maximumf, minimumf (no NaN arises anywhere in the chain)
  config 3  8192x2048 i8 / i32 / i64, uniform full range with 1% edge
            values (INT_MIN, INT_MAX, -1, 0); addi muli subi andi xori,
            shli by amounts in [0, w), divsi and remsi by nonzero divisors
            that include INT_MIN / -1 pairs
  config 4  16M f32 normal(0, 1e3) with 1% quiet NaN, +-inf and denormals;
            truncf to bf16 / f16, extf back, fptosi of an in-range tensor,
            sitofp of uniform i32, cmpf olt / une; variant 4b pre-rounds
            the inputs so the conversions fold
  config 5  4096 functions, each two 256x256 f32 uniform[-1,1) -> addf ->
            mulf -> tosa.reciprocal, plus one 16384x16384 bf16
            uniform[-0.1,0.1) tosa.transpose perms [1, 0]
"""
from __future__ import annotations

import os

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)


def splitmix64_np(seed: int, n: int, start: int = 0) -> np.ndarray:
    """Outputs start+1 .. start+n of SplitMix64 seeded with `seed` (numpy:
    the definition that libdcfgen.so restates)."""
    with np.errstate(over="ignore"):
        i = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        z = np.uint64(seed) + i * GOLDEN
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
        return z ^ (z >> np.uint64(31))


def uniform_f32_np(seed: int, n: int, lo: float, hi: float) -> np.ndarray:
    u = (splitmix64_np(seed, n) >> np.uint64(40)).astype(np.float64) / float(1 << 24)
    return (lo + (hi - lo) * u).astype(np.float32)


def uniform_bf16_bits_np(seed: int, n: int, lo: float, hi: float) -> np.ndarray:
    """bf16 bit patterns of uniform[lo, hi) values (round to nearest even)."""
    x = uniform_f32_np(seed, n, lo, hi).view(np.uint32)
    rounded = x + np.uint32(0x7FFF) + ((x >> np.uint32(16)) & np.uint32(1))
    return (rounded >> np.uint32(16)).astype(np.uint16)


_gen = None


def gen_lib():
    """libdcfgen.so: the same generators in C (built on first use)."""
    global _gen
    if _gen is None:
        import ctypes
        from .build import GEN_LIB, build_gen
        if not os.path.exists(GEN_LIB):
            build_gen()
        L = ctypes.CDLL(GEN_LIB)
        u64, vp, dbl = ctypes.c_uint64, ctypes.c_void_p, ctypes.c_double
        L.dcg_splitmix64.argtypes = [u64, u64, u64, vp]
        L.dcg_uniform_f32.argtypes = [u64, u64, dbl, dbl, vp]
        L.dcg_uniform_bf16.argtypes = [u64, u64, dbl, dbl, vp]
        L.dcg_hex_upper.argtypes = [vp, u64, vp]
        for f in (L.dcg_splitmix64, L.dcg_uniform_f32, L.dcg_uniform_bf16, L.dcg_hex_upper):
            f.restype = None
        _gen = L
    return _gen


def splitmix64(seed: int, n: int, start: int = 0) -> np.ndarray:
    """Outputs start+1 .. start+n of SplitMix64 seeded with `seed`."""
    out = np.empty(n, dtype=np.uint64)
    gen_lib().dcg_splitmix64(seed & 0xFFFFFFFFFFFFFFFF, start, n, out.ctypes.data)
    return out


def uniform_f32(seed: int, n: int, lo: float, hi: float) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    gen_lib().dcg_uniform_f32(seed, n, lo, hi, out.ctypes.data)
    return out


def uniform_bf16_bits(seed: int, n: int, lo: float, hi: float) -> np.ndarray:
    """bf16 bit patterns of uniform[lo, hi) values (round to nearest even)."""
    out = np.empty(n, dtype=np.uint16)
    gen_lib().dcg_uniform_bf16(seed, n, lo, hi, out.ctypes.data)
    return out


def hex_upper(a: np.ndarray) -> str:
    """Uppercase hex of an array's raw bytes (a dense<"0x…"> body)."""
    b = np.ascontiguousarray(a).reshape(-1).view(np.uint8)
    out = bytearray(2 * b.size)
    if b.size:
        import ctypes
        buf = (ctypes.c_char * len(out)).from_buffer(out)
        gen_lib().dcg_hex_upper(b.ctypes.data, b.size, ctypes.addressof(buf))
        del buf
    return out.decode("ascii")


def normal_f32(seed: int, n: int, sigma: float) -> np.ndarray:
    r = splitmix64(seed, 2 * n)
    u1 = (r[0::2] >> np.uint64(11)).astype(np.float64) / float(1 << 53)
    u2 = (r[1::2] >> np.uint64(11)).astype(np.float64) / float(1 << 53)
    z = np.sqrt(-2.0 * np.log1p(-u1)) * np.cos(2.0 * np.pi * u2)
    return (sigma * z).astype(np.float32)


def positions(seed: int, n: int, count: int) -> np.ndarray:
    """`count` distinct seeded positions in [0, n)."""
    r = splitmix64(seed, count * 2)
    pos = np.unique((r % np.uint64(n)).astype(np.int64))
    return pos[:count]


def seed(config: int, index: int) -> int:
    return config * 1000 + index


# ----------------------------------------------------------------- config 1

def config1():
    n = 1024 * 1024
    return {"A": uniform_f32(seed(1, 0), n, -1.0, 1.0), "B": uniform_f32(seed(1, 1), n, -1.0, 1.0),
            "shape": (1024, 1024)}


# ----------------------------------------------------------------- config 2

CHAIN2 = [("addf", "A", "B", "t1"), ("mulf", "t1", "C", "t2"), ("subf", "t2", "D", "t3"),
          ("divf", "t3", "D", "t4"), ("maximumf", "t4", "A", "t5"), ("minimumf", "t5", "B", "t6")]


def config2(side: int = 4096):
    n = side * side
    A = uniform_f32(seed(2, 0), n, -4.0, 4.0)
    B = uniform_f32(seed(2, 1), n, -4.0, 4.0)
    C = uniform_f32(seed(2, 2), n, -4.0, 4.0)
    D = uniform_f32(seed(2, 3), n, -4.0, 4.0)
    zeros = positions(seed(2, 4), n, max(1, n // 200))
    # At the divisor's zeros the numerator (A+B)*C must be nonzero, so the
    # quotient is +-inf and never NaN.
    s = A[zeros] + B[zeros]
    A[zeros] = np.where(s == 0, np.float32(1.0), A[zeros])
    B[zeros] = np.where(s == 0, np.float32(0.5), B[zeros])
    C[zeros] = np.where(C[zeros] == 0, np.float32(1.0), C[zeros])
    D[zeros] = np.float32(0.0)
    # Elsewhere keep the divisor away from zero (a uniform draw of exactly 0
    # is possible but must not add zeros beyond the planted ones).
    D[(D == 0)] = np.float32(0.25)
    D[zeros] = np.float32(0.0)
    return {"A": A, "B": B, "C": C, "D": D, "shape": (side, side), "zeros": zeros}


# ----------------------------------------------------------------- config 3

INT_OPS3 = ["addi", "muli", "subi", "andi", "xori", "shli", "divsi", "remsi"]
INT_NP = {"i8": np.int8, "i32": np.int32, "i64": np.int64}
INT_W = {"i8": 8, "i32": 32, "i64": 64}


def config3(dtype: str, rows: int = 8192, cols: int = 2048):
    n = rows * cols
    w = INT_W[dtype]
    st = {8: np.uint8, 32: np.uint32, 64: np.uint64}[w]
    k = {"i8": 0, "i32": 10, "i64": 20}[dtype]
    mask = np.uint64((1 << w) - 1)
    X = (splitmix64(seed(3, k + 0), n) & mask).astype(st)
    Y = (splitmix64(seed(3, k + 1), n) & mask).astype(st)
    imin, imax = st(1 << (w - 1)), st((1 << (w - 1)) - 1)
    neg1, zero = st((1 << w) - 1), st(0)
    edges = np.array([imin, imax, neg1, zero], dtype=st)
    for arr, sd in ((X, k + 2), (Y, k + 3)):
        pos = positions(seed(3, sd), n, n // 100)
        pick = (splitmix64(seed(3, sd + 100), len(pos)) % np.uint64(4)).astype(np.int64)
        arr[pos] = edges[pick]
    S = (splitmix64(seed(3, k + 4), n) % np.uint64(w)).astype(st)
    # Nonzero divisor with INT_MIN / -1 pairs planted.
    Yd = Y.copy()
    Yd[Yd == 0] = st(1)
    pairs = positions(seed(3, k + 5), n, max(1, n // 1000))
    Xd = X.copy()
    Xd[pairs] = imin
    Yd[pairs] = neg1
    return {"X": X, "Y": Y, "S": S, "Xd": Xd, "Yd": Yd, "shape": (rows, cols), "pairs": pairs}


# ----------------------------------------------------------------- config 4

def config4(n: int = 16 * 1024 * 1024, prerounded: bool = False):
    x = normal_f32(seed(4, 0), n, 1000.0).view(np.uint32).copy()
    special = positions(seed(4, 1), n, n // 100)
    kinds = (splitmix64(seed(4, 2), len(special)) % np.uint64(4)).astype(np.int64)
    den = (splitmix64(seed(4, 3), len(special)) & np.uint64(0x7FFFFF)).astype(np.uint32) | np.uint32(1)
    vals = np.where(kinds == 0, np.uint32(0x7FC00000),
                    np.where(kinds == 1, np.uint32(0x7F800000),
                             np.where(kinds == 2, np.uint32(0xFF800000), den)))
    x[special] = vals.astype(np.uint32)
    ints = (splitmix64(seed(4, 4), n) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    # fptosi input: finite and |x| < 2^31.
    inrange = normal_f32(seed(4, 5), n, 1.0e6).view(np.uint32).copy()
    if prerounded:
        # bf16-representable: clear the low 16 bits (NaN stays quiet 0x7FC0.., inf stays inf;
        # denormals keep their top bits).  f16-representable inputs are made separately.
        x = x & np.uint32(0xFFFF0000)
        xf = x.view(np.float32)
        finite = np.isfinite(xf)
        # f16 range and precision: round to f16 and back through numpy.
        h = np.where(finite, np.clip(xf, -60000.0, 60000.0), xf).astype(np.float16)
        x16 = h.astype(np.float32).view(np.uint32)
        return {"x": x, "x_f16": x16, "ints": ints, "inrange": inrange, "n": n}
    return {"x": x, "ints": ints, "inrange": inrange, "n": n}


# ----------------------------------------------------------------- config 5

def config5_func(i: int, side: int = 256):
    n = side * side
    return (uniform_f32(seed(5, 10 + 2 * i), n, -1.0, 1.0), uniform_f32(seed(5, 11 + 2 * i), n, -1.0, 1.0))


def config5_weight(side: int = 16384):
    return uniform_bf16_bits(seed(5, 0), side * side, -0.1, 0.1)
