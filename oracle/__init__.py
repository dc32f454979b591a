"""CPU oracle for the dense-constant folds — TEST INFRASTRUCTURE ONLY.

Binding of oracle/_build/libdcforacle.so, the plain-C restatement of the
reference's fold closures (dcf_oracle.c).  Only tests/, the smoke check of
__graft_entry__ and bench.py's CPU-baseline leg may use it, and only as the
checker or as the timed CPU baseline — never as the product path.

The functions mirror mlirpass_b200's host API so a test drives both the same
way.  Parity is pinned against the reference's fixture golden vectors in
tests/golden/fold_vectors.json; the NaN payload of invalid float
arithmetic (inf-inf, 0*inf, 0/0) is the one unpinned choice (LLVM APFloat's
positive quiet NaN, switchable by flag).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libdcforacle.so")

from mlirpass_b200 import BOOL_RESULT_OPS, DTYPES, OPS, Fold, Result, as_storage, storage  # noqa: E402

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            from mlirpass_b200.build import build_oracle
            build_oracle()
        L = ctypes.CDLL(LIB_PATH)
        vp, u64, i, u32, sz = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_uint32, ctypes.c_size_t
        rp = ctypes.POINTER(Result)
        L.dco_binary.argtypes = [i, i, vp, i, vp, i, u64, u32, vp, rp]
        L.dco_convert.argtypes = [i, i, i, vp, i, u64, u32, vp, rp]
        L.dco_reciprocal.argtypes = [i, vp, i, u64, u32, vp, rp]
        L.dco_select.argtypes = [sz, vp, i, vp, i, vp, i, u64, vp, rp]
        L.dco_transpose.argtypes = [sz, i, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), vp, vp]
        L.dco_hex_encode.argtypes = [vp, u64, vp]
        L.dco_hex_decode.argtypes = [vp, u64, vp]
        L.dco_splat_check.argtypes = [vp, sz, u64]
        L.dco_float_convert_bits.argtypes = [i, i, u64, ctypes.POINTER(ctypes.c_int)]
        L.dco_float_convert_bits.restype = u64
        L.dco_round_from_double.argtypes = [i, ctypes.c_double]
        L.dco_round_from_double.restype = u64
        L.dco_hash.argtypes = [vp, u64]
        L.dco_hash.restype = u64
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _rc(rc):
    if rc < 0:
        raise RuntimeError(f"oracle error {rc}")


def binary(op, dtype, lhs, rhs, *, n=None, lhs_splat=False, rhs_splat=False, flags=0, out=None) -> Fold:
    l, r = as_storage(lhs, dtype), as_storage(rhs, dtype)
    if n is None:
        n = 1 if (lhs_splat and rhs_splat) else max(len(l), len(r))
    odt = "i1" if op in BOOL_RESULT_OPS else dtype
    if out is None:
        out = np.zeros(n, dtype=storage(odt))
    res = Result()
    _rc(lib().dco_binary(OPS[op], DTYPES[dtype], _p(l), int(lhs_splat), _p(r), int(rhs_splat), n, flags, _p(out),
                         ctypes.byref(res)))
    return Fold(bool(res.folded), bool(res.is_splat), int(res.first_fail_index), out)


def convert(op, from_dtype, to_dtype, x, *, n=None, splat=False, flags=0, out=None) -> Fold:
    a = as_storage(x, from_dtype)
    if n is None:
        n = len(a)
    if out is None:
        out = np.zeros(n, dtype=storage(to_dtype))
    res = Result()
    _rc(lib().dco_convert(OPS[op], DTYPES[from_dtype], DTYPES[to_dtype], _p(a), int(splat), n, flags, _p(out),
                          ctypes.byref(res)))
    return Fold(bool(res.folded), bool(res.is_splat), int(res.first_fail_index), out)


def reciprocal(dtype, x, *, n=None, splat=False, flags=0, out=None) -> Fold:
    a = as_storage(x, dtype)
    if n is None:
        n = len(a)
    if out is None:
        out = np.zeros(n, dtype=storage(dtype))
    res = Result()
    _rc(lib().dco_reciprocal(DTYPES[dtype], _p(a), int(splat), n, flags, _p(out), ctypes.byref(res)))
    return Fold(bool(res.folded), bool(res.is_splat), int(res.first_fail_index), out)


def select(cond, t, f, *, n=None, cond_splat=False, t_splat=False, f_splat=False) -> Fold:
    c = np.ascontiguousarray(cond, dtype=np.uint8).reshape(-1)
    a = np.ascontiguousarray(t).reshape(-1)
    b = np.ascontiguousarray(f).reshape(-1)
    if n is None:
        n = max(len(c), len(a), len(b))
    out = np.zeros(n, dtype=a.dtype)
    res = Result()
    _rc(lib().dco_select(a.dtype.itemsize, _p(c), int(cond_splat), _p(a), int(t_splat), _p(b), int(f_splat), n,
                         _p(out), ctypes.byref(res)))
    return Fold(bool(res.folded), bool(res.is_splat), int(res.first_fail_index), out)


def transpose(x, shape, perms):
    a = np.ascontiguousarray(x).reshape(-1)
    out = np.empty_like(a)
    rank = len(shape)
    _rc(lib().dco_transpose(a.dtype.itemsize, rank, (ctypes.c_int64 * rank)(*shape),
                            (ctypes.c_int64 * rank)(*perms), _p(a), _p(out)))
    return out.reshape([shape[p] for p in perms])


def hex_encode(data) -> bytes:
    a = np.frombuffer(bytes(data), dtype=np.uint8)
    out = np.empty(2 * len(a), dtype=np.uint8)
    _rc(lib().dco_hex_encode(_p(a), len(a), _p(out)))
    return out.tobytes()


def hex_decode(text) -> bytes:
    t = text.encode() if isinstance(text, str) else bytes(text)
    a = np.frombuffer(t, dtype=np.uint8)
    out = np.empty(len(a) // 2, dtype=np.uint8)
    _rc(lib().dco_hex_decode(_p(a), len(a), _p(out)))
    return out.tobytes()


def splat_check(x) -> bool:
    a = np.ascontiguousarray(x).reshape(-1)
    return bool(lib().dco_splat_check(_p(a), a.dtype.itemsize, len(a)))


def float_convert_bits(from_dtype, to_dtype, bits):
    ok = ctypes.c_int(0)
    r = lib().dco_float_convert_bits(DTYPES[from_dtype], DTYPES[to_dtype], bits, ctypes.byref(ok))
    return bool(ok.value), int(r)


def hash_bytes(data) -> int:
    a = np.frombuffer(bytes(data), dtype=np.uint8)
    return int(lib().dco_hash(_p(a) if len(a) else None, len(a)))
