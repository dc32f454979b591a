"""mlirpass_b200 — B200-native dense-constant folding for mlirpass.

Python binding of libdcfold.so (include/dcfold.h).  The library replaces the
per-element loops of mlirpass's fold hooks (Folder::binary / Folder::unary in
src/patterns/arith/canonicalize.rs, Tf::transpose / Tf::reciprocal in
src/patterns/tosa/canonicalize.rs) with sm_100a kernels.

Values cross the boundary as raw little-endian element storage: numpy arrays
whose itemsize equals the element size (bit patterns; a float32 array is fine
for f32).  Importing this package does not need a GPU; every compute call
does, and raises DcfError when the library reports no device — there is no
CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdcfold.so")

DTYPES = {
    "i1": 1, "i8": 2, "i16": 3, "i32": 4, "i64": 5,
    "f16": 16, "bf16": 17, "f32": 18, "f64": 19,
    "f8E5M2": 20, "f8E4M3": 21, "f8E3M4": 22,
}
DTYPE_SIZE = {"i1": 1, "i8": 1, "i16": 2, "i32": 4, "i64": 8, "f16": 2, "bf16": 2, "f32": 4, "f64": 8,
              "f8E5M2": 1, "f8E4M3": 1, "f8E3M4": 1}
FLOAT_DTYPES = ("f16", "bf16", "f32", "f64", "f8E5M2", "f8E4M3", "f8E3M4")
INT_DTYPES = ("i1", "i8", "i16", "i32", "i64")
STORAGE = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}

OPS = {
    "addf": 1, "subf": 2, "mulf": 3, "divf": 4, "maximumf": 5, "minimumf": 6, "maxnumf": 7, "minnumf": 8,
    "remf": 9,
    "addi": 16, "subi": 17, "muli": 18, "andi": 19, "ori": 20, "xori": 21, "shli": 22, "shrui": 23,
    "shrsi": 24, "divsi": 25, "divui": 26, "remsi": 27, "remui": 28, "maxsi": 29, "maxui": 30,
    "minsi": 31, "minui": 32, "ceildivui": 33, "ceildivsi": 34, "floordivsi": 35, "mulsi_hi": 36,
    "mului_hi": 37, "cmpi": 48, "cmpf": 49, "addui_carry": 50,
    "extf": 64, "truncf": 65, "sitofp": 66, "uitofp": 67, "fptosi": 68, "fptoui": 69,
    "negf": 70, "flush_denormals": 71, "extsi": 72, "extui": 73, "trunci": 74,
    "reciprocal": 80,
    # math dialect (exact folds only)
    "absf": 96, "ceil": 97, "floor": 98, "roundeven": 99, "round": 100, "trunc": 101, "sqrt": 102,
    "rsqrt": 103, "absi": 104, "ctlz": 105, "cttz": 106, "ctpop": 107, "copysign": 112, "ipowi": 113,
}
BINARY_OPS = tuple(k for k, v in OPS.items() if v < 64 or k in ("copysign", "ipowi"))
FLOAT_BINARY_OPS = tuple(k for k, v in OPS.items() if v < 16 or k in ("cmpf", "copysign"))
MATH_FLOAT_UNARY_OPS = ("absf", "ceil", "floor", "roundeven", "round", "trunc", "sqrt", "rsqrt")
MATH_INT_UNARY_OPS = ("absi", "ctlz", "cttz", "ctpop")
INT_BINARY_OPS = tuple(k for k in BINARY_OPS if k not in FLOAT_BINARY_OPS)
BOOL_RESULT_OPS = ("cmpi", "cmpf", "addui_carry")
CONVERT_OPS = ("extf", "truncf", "sitofp", "uitofp", "fptosi", "fptoui", "negf", "flush_denormals", "extsi",
               "extui", "trunci") + MATH_FLOAT_UNARY_OPS + MATH_INT_UNARY_OPS

FLAG_PRED_SHIFT = 8
FLAG_NEG_DEFAULT_NAN = 1 << 16

ERRORS = {-1: "EINVAL", -2: "ENODEV", -3: "ENOMEM", -4: "ECUDA", -5: "EUNSUPPORTED", -6: "ETIMEOUT",
          -7: "EPARSE"}


def flags(roundingmode: int = 0, predicate: int = 0, neg_default_nan: bool = False) -> int:
    """Pack the flags word (DCF_FLAG_* in include/dcfold.h)."""
    return (roundingmode & 7) | ((predicate & 15) << FLAG_PRED_SHIFT) | (FLAG_NEG_DEFAULT_NAN if neg_default_nan else 0)


class DcfError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"dcfold {ERRORS.get(code, code)}: {msg}")
        self.code = code


class Result(ctypes.Structure):
    _fields_ = [("folded", ctypes.c_uint8), ("is_splat", ctypes.c_uint8), ("reserved", ctypes.c_uint8 * 6),
                ("first_fail_index", ctypes.c_uint64)]


class Status(ctypes.Structure):
    _fields_ = [("first_fail", ctypes.c_uint64), ("splat_word", ctypes.c_uint32), ("error", ctypes.c_uint32)]


class Job(ctypes.Structure):
    _fields_ = [("op", ctypes.c_uint32), ("dtype", ctypes.c_uint32), ("out_dtype", ctypes.c_uint32),
                ("flags", ctypes.c_uint32), ("lhs", ctypes.c_void_p), ("rhs", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("n", ctypes.c_uint64), ("lhs_splat", ctypes.c_uint8),
                ("rhs_splat", ctypes.c_uint8), ("reserved", ctypes.c_uint8 * 6), ("result", Result)]


# Every symbol include/dcfold.h declares, with its ctypes signature.
_VP, _U64, _I, _U32, _SZ = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_uint32, ctypes.c_size_t
_RP, _SP = ctypes.POINTER(Result), ctypes.POINTER(Status)
SIGNATURES = {
    "dcf_init": (_I, [_I]),
    "dcf_shutdown": (_I, []),
    "dcf_device_count": (_I, []),
    "dcf_last_error": (ctypes.c_char_p, []),
    "dcf_version": (ctypes.c_char_p, []),
    "dcf_dtype_size": (_SZ, [_I]),
    "dcf_kernel_launches": (_U64, []),
    "dcf_binary": (_I, [_I, _I, _VP, _I, _VP, _I, _U64, _U32, _VP, _RP]),
    "dcf_convert": (_I, [_I, _I, _I, _VP, _I, _U64, _U32, _VP, _RP]),
    "dcf_reciprocal": (_I, [_I, _VP, _I, _U64, _U32, _VP, _RP]),
    "dcf_select": (_I, [_SZ, _VP, _I, _VP, _I, _VP, _I, _U64, _VP, _RP]),
    "dcf_transpose": (_I, [_SZ, _I, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), _VP, _VP, _RP]),
    "dcf_hex_encode": (_I, [_VP, _U64, _VP]),
    "dcf_hex_decode": (_I, [_VP, _U64, _VP]),
    "dcf_splat_check": (_I, [_VP, _SZ, _U64, ctypes.POINTER(ctypes.c_int)]),
    "dcf_batch": (_I, [ctypes.POINTER(Job), _SZ]),
    "dcf_batch_noalloc": (_I, [ctypes.POINTER(Job), _SZ, _VP]),
    "dcf_status_reset_async": (_I, [_VP, _VP]),
    "dcf_binary_async": (_I, [_I, _I, _VP, _I, _VP, _I, _U64, _U32, _VP, _VP, _VP]),
    "dcf_convert_async": (_I, [_I, _I, _I, _VP, _I, _U64, _U32, _VP, _VP, _VP]),
    "dcf_reciprocal_async": (_I, [_I, _VP, _I, _U64, _U32, _VP, _VP, _VP]),
    "dcf_select_async": (_I, [_SZ, _VP, _I, _VP, _I, _VP, _I, _U64, _VP, _VP, _VP]),
    "dcf_transpose2d_async": (_I, [_SZ, _U64, _U64, _VP, _VP, _VP]),
    "dcf_permute_async": (_I, [_SZ, _I, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), _VP, _VP,
                               _VP]),
    "dcf_permute_status_async": (_I, [_SZ, _I, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), _VP,
                                      _VP, _VP, _VP]),
    "dcf_splat_check_async": (_I, [_VP, _SZ, _U64, _VP, _VP]),
    "dcf_hex_encode_async": (_I, [_VP, _U64, _VP, _VP]),
    "dcf_hex_decode_async": (_I, [_VP, _U64, _VP, _VP, _VP]),
    "dcf_hex_decode_many_async": (_I, [_VP, _SZ, _U64, _VP, _VP]),
    "dcf_hash_many_async": (_I, [_VP, _SZ, _U64, _VP, _VP]),
    "dcf_status_read": (_I, [_VP, _VP, _RP]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libdcfold.so (built by `python -m mlirpass_b200.build`)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m mlirpass_b200.build` first")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(rc: int) -> int:
    if rc < 0:
        raise DcfError(rc, lib().dcf_last_error().decode())
    return rc


def init(n_gpus: int = 1) -> int:
    """Choose the GPUs host calls shard over (devices 0..n-1)."""
    return _check(lib().dcf_init(n_gpus))


def shutdown() -> None:
    _check(lib().dcf_shutdown())


def device_count() -> int:
    return lib().dcf_device_count()


def kernel_launches() -> int:
    """Kernels launched by libdcfold.so in this process so far."""
    return int(lib().dcf_kernel_launches())


def storage(dtype: str):
    return STORAGE[DTYPE_SIZE[dtype]]


def as_storage(x, dtype: str) -> np.ndarray:
    """A C-contiguous numpy view of x with the element storage of dtype."""
    a = np.ascontiguousarray(x)
    st = storage(dtype)
    if a.dtype.itemsize != np.dtype(st).itemsize:
        raise ValueError(f"array itemsize {a.dtype.itemsize} does not match {dtype}")
    return a.view(st).reshape(-1)


@dataclass
class Fold:
    """Outcome of one fold: `out` is meaningful only when `folded`."""
    folded: bool
    is_splat: bool
    first_fail_index: int
    out: np.ndarray | None


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def binary(op: str, dtype: str, lhs, rhs, *, n: int | None = None, lhs_splat: bool = False,
           rhs_splat: bool = False, flags: int = 0, out: np.ndarray | None = None) -> Fold:
    """Elementwise binary fold (Folder::binary's loop) on host buffers."""
    l, r = as_storage(lhs, dtype), as_storage(rhs, dtype)
    if n is None:
        n = 1 if (lhs_splat and rhs_splat) else max(len(l), len(r))
    odt = "i1" if op in BOOL_RESULT_OPS else dtype
    if out is None:
        out = np.empty(n, dtype=storage(odt))
    res = Result()
    _check(lib().dcf_binary(OPS[op], DTYPES[dtype], _ptr(l), int(lhs_splat), _ptr(r), int(rhs_splat), n, flags,
                            _ptr(out), ctypes.byref(res)))
    return Fold(bool(res.folded), bool(res.is_splat), int(res.first_fail_index), out)


def convert(op: str, from_dtype: str, to_dtype: str, x, *, n: int | None = None, splat: bool = False,
            flags: int = 0, out: np.ndarray | None = None) -> Fold:
    """Elementwise conversion fold (the Const::map closures of Folder::unary)."""
    a = as_storage(x, from_dtype)
    if n is None:
        n = len(a)
    if out is None:
        out = np.empty(n, dtype=storage(to_dtype))
    res = Result()
    _check(lib().dcf_convert(OPS[op], DTYPES[from_dtype], DTYPES[to_dtype], _ptr(a), int(splat), n, flags,
                             _ptr(out), ctypes.byref(res)))
    return Fold(bool(res.folded), bool(res.is_splat), int(res.first_fail_index), out)


def reciprocal(dtype: str, x, *, n: int | None = None, splat: bool = False, flags: int = 0,
               out: np.ndarray | None = None) -> Fold:
    a = as_storage(x, dtype)
    if n is None:
        n = len(a)
    if out is None:
        out = np.empty(n, dtype=storage(dtype))
    res = Result()
    _check(lib().dcf_reciprocal(DTYPES[dtype], _ptr(a), int(splat), n, flags, _ptr(out), ctypes.byref(res)))
    return Fold(bool(res.folded), bool(res.is_splat), int(res.first_fail_index), out)


def select(cond, t, f, *, n: int | None = None, cond_splat: bool = False, t_splat: bool = False,
           f_splat: bool = False, out: np.ndarray | None = None) -> Fold:
    """Elementwise select over dense constants (Folder::select's value loop):
    out[i] = t[i] if cond[i] else f[i].  t and f share one storage dtype."""
    c = np.ascontiguousarray(cond, dtype=np.uint8).reshape(-1)
    a = np.ascontiguousarray(t).reshape(-1)
    b = np.ascontiguousarray(f).reshape(-1)
    if a.dtype.itemsize != b.dtype.itemsize:
        raise ValueError("t and f must have the same element size")
    if n is None:
        n = max(len(c), len(a), len(b))
    if out is None:
        out = np.empty(n, dtype=a.dtype)
    res = Result()
    _check(lib().dcf_select(a.dtype.itemsize, _ptr(c), int(cond_splat), _ptr(a), int(t_splat), _ptr(b),
                            int(f_splat), n, _ptr(out), ctypes.byref(res)))
    return Fold(bool(res.folded), bool(res.is_splat), int(res.first_fail_index), out)


def transpose(x: np.ndarray, shape, perms, out: np.ndarray | None = None) -> Fold:
    """Permute a dense row-major tensor (elements of x's itemsize)."""
    a = np.ascontiguousarray(x).reshape(-1)
    rank = len(shape)
    if out is None:
        out = np.empty_like(a)
    sh = (ctypes.c_int64 * rank)(*shape)
    pm = (ctypes.c_int64 * rank)(*perms)
    res = Result()
    _check(lib().dcf_transpose(a.dtype.itemsize, rank, sh, pm, _ptr(a), _ptr(out), ctypes.byref(res)))
    out_shape = [shape[p] for p in perms]
    return Fold(bool(res.folded), bool(res.is_splat), int(res.first_fail_index), out.reshape(out_shape))


def hex_encode(data) -> bytes:
    a = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else \
        np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    out = np.empty(2 * len(a), dtype=np.uint8)
    _check(lib().dcf_hex_encode(_ptr(a), len(a), _ptr(out)))
    return out.tobytes()


def hex_decode(text) -> bytes:
    t = text.encode() if isinstance(text, str) else bytes(text)
    a = np.frombuffer(t, dtype=np.uint8)
    out = np.empty(len(a) // 2, dtype=np.uint8)
    _check(lib().dcf_hex_decode(_ptr(a), len(a), _ptr(out)))
    return out.tobytes()


def splat_check(x) -> bool:
    a = np.ascontiguousarray(x).reshape(-1)
    v = ctypes.c_int(0)
    _check(lib().dcf_splat_check(_ptr(a), a.dtype.itemsize, len(a), ctypes.byref(v)))
    return bool(v.value)


def batch(jobs: list[dict]) -> list[Fold]:
    """Run independent folds in one launch per (op, dtype) group per GPU.

    Each job dict: op, dtype, [out_dtype], lhs, [rhs], [lhs_splat], [rhs_splat], [n], [flags].
    """
    arr = (Job * len(jobs))()
    keep = []
    outs = []
    for i, j in enumerate(jobs):
        op, dt = j["op"], j["dtype"]
        odt = j.get("out_dtype") or ("i1" if op in BOOL_RESULT_OPS else dt)
        l = as_storage(j["lhs"], dt)
        r = as_storage(j["rhs"], dt) if "rhs" in j else None
        n = j.get("n") or max(len(l), len(r) if r is not None else 0)
        o = np.empty(n, dtype=storage(odt))
        keep += [l, r]
        outs.append(o)
        arr[i].op, arr[i].dtype, arr[i].out_dtype = OPS[op], DTYPES[dt], DTYPES[odt]
        arr[i].flags = j.get("flags", 0)
        arr[i].lhs = l.ctypes.data
        arr[i].rhs = r.ctypes.data if r is not None else None
        arr[i].out = o.ctypes.data
        arr[i].n = n
        arr[i].lhs_splat = int(j.get("lhs_splat", False))
        arr[i].rhs_splat = int(j.get("rhs_splat", False))
    _check(lib().dcf_batch(arr, len(jobs)))
    return [Fold(bool(arr[i].result.folded), bool(arr[i].result.is_splat), int(arr[i].result.first_fail_index),
                 outs[i]) for i in range(len(jobs))]


# ------------------------------------------------------------------ device

NOALLOC_MAX_JOBS = 1024


def batch_noalloc(jobs: list[dict], stream=None) -> list[Fold]:
    """dcf_batch_noalloc: folds on device tensors with no allocation at all.

    For callers that cannot allocate device memory while they fold (their
    allocator owns all of HBM, or they cannot afford the synchronisation of
    cudaMalloc).  Each job dict: op, dtype, [out_dtype], lhs, [rhs], out
    (torch CUDA tensors on one device), [lhs_splat], [rhs_splat], [n],
    [flags].  At most NOALLOC_MAX_JOBS jobs per call; overlapping calls on
    the GPU race on the library's one scratch array.
    """
    arr = device_jobs(jobs)
    run_device_jobs(arr, stream)
    return [Fold(bool(arr[i].result.folded), bool(arr[i].result.is_splat), int(arr[i].result.first_fail_index),
                 None) for i in range(len(jobs))]


def device_jobs(jobs: list[dict]):
    """The ctypes job table of batch_noalloc, built once so that a caller can
    run the same batch repeatedly (run_device_jobs)."""
    arr = (Job * len(jobs))()
    for i, j in enumerate(jobs):
        op, dt = j["op"], j["dtype"]
        odt = j.get("out_dtype") or ("i1" if op in BOOL_RESULT_OPS else dt)
        arr[i].op, arr[i].dtype, arr[i].out_dtype = OPS[op], DTYPES[dt], DTYPES[odt]
        arr[i].flags = j.get("flags", 0)
        arr[i].lhs = _tptr(j["lhs"])
        arr[i].rhs = _tptr(j["rhs"]) if "rhs" in j else None
        arr[i].out = _tptr(j["out"])
        arr[i].n = j.get("n") or j["out"].numel()
        arr[i].lhs_splat = int(j.get("lhs_splat", False))
        arr[i].rhs_splat = int(j.get("rhs_splat", False))
    return arr


def run_device_jobs(arr, stream=None) -> None:
    """dcf_batch_noalloc on a table from device_jobs; results land in it."""
    _check(lib().dcf_batch_noalloc(arr, len(arr), _stream(stream)))

def _tptr(t) -> int:
    return t.data_ptr()


def _stream(stream) -> int:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


def status_reset(status, stream=None) -> None:
    _check(lib().dcf_status_reset_async(_tptr(status), _stream(stream)))


def binary_async(op: str, dtype: str, lhs, rhs, out, status, *, n: int | None = None, lhs_splat: bool = False,
                 rhs_splat: bool = False, flags: int = 0, stream=None) -> None:
    """Launch a binary fold on device tensors (no synchronisation)."""
    if n is None:
        n = out.numel()
    _check(lib().dcf_binary_async(OPS[op], DTYPES[dtype], _tptr(lhs), int(lhs_splat), _tptr(rhs), int(rhs_splat), n,
                                  flags, _tptr(out), _tptr(status), _stream(stream)))


def convert_async(op: str, from_dtype: str, to_dtype: str, x, out, status, *, n: int | None = None,
                  splat: bool = False, flags: int = 0, stream=None) -> None:
    if n is None:
        n = out.numel()
    _check(lib().dcf_convert_async(OPS[op], DTYPES[from_dtype], DTYPES[to_dtype], _tptr(x), int(splat), n, flags,
                                   _tptr(out), _tptr(status), _stream(stream)))


def reciprocal_async(dtype: str, x, out, status, *, n: int | None = None, splat: bool = False, flags: int = 0,
                     stream=None) -> None:
    if n is None:
        n = out.numel()
    _check(lib().dcf_reciprocal_async(DTYPES[dtype], _tptr(x), int(splat), n, flags, _tptr(out), _tptr(status),
                                      _stream(stream)))


def select_async(cond, t, f, out, status, *, n: int | None = None, cond_splat: bool = False, t_splat: bool = False,
                 f_splat: bool = False, stream=None) -> None:
    if n is None:
        n = out.numel()
    _check(lib().dcf_select_async(out.element_size(), _tptr(cond), int(cond_splat), _tptr(t), int(t_splat), _tptr(f),
                                  int(f_splat), n, _tptr(out), _tptr(status), _stream(stream)))


def permute_async(elem_size: int, shape, perms, x, out, status, stream=None) -> None:
    """dcf_permute_status_async on device tensors (2-byte transposes take the
    bulk-tensor kernel)."""
    rank = len(shape)
    sh = (ctypes.c_int64 * rank)(*shape)
    pm = (ctypes.c_int64 * rank)(*perms)
    _check(lib().dcf_permute_status_async(elem_size, rank, sh, pm, _tptr(x), _tptr(out), _tptr(status),
                                          _stream(stream)))


def transpose2d_async(elem_size: int, rows: int, cols: int, x, out, stream=None) -> None:
    _check(lib().dcf_transpose2d_async(elem_size, rows, cols, _tptr(x), _tptr(out), _stream(stream)))


def hex_encode_async(x, nbytes: int, out, stream=None) -> None:
    _check(lib().dcf_hex_encode_async(_tptr(x), nbytes, _tptr(out), _stream(stream)))


def hex_decode_async(x, nchars: int, out, status, stream=None) -> None:
    _check(lib().dcf_hex_decode_async(_tptr(x), nchars, _tptr(out), _tptr(status), _stream(stream)))


def status_read(status, stream=None) -> Fold:
    res = Result()
    _check(lib().dcf_status_read(_tptr(status), _stream(stream), ctypes.byref(res)))
    return Fold(bool(res.folded), bool(res.is_splat), int(res.first_fail_index), None)
